// Token embedding of the ViT forward: the patch unfold ahead of the patch-projection GEMM and the
// class-token / position-embedding assembly after it.  timm's PatchEmbed runs a strided Conv2d,
// then the model concatenates the class token and adds the position embedding
// (torch.cat + add: two full passes over the (B, T, d) activations).  Here the unfold writes the
// GEMM operand with its K padded to a multiple of 8 (16-byte rows, which cuBLAS needs for its
// sm_100 kernels: with K = 588 it falls back to a much slower kernel), and one pass writes
// x = [cls + pos_0; y + pos_1..] with the same bf16 roundings as cat + add.
#include "vf4_common.cuh"
#include "vf4_host.h"

namespace vf4 {

// One CTA per (image, row of patches): the C * p image rows of that patch row are staged in shared
// memory with 16-byte loads, then the gw patches are written as rows of Kp bf16 values, K = C p p
// in (c, i, j) order (the flattening of the Conv2d weight (d, C, p, p)), zeros in [K, Kp).
__global__ void __launch_bounds__(256) patchify_kernel(const __nv_bfloat16* __restrict__ img, int C, int Hh, int Ww,
                                                       int p, int Kp, __nv_bfloat16* __restrict__ out) {
  extern __shared__ __align__(16) __nv_bfloat16 rows[];   // [C][p][Ww]
  const int gh = Hh / p, gw = Ww / p;
  const int b = blockIdx.x / gh, gy = blockIdx.x - b * gh;
  const int vec_per_row = Ww / 8;
  for (int i = threadIdx.x; i < C * p * vec_per_row; i += blockDim.x) {
    const int row = i / vec_per_row, v = i - row * vec_per_row;
    const int c = row / p, r = row - c * p;
    const uint4* src = reinterpret_cast<const uint4*>(img + (((int64_t)b * C + c) * Hh + gy * p + r) * Ww) + v;
    reinterpret_cast<uint4*>(rows + (int64_t)row * Ww)[v] = __ldg(src);
  }
  __syncthreads();
  const int K = C * p * p, pp = p * p;
  const int per_patch = Kp / 8;   // 16-byte output chunks per patch row
  __nv_bfloat16* dst = out + ((int64_t)b * gh + gy) * gw * Kp;
  for (int i = threadIdx.x; i < gw * per_patch; i += blockDim.x) {
    const int gx = i / per_patch, k0 = (i - gx * per_patch) * 8;
    __align__(16) __nv_bfloat16 v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + e;
      if (k < K) {
        const int c = k / pp, rem = k - c * pp, r = rem / p, j = rem - r * p;
        v[e] = rows[(c * p + r) * Ww + gx * p + j];
      } else {
        v[e] = __float2bfloat16_rn(0.f);
      }
    }
    *reinterpret_cast<uint4*>(dst + (int64_t)gx * Kp + k0) = *reinterpret_cast<const uint4*>(v);
  }
}

// x[b, 0, :] = cls + pos[0, :], x[b, 1 + t, :] = y[b, t, :] + pos[1 + t, :]; 8 bf16 per thread
__global__ void __launch_bounds__(256) embed_tokens_kernel(const __nv_bfloat16* __restrict__ y,
                                                           const __nv_bfloat16* __restrict__ cls,
                                                           const __nv_bfloat16* __restrict__ pos, int64_t B, int T,
                                                           int D, __nv_bfloat16* __restrict__ x) {
  const int dv = D / 8;
  const int64_t total = B * T * dv;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t bt = i / dv;
    const int v = (int)(i - bt * dv);
    const int t = (int)(bt % T);
    const int64_t b = bt / T;
    const uint4 a = t == 0 ? __ldg(reinterpret_cast<const uint4*>(cls) + v)
                           : __ldg(reinterpret_cast<const uint4*>(y + ((b * (T - 1) + t - 1) * (int64_t)D)) + v);
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(pos + (int64_t)t * D) + v);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, qw[4] = {q.x, q.y, q.z, q.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o[e] = bf16x2_round(add_f32x2(bf16x2_to_f32x2(aw[e]), bf16x2_to_f32x2(qw[e])));
    reinterpret_cast<uint4*>(x + bt * D)[v] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace vf4

using namespace vf4;

extern "C" {

int vf4_patchify(const void* images, int64_t B, int64_t C, int64_t H, int64_t W, int64_t p, int64_t k_pad,
                 void* out, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (B <= 0 || C <= 0 || p <= 0 || H % p || W % p || W % 8 || k_pad < C * p * p || k_pad % 8)
    return fail(VF4_ERR_ARG, "vf4_patchify: bad sizes (B=%lld C=%lld H=%lld W=%lld p=%lld k_pad=%lld)", (long long)B,
                (long long)C, (long long)H, (long long)W, (long long)p, (long long)k_pad);
  if (!images || !out || !aligned16(images) || !aligned16(out))
    return fail(VF4_ERR_ALIGN, "vf4_patchify: 16-byte aligned pointers needed");
  const int64_t smem = C * p * W * 2;
  if (smem > 200 * 1024) return fail(VF4_ERR_UNSUPPORTED, "vf4_patchify: a row of patches needs %lld bytes", (long long)smem);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (smem > 48 * 1024) {
    if (int st = smem_optin(patchify_kernel, (int)smem)) return st;
  }
  patchify_kernel<<<(unsigned)(B * (H / p)), 256, (size_t)smem, s>>>(static_cast<const __nv_bfloat16*>(images),
                                                                     (int)C, (int)H, (int)W, (int)p, (int)k_pad,
                                                                     static_cast<__nv_bfloat16*>(out));
  return launch_status("vf4_patchify");
}

int vf4_embed_tokens(const void* y, const void* cls, const void* pos, int64_t B, int64_t T, int64_t D, void* x,
                     vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (B <= 0 || T <= 1 || D <= 0 || D % 8) return fail(VF4_ERR_ARG, "vf4_embed_tokens: bad sizes");
  if (!y || !cls || !pos || !x || !aligned16(y) || !aligned16(cls) || !aligned16(pos) || !aligned16(x))
    return fail(VF4_ERR_ALIGN, "vf4_embed_tokens: 16-byte aligned pointers needed");
  const int64_t work = B * T * (D / 8);
  int64_t grid = (work + 255) / 256;
  if (grid > (int64_t)num_sms() * 16) grid = (int64_t)num_sms() * 16;
  embed_tokens_kernel<<<(unsigned)grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), static_cast<const __nv_bfloat16*>(cls),
      static_cast<const __nv_bfloat16*>(pos), B, (int)T, (int)D, static_cast<__nv_bfloat16*>(x));
  return launch_status("vf4_embed_tokens");
}

}  // extern "C"
