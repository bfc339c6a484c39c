// NVFP4 cast family: amax reduction, global scale, the bit-exact block quantizer
// (RTN "six" / Four-Over-Six "mse", optional bias + GELU), and the pack / swizzle helpers.
//
// Reference semantics (Dev-Jahn/vit-nvfp4): src/vit_nvfp4/nvfp4/quant.py:6-69,
// format.py:17-25, pack.py:4-58, triton_cast.py:138-370 (the GELU-fused cast).
//
// The cast is HBM-bound: one thread quantizes one 16-element block (two 16-byte loads for
// bf16), writes its 8 packed bytes, and each aligned group of four lanes merges its four
// E4M3 scale bytes into one 32-bit store of the 128x4-tiled scale layout.
#include "vf4_common.cuh"
#include "vf4_host.h"

namespace vf4 {

static __device__ int g_cast_err;

int cast_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_cast_err, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_cast_err, &z, sizeof(int));
  }
  return v;
}

template <typename T>
VF4_DEV float to_f32(T v);
template <>
VF4_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
VF4_DEV float to_f32<float>(float v) {
  return v;
}

// Load 16 consecutive elements (16-byte aligned) as fp32.
template <typename T>
VF4_DEV void load16(const T* p, float* v);
template <>
VF4_DEV void load16<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
  uint4 a = __ldg(q), b = __ldg(q + 1);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
VF4_DEV void load16<float>(const float* p, float* v) {
  const float4* q = reinterpret_cast<const float4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4 a = __ldg(q + i);
    v[4 * i] = a.x;
    v[4 * i + 1] = a.y;
    v[4 * i + 2] = a.z;
    v[4 * i + 3] = a.w;
  }
}

template <typename T, bool kGelu, bool kBias>
VF4_DEV void prologue16(float* v, const T* bias, int64_t col0) {
  if constexpr (kBias) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = v[i] + to_f32<T>(bias[col0 + i]);
  }
  if constexpr (kGelu) {
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = gelu_erf(v[i]);
  }
}

// ---------------------------------------------------------------------------------------
// amax over a (rows, K) matrix of stride ld; K % 16 == 0, 16-byte aligned rows.
// ---------------------------------------------------------------------------------------
template <typename T, bool kGelu, bool kBias>
__global__ void __launch_bounds__(256) amax_rows_kernel(const T* __restrict__ x, int64_t rows,
                                                        int64_t K, int64_t ld,
                                                        const T* __restrict__ bias,
                                                        float* __restrict__ out) {
  const int64_t nb = K / 16;
  const int64_t total = rows * nb;
  float m = 0.f;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = t / nb, b = t - r * nb;
    float v[16];
    load16<T>(x + r * ld + b * 16, v);
    prologue16<T, kGelu, kBias>(v, bias, b * 16);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = fmaxf(m, fabsf(v[i]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __shared__ float red[8];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(m));
  }
}

// Generic flat amax (any n, any alignment) — scalar loads.
template <typename T, bool kGelu>
__global__ void __launch_bounds__(256) amax_flat_kernel(const T* __restrict__ x, int64_t n,
                                                        float* __restrict__ out) {
  float m = 0.f;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < n;
       t += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f32<T>(x[t]);
    if constexpr (kGelu) v = gelu_erf(v);
    m = fmaxf(m, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(m));
}

__global__ void global_scale_kernel(const float* amax, float denom, float* gs) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *gs = __fdiv_rn(fmaxf(*amax, 1e-12f), denom);
}

// ---------------------------------------------------------------------------------------
// The cast.  Thread t covers block (row, blk) of the padded (ceil128(M), ceil4(K/16)) grid;
// threads outside (M, K/16) only contribute zero scale bytes to the padding.
// ---------------------------------------------------------------------------------------
template <typename T, bool kMse, bool kGelu, bool kBias>
__global__ void __launch_bounds__(256) cast_kernel(const T* __restrict__ x, int64_t M, int64_t K,
                                                   int64_t ld, const float* __restrict__ gs_ptr,
                                                   const T* __restrict__ bias,
                                                   uint8_t* __restrict__ out_packed,
                                                   uint8_t* __restrict__ sf_swz,
                                                   uint8_t* __restrict__ sf_lin) {
  const int64_t nb = K / 16;
  const int64_t nb4 = (nb + 3) & ~int64_t(3);
  const int64_t ncb = nb4 >> 2;
  const int64_t Mp = (M + 127) & ~int64_t(127);
  const int64_t total = Mp * nb4;
  const float gs = *gs_ptr;
  const float s_enc = __fdiv_rn(1.0f, gs);
  const int lane = threadIdx.x & 31;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t0 = blockIdx.x * (int64_t)blockDim.x + (threadIdx.x & ~31); t0 < total;
       t0 += stride) {
    const int64_t t = t0 + lane;
    const int64_t row = t / nb4;
    const int64_t blk = t - row * nb4;
    const bool in_grid = t < total;
    const bool valid = in_grid && row < M && blk < nb;
    uint32_t sf = 0;
    if (valid) {
      float v[16];
      load16<T>(x + row * ld + blk * 16, v);
      prologue16<T, kGelu, kBias>(v, bias, blk * 16);
      BlockQ q = quantize_block<kMse>(v, gs, s_enc);
      *reinterpret_cast<uint64_t*>(out_packed + row * (K / 2) + blk * 8) = q.packed;
      sf = q.sf;
      if (sf_lin) sf_lin[row * nb + blk] = (uint8_t)sf;
    }
    // merge the 4 scale bytes of an aligned lane quad (same row, blk%4 = 0..3)
    uint32_t w = sf << (8 * (blk & 3));
    w |= __shfl_xor_sync(0xffffffffu, w, 1);
    w |= __shfl_xor_sync(0xffffffffu, w, 2);
    if (sf_swz && in_grid && (blk & 3) == 0) {
      int64_t off = ((row >> 7) * ncb + (blk >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4;
      *reinterpret_cast<uint32_t*>(sf_swz + off) = w;
    }
  }
}

__global__ void pack_kernel(const uint8_t* __restrict__ codes, int64_t n_out,
                            uint8_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_out;
       i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (uint8_t)((codes[2 * i + 1] << 4) | codes[2 * i]);
}

__global__ void unpack_kernel(const uint8_t* __restrict__ packed, int64_t n_in,
                              uint8_t* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n_in;
       i += (int64_t)gridDim.x * blockDim.x) {
    uint8_t b = packed[i];
    out[2 * i] = b & 0xF;
    out[2 * i + 1] = (b >> 4) & 0xF;
  }
}

__global__ void to_blocked_kernel(const uint8_t* __restrict__ sf, int64_t R, int64_t C,
                                  uint8_t* __restrict__ out) {
  const int64_t ncb = (C + 3) / 4;
  const int64_t Rp = (R + 127) & ~int64_t(127);
  const int64_t total = Rp * ncb;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i / ncb, cb = i - r * ncb;
    uint32_t w = 0;
    if (r < R) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int64_t c = cb * 4 + j;
        if (c < C) w |= (uint32_t)sf[r * C + c] << (8 * j);
      }
    }
    int64_t off = ((r >> 7) * ncb + cb) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4;
    *reinterpret_cast<uint32_t*>(out + off) = w;
  }
}

static int grid_for(int64_t work, int per_block = 256) {
  int64_t b = (work + per_block - 1) / per_block;
  int64_t cap = (int64_t)num_sms() * 16;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

template <typename T, bool kGelu, bool kBias>
static void launch_amax_rows(const void* x, int64_t rows, int64_t K, int64_t ld, const void* bias,
                             float* out, cudaStream_t s) {
  amax_rows_kernel<T, kGelu, kBias><<<grid_for(rows * (K / 16)), 256, 0, s>>>(
      static_cast<const T*>(x), rows, K, ld, static_cast<const T*>(bias), out);
}

template <typename T, bool kMse, bool kGelu, bool kBias>
static void launch_cast(const void* x, int64_t M, int64_t K, int64_t ld, const float* gs,
                        const void* bias, uint8_t* op, uint8_t* sfs, uint8_t* sfl, cudaStream_t s) {
  int64_t nb4 = ((K / 16) + 3) & ~int64_t(3);
  int64_t Mp = (M + 127) & ~int64_t(127);
  cast_kernel<T, kMse, kGelu, kBias><<<grid_for(Mp * nb4), 256, 0, s>>>(
      static_cast<const T*>(x), M, K, ld, gs, static_cast<const T*>(bias), op, sfs, sfl);
}

template <typename T>
static void dispatch_amax(const void* x, int64_t M, int64_t K, int64_t ld, int gelu,
                          const void* bias, float* out, cudaStream_t s) {
  if (gelu && bias) launch_amax_rows<T, true, true>(x, M, K, ld, bias, out, s);
  else if (gelu) launch_amax_rows<T, true, false>(x, M, K, ld, bias, out, s);
  else if (bias) launch_amax_rows<T, false, true>(x, M, K, ld, bias, out, s);
  else launch_amax_rows<T, false, false>(x, M, K, ld, bias, out, s);
}

template <typename T>
static void dispatch_cast(const void* x, int64_t M, int64_t K, int64_t ld, const float* gs, int mse,
                          int gelu, const void* bias, uint8_t* op, uint8_t* sfs, uint8_t* sfl,
                          cudaStream_t s) {
#define VF4_CAST_CASE(MS, GE, BI)                                                       \
  if (!!mse == MS && !!gelu == GE && !!(bias != nullptr) == BI) {                       \
    launch_cast<T, MS, GE, BI>(x, M, K, ld, gs, bias, op, sfs, sfl, s);                 \
    return;                                                                             \
  }
  VF4_CAST_CASE(false, false, false)
  VF4_CAST_CASE(false, false, true)
  VF4_CAST_CASE(false, true, false)
  VF4_CAST_CASE(false, true, true)
  VF4_CAST_CASE(true, false, false)
  VF4_CAST_CASE(true, false, true)
  VF4_CAST_CASE(true, true, false)
  VF4_CAST_CASE(true, true, true)
#undef VF4_CAST_CASE
}

}  // namespace vf4

using namespace vf4;

extern "C" {

int vf4_amax(const void* x, int dtype, int64_t n, int gelu, float* amax_out, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (!amax_out || n < 0 || (n > 0 && !x)) return fail(VF4_ERR_ARG, "vf4_amax: bad arguments");
  if (dtype != VF4_BF16 && dtype != VF4_F32) return fail(VF4_ERR_ARG, "vf4_amax: bad dtype %d", dtype);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(amax_out, 0, sizeof(float), s) != cudaSuccess)
    return fail(VF4_ERR_CUDA, "vf4_amax: memset failed");
  if (n == 0) return VF4_OK;
  if (n % 16 == 0 && aligned16(x)) {
    if (dtype == VF4_BF16) dispatch_amax<__nv_bfloat16>(x, 1, n, n, gelu, nullptr, amax_out, s);
    else dispatch_amax<float>(x, 1, n, n, gelu, nullptr, amax_out, s);
  } else {
    int g = grid_for(n);
    if (dtype == VF4_BF16) {
      if (gelu) amax_flat_kernel<__nv_bfloat16, true><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n, amax_out);
      else amax_flat_kernel<__nv_bfloat16, false><<<g, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(x), n, amax_out);
    } else {
      if (gelu) amax_flat_kernel<float, true><<<g, 256, 0, s>>>(static_cast<const float*>(x), n, amax_out);
      else amax_flat_kernel<float, false><<<g, 256, 0, s>>>(static_cast<const float*>(x), n, amax_out);
    }
  }
  return launch_status("vf4_amax");
}

int vf4_global_scale(const float* amax, int block_select, float* gs_out, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (!amax || !gs_out) return fail(VF4_ERR_ARG, "vf4_global_scale: null pointer");
  if (block_select != VF4_SIX && block_select != VF4_MSE)
    return fail(VF4_ERR_ARG, "vf4_global_scale: bad block_select %d", block_select);
  float denom = block_select == VF4_MSE ? 6.f * 256.f : 6.f * 448.f;
  global_scale_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(amax, denom, gs_out);
  return launch_status("vf4_global_scale");
}

int vf4_cast_nvfp4(const void* x, int dtype, int64_t M, int64_t K, int64_t ld, const float* gs,
                   int block_select, int gelu, const void* bias, uint8_t* out_packed,
                   uint8_t* out_sf_swizzled, uint8_t* out_sf_linear, float* gs_out,
                   vf4_stream_t stream) {
  if (int st = check_device()) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (dtype != VF4_BF16 && dtype != VF4_F32) return fail(VF4_ERR_ARG, "vf4_cast_nvfp4: bad dtype %d", dtype);
  if (block_select != VF4_SIX && block_select != VF4_MSE)
    return fail(VF4_ERR_ARG, "vf4_cast_nvfp4: bad block_select %d", block_select);
  if (M < 0 || K <= 0 || K % 16 != 0 || ld < K)
    return fail(VF4_ERR_ARG, "vf4_cast_nvfp4: need M>=0, K>0, K%%16==0, ld>=K (M=%lld K=%lld ld=%lld)",
                (long long)M, (long long)K, (long long)ld);
  if (!gs && !gs_out) return fail(VF4_ERR_ARG, "vf4_cast_nvfp4: gs and gs_out both NULL");
  if (M > 0 && (!x || !out_packed)) return fail(VF4_ERR_ARG, "vf4_cast_nvfp4: null input/output");
  const int64_t esz = dtype == VF4_BF16 ? 2 : 4;
  if (M > 0 && (!aligned16(x) || (ld * esz) % 16 != 0))
    return fail(VF4_ERR_ALIGN, "vf4_cast_nvfp4: x must be 16-byte aligned with ld*elem %% 16 == 0");
  if ((reinterpret_cast<uintptr_t>(out_packed) & 7u) || (reinterpret_cast<uintptr_t>(out_sf_swizzled) & 3u))
    return fail(VF4_ERR_ALIGN, "vf4_cast_nvfp4: out_packed must be 8-byte, out_sf 4-byte aligned");
  const float* use_gs = gs;
  if (!gs) {
    if (cudaMemsetAsync(gs_out, 0, sizeof(float), s) != cudaSuccess)
      return fail(VF4_ERR_CUDA, "vf4_cast_nvfp4: memset failed");
    if (M > 0) {
      if (dtype == VF4_BF16) dispatch_amax<__nv_bfloat16>(x, M, K, ld, gelu, bias, gs_out, s);
      else dispatch_amax<float>(x, M, K, ld, gelu, bias, gs_out, s);
    }
    float denom = block_select == VF4_MSE ? 6.f * 256.f : 6.f * 448.f;
    global_scale_kernel<<<1, 32, 0, s>>>(gs_out, denom, gs_out);
    use_gs = gs_out;
  } else if (gs_out && gs_out != gs) {
    if (cudaMemcpyAsync(gs_out, gs, sizeof(float), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return fail(VF4_ERR_CUDA, "vf4_cast_nvfp4: gs copy failed");
  }
  if (M == 0) return launch_status("vf4_cast_nvfp4");
  if (dtype == VF4_BF16)
    dispatch_cast<__nv_bfloat16>(x, M, K, ld, use_gs, block_select == VF4_MSE, gelu, bias, out_packed,
                                 out_sf_swizzled, out_sf_linear, s);
  else
    dispatch_cast<float>(x, M, K, ld, use_gs, block_select == VF4_MSE, gelu, bias, out_packed,
                         out_sf_swizzled, out_sf_linear, s);
  return launch_status("vf4_cast_nvfp4");
}

int vf4_pack_e2m1(const uint8_t* codes, int64_t rows, int64_t K, uint8_t* out, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (rows < 0 || K < 0 || K % 2 || (rows * K > 0 && (!codes || !out)))
    return fail(VF4_ERR_ARG, "vf4_pack_e2m1: bad arguments");
  int64_t n = rows * K / 2;
  if (n == 0) return VF4_OK;
  pack_kernel<<<grid_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(codes, n, out);
  return launch_status("vf4_pack_e2m1");
}

int vf4_unpack_e2m1(const uint8_t* packed, int64_t rows, int64_t Kh, uint8_t* out,
                    vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (rows < 0 || Kh < 0 || (rows * Kh > 0 && (!packed || !out)))
    return fail(VF4_ERR_ARG, "vf4_unpack_e2m1: bad arguments");
  int64_t n = rows * Kh;
  if (n == 0) return VF4_OK;
  unpack_kernel<<<grid_for(n), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(packed, n, out);
  return launch_status("vf4_unpack_e2m1");
}

int vf4_to_blocked(const uint8_t* sf, int64_t R, int64_t C, uint8_t* out, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (R < 0 || C < 0 || (R * C > 0 && (!sf || !out)) || (reinterpret_cast<uintptr_t>(out) & 3u))
    return fail(VF4_ERR_ARG, "vf4_to_blocked: bad arguments");
  if (R == 0 || C == 0) return VF4_OK;
  int64_t total = ((R + 127) & ~int64_t(127)) * ((C + 3) / 4);
  to_blocked_kernel<<<grid_for(total), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(sf, R, C, out);
  return launch_status("vf4_to_blocked");
}

}  // extern "C"
