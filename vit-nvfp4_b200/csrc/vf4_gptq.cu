// GPTQ column loop for NVFP4 weights on the GPU (reference: src/vit_nvfp4/ptq/gptq.py:101-122).
//
// GPTQ quantizes a weight W (N x K) one input column at a time and feeds each column's
// quantization error, weighted by the upper Cholesky factor Hinv of the inverse Hessian, into
// the columns not yet quantized.  The reference runs it as a Python loop of torch ops per column
// inside 128-column blocks, with a GEMM between blocks.  The rows of W are independent within a
// block (every row sees the same Hinv), so this kernel gives each row to one warp: lane l holds
// the row's columns l, l + 32, l + 64, l + 96 of the block in registers, the block's Hinv sits in
// shared memory, and per column i
//     w_i      <- the owner lane's register (warp shuffle)
//     code     =  E2M1 code of w_i / s_b          (s_b = e4m3 block scale * global, frozen)
//     q        =  value(code) * s_b
//     err_i    =  (w_i - q) / Hinv[i][i]
//     w_c      -= err_i * Hinv[i][c]             for every later column c of the block
// with the reference's roundings (correctly rounded division, the product rounded before the
// subtraction: no fused multiply-add).  The row's error vector goes to `err` for the host's
// cross-block GEMM (W[:, i2:] -= Err @ Hinv[i1:i2, i2:]); the output code is the reference's
// final re-encoding, the E2M1 code of q / s_b.  Given the same W block, Hinv and scales the
// codes and errors are bit-identical to the reference's.
#include "vf4_common.cuh"
#include "vf4_host.h"

namespace vf4 {

constexpr int kGptqWarps = 8;
constexpr int kGptqMaxCols = 128;

__global__ void __launch_bounds__(kGptqWarps * 32)
    gptq_block_kernel(const float* __restrict__ w, int64_t ldw, const float* __restrict__ hinv, int64_t ldh,
                      const uint8_t* __restrict__ bscale, int64_t ldb, const float* __restrict__ gs, int N, int col0,
                      int count, uint8_t* __restrict__ codes, int64_t ldc, float* __restrict__ err, int64_t lde) {
  extern __shared__ float hs[];   // [count][count]: this block's Hinv
  for (int idx = threadIdx.x; idx < count * count; idx += blockDim.x) {
    const int i = idx / count, c = idx - i * count;
    hs[idx] = hinv[(int64_t)i * ldh + c];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float g = *gs;
  const int nblk = count / 16;
  for (int n = blockIdx.x * kGptqWarps + warp; n < N; n += gridDim.x * kGptqWarps) {
    float wv[4], ev[4];
    uint32_t cv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = 32 * k + lane;
      wv[k] = c < count ? w[(int64_t)n * ldw + c] : 0.f;
      ev[k] = 0.f;
      cv[k] = 0u;
    }
    // decode scale of 16-column block b of this range, held by lane b
    const float sv = lane < nblk ? __fmul_rn(e4m3_to_f32(bscale[(int64_t)n * ldb + col0 / 16 + lane]), g) : 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (32 * k < count) {
        for (int l = 0; l < 32 && 32 * k + l < count; ++l) {
          const int i = 32 * k + l;
          const float wi = __shfl_sync(0xffffffffu, wv[k], l);
          const float s = __shfl_sync(0xffffffffu, sv, i >> 4);
          const float q = __fmul_rn(e2m1_value(e2m1_code(__fdiv_rn(wi, s))), s);
          const float e = __fdiv_rn(__fsub_rn(wi, q), hs[i * count + i]);
          if (lane == l) {
            ev[k] = e;
            cv[k] = e2m1_code(__fdiv_rn(q, s));
          }
#pragma unroll
          for (int k2 = k; k2 < 4; ++k2) {
            const int c = 32 * k2 + lane;
            if (c > i && c < count) wv[k2] = __fsub_rn(wv[k2], __fmul_rn(e, hs[i * count + c]));
          }
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = 32 * k + lane;
      if (c < count) {
        codes[(int64_t)n * ldc + col0 + c] = (uint8_t)cv[k];
        err[(int64_t)n * lde + c] = ev[k];
      }
    }
  }
}

}  // namespace vf4

using namespace vf4;

extern "C" int vf4_gptq_block(const float* w, int64_t ldw, const float* hinv, int64_t ldh, const uint8_t* block_scale,
                              int64_t ldb, const float* global_scale, int64_t N, int64_t col0, int64_t count,
                              uint8_t* codes, int64_t ldc, float* err, int64_t lde, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (!w || !hinv || !block_scale || !global_scale || !codes || !err) return fail(VF4_ERR_ARG, "vf4_gptq_block: null pointer");
  if (N <= 0 || N > INT32_MAX || count <= 0 || count > kGptqMaxCols || count % 16 != 0 || col0 < 0 || col0 % 16 != 0 ||
      col0 > INT32_MAX - count)
    return fail(VF4_ERR_ARG, "vf4_gptq_block: needs N >= 1, 16 <= count <= 128 and col0 multiples of 16");
  if (ldw < count || ldh < count || ldb < (col0 + count) / 16 || ldc < col0 + count || lde < count)
    return fail(VF4_ERR_ARG, "vf4_gptq_block: leading dimension smaller than the block");
  const int smem = (int)(count * count * sizeof(float));
  if (int st = smem_optin(gptq_block_kernel, smem)) return st;
  const int64_t need = (N + kGptqWarps - 1) / kGptqWarps;
  const int grid = (int)(need < 4 * num_sms() ? need : 4 * num_sms());
  gptq_block_kernel<<<grid, kGptqWarps * 32, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      w, ldw, hinv, ldh, block_scale, ldb, global_scale, (int)N, (int)col0, (int)count, codes, ldc, err, lde);
  return launch_status("vf4_gptq_block");
}
