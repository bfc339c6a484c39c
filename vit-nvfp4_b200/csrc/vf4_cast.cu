// NVFP4 cast family: amax reduction, global scale, the bit-exact block quantizer
// (RTN "six" / Four-Over-Six "mse", optional bias + GELU), and the pack / swizzle helpers.
//
// Reference semantics (Dev-Jahn/vit-nvfp4): src/vit_nvfp4/nvfp4/quant.py:6-69,
// format.py:17-25, pack.py:4-58, triton_cast.py:138-370 (the GELU-fused cast).
//
// The cast is HBM-bound: one thread quantizes one 16-element block (two 16-byte loads for
// bf16), writes its 8 packed bytes, and each aligned group of four lanes merges its four
// E4M3 scale bytes into one 32-bit store of the 128x4-tiled scale layout.
#include <type_traits>

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

// 16 elements held as raw 16-byte words (2 for bf16, 4 for fp32): a block loaded one iteration
// ahead of its use, so a thread's next load is in flight while it encodes the current block.
template <typename T>
struct Raw16 {
  uint4 w[sizeof(T)];
};

template <typename T>
VF4_DEV void load_raw16(const T* p, Raw16<T>& r) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < (int)sizeof(T); ++i) r.w[i] = __ldg(q + i);
}

template <typename T>
VF4_DEV void raw16_to_f32(const Raw16<T>& r, float* v) {
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint32_t w[4] = {r.w[i].x, r.w[i].y, r.w[i].z, r.w[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * i + 2 * j] = __uint_as_float(w[j] << 16);
        v[8 * i + 2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[4 * i] = __uint_as_float(r.w[i].x);
      v[4 * i + 1] = __uint_as_float(r.w[i].y);
      v[4 * i + 2] = __uint_as_float(r.w[i].z);
      v[4 * i + 3] = __uint_as_float(r.w[i].w);
    }
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
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float m = 0.f;
  int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  // (row, block) of t, advanced by the grid stride without dividing
  const int64_t d_r = stride / nb, d_b = stride - d_r * nb;
  int64_t r = t / nb, b = t - r * nb;
  Raw16<T> raw;
  if (t < total) load_raw16<T>(x + r * ld + b * 16, raw);
  for (; t < total; t += stride) {   // each block's load is issued one iteration ahead
    const Raw16<T> cur = raw;
    const int64_t bc = b;
    r += d_r;
    b += d_b;
    if (b >= nb) {
      b -= nb;
      ++r;
    }
    if (t + stride < total) load_raw16<T>(x + r * ld + b * 16, raw);
    float v[16];
    raw16_to_f32<T>(cur, v);
    prologue16<T, kGelu, kBias>(v, bias, bc * 16);
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
    // GELU of a bf16 tensor is a bf16 tensor in the reference (F.gelu keeps the dtype): round the
    // maximum once (rounding is monotone, so this is the max of the rounded values)
    if constexpr (kGelu && sizeof(T) == 2) m = bf16_round(m);
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
  if constexpr (kGelu && sizeof(T) == 2) m = bf16_round(m);
  if ((threadIdx.x & 31) == 0) atomicMax(reinterpret_cast<unsigned int*>(out), __float_as_uint(m));
}

__global__ void global_scale_kernel(const float* amax, float denom, float* gs) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *gs = __fdiv_rn(fmaxf(*amax, 1e-12f), denom);
}

// ---------------------------------------------------------------------------------------
// The cast.  Thread t covers block (row, blk) of the padded (ceil128(M), ceil4(K/16)) grid;
// threads outside (M, K/16) only contribute zero scale bytes to the padding.
// ---------------------------------------------------------------------------------------
template <typename T, bool kGelu, bool kBias>
constexpr bool kBf16Exact = std::is_same<T, __nv_bfloat16>::value && !kGelu && !kBias;

// I: the index type, int32_t when every flat index and element offset of the call fits (the
// launcher checks), else int64_t; 32-bit index arithmetic takes about a tenth of the kernel's
// instructions off.
template <typename T, bool kMse, bool kGelu, bool kBias, typename I = int64_t>
__global__ void __launch_bounds__(256) cast_kernel(const T* __restrict__ x, int64_t M_, int64_t K_,
                                                   int64_t ld_, const float* __restrict__ gs_ptr,
                                                   const T* __restrict__ bias,
                                                   uint8_t* __restrict__ out_packed,
                                                   uint8_t* __restrict__ sf_swz,
                                                   uint8_t* __restrict__ sf_lin) {
  const I M = (I)M_, K = (I)K_, ld = (I)ld_;
  // six rule: {dec, lo, hi} of every scale byte (scale_entry), looked up per block
  __shared__ float4 s_q[kMse ? 1 : 128];
  if constexpr (!kMse) {
    const float gsv = *gs_ptr;
    for (int i = threadIdx.x; i < 128; i += blockDim.x) s_q[i] = scale_entry((uint32_t)i, gsv);
    __syncthreads();
  }
  const I nb = K / 16;
  const I nb4 = (nb + 3) & ~I(3);
  const I ncb = nb4 >> 2;
  const I Mp = (M + 127) & ~I(127);
  const I total = Mp * nb4;
  const float gs = *gs_ptr;
  const float s_enc = __fdiv_rn(1.0f, gs);
  const int lane = threadIdx.x & 31;
  const I stride = (I)gridDim.x * (I)blockDim.x;
  // (row, blk) of this thread's flat index, advanced by the grid stride without dividing
  const I t_first = (I)blockIdx.x * (I)blockDim.x + (I)threadIdx.x;
  const I d_row = stride / nb4, d_blk = stride - d_row * nb4;
  I row = t_first / nb4, blk = t_first - row * nb4;
  Raw16<T> raw;
  if (t_first < total && row < M && blk < nb) load_raw16<T>(x + row * ld + blk * 16, raw);
  for (I t0 = t_first - lane; t0 < total; t0 += stride) {
    const I t = t0 + lane;
    const bool in_grid = t < total;
    const bool valid = in_grid && row < M && blk < nb;
    const Raw16<T> cur = raw;
    // the next item of this thread, loaded now and used in the next iteration
    I nrow = row + d_row, nblk = blk + d_blk;
    if (nblk >= nb4) {
      nblk -= nb4;
      ++nrow;
    }
    if (t + stride < total && nrow < M && nblk < nb) load_raw16<T>(x + nrow * ld + nblk * 16, raw);
    uint32_t sf = 0;
    if (valid) {
      float v[16];
      raw16_to_f32<T>(cur, v);
      prologue16<T, kGelu, kBias>(v, bias, blk * 16);
      // bf16 inputs are >= 2^-133 in magnitude when non-zero (see encode16_bracket)
      constexpr float dec_max = kBf16Exact<T, kGelu, kBias> ? 0x1p17f : 2.0f;
      uint64_t packed;
      if constexpr (kMse) {
        const BlockQ q = quantize_block<kMse>(v, gs, s_enc, dec_max);
        packed = q.packed;
        sf = q.sf;
      } else {   // quantize_block's six rule with the table
        sf = six_code(amax16(v), s_enc);
        packed = encode16_bracket_q(v, s_q[sf], dec_max);
      }
      *reinterpret_cast<uint64_t*>(out_packed + row * (K / 2) + blk * 8) = packed;
      if (sf_lin) sf_lin[row * nb + blk] = (uint8_t)sf;
    }
    // merge the 4 scale bytes of an aligned lane quad (same row, blk%4 = 0..3)
    uint32_t w = sf << (8 * (blk & 3));
    w |= __shfl_xor_sync(0xffffffffu, w, 1);
    w |= __shfl_xor_sync(0xffffffffu, w, 2);
    if (sf_swz && in_grid && (blk & 3) == 0) {
      const I off = ((row >> 7) * ncb + (blk >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4;
      *reinterpret_cast<uint32_t*>(sf_swz + off) = w;
    }
    row = nrow;
    blk = nblk;
  }
}

// Cast of row groups into interleaved rows of one NVFP4 operand: input row t of group g
// (x + (g * rows_in + t) * K, bf16, groups contiguous) becomes output row g * rows_out + row_off + t.
// Same per-block arithmetic as cast_kernel (six rule, exact encoder); the scale bytes of an aligned
// lane quad merge into one word of the to_blocked layout.  Padding rows are not touched here.
__global__ void __launch_bounds__(256) cast_rows_kernel(const __nv_bfloat16* __restrict__ x, int64_t rows_total,
                                                        int64_t rows_in, int64_t K, const float* __restrict__ gs_ptr,
                                                        int64_t rows_out, int64_t row_off,
                                                        uint8_t* __restrict__ out_packed, uint8_t* __restrict__ sf_swz) {
  // 32-bit indices (the entry point checks rows_total * K / 16 < 2^31); (row, blk) advanced by the
  // grid stride without dividing, one 32-bit division per item for the row's group
  const uint32_t nb = (uint32_t)(K / 16);
  const uint32_t ncb = nb >> 2;
  const uint32_t total = (uint32_t)rows_total * nb;
  const uint32_t rin = (uint32_t)rows_in, rout = (uint32_t)rows_out, roff = (uint32_t)row_off;
  const float gs = *gs_ptr;
  const float s_enc = __fdiv_rn(1.0f, gs);
  const int lane = threadIdx.x & 31;
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t t_first = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t d_row = stride / nb, d_blk = stride - d_row * nb;
  uint32_t r = t_first / nb, blk = t_first - r * nb;
  for (uint32_t t0 = t_first - lane; t0 < total; t0 += stride) {
    const bool in_grid = t0 + lane < total;
    const uint32_t grp = r / rin;
    const int64_t orow = (int64_t)grp * rout + roff + (r - grp * rin);
    uint32_t sf = 0;
    if (in_grid) {
      float v[16];
      load16<__nv_bfloat16>(x + (int64_t)r * K + blk * 16, v);
      BlockQ q = quantize_block<false>(v, gs, s_enc, 0x1p17f);
      *reinterpret_cast<uint64_t*>(out_packed + orow * (K / 2) + blk * 8) = q.packed;
      sf = q.sf;
    }
    uint32_t w = sf << (8 * (blk & 3));
    w |= __shfl_xor_sync(0xffffffffu, w, 1);
    w |= __shfl_xor_sync(0xffffffffu, w, 2);
    if (in_grid && (blk & 3) == 0)
      *reinterpret_cast<uint32_t*>(sf_swz + ((orow >> 7) * ncb + (blk >> 2)) * 512 + (orow & 31) * 16 +
                                   ((orow >> 5) & 3) * 4) = w;
    r += d_row;
    blk += d_blk;
    if (blk >= nb) {
      blk -= nb;
      ++r;
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
  const int grid = grid_for(Mp * nb4);
  // 32-bit indices when the flat block index (plus one grid stride), the element offsets of x and
  // the byte offsets of the codes and scales all stay below 2^31 (VF4_CAST_INDEX64 set in the
  // environment keeps the 64-bit kernel, which the tests compare with the 32-bit one)
  const int64_t lim = int64_t(1) << 31;
  if (Mp * nb4 + (int64_t)grid * 256 < lim && Mp * (ld > K ? ld : K) < lim && Mp * nb4 * 16 < lim &&
      !getenv("VF4_CAST_INDEX64"))
    cast_kernel<T, kMse, kGelu, kBias, int32_t><<<grid, 256, 0, s>>>(
        static_cast<const T*>(x), M, K, ld, gs, static_cast<const T*>(bias), op, sfs, sfl);
  else
    cast_kernel<T, kMse, kGelu, kBias, int64_t><<<grid, 256, 0, s>>>(
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

// ---------------------------------------------------------------------------------------
// LayerNorm fused into the NVFP4 cast (optionally with the residual + LayerScale before it).
// One warp per row; lane l holds elements [256c + 8l, 256c + 8l + 8) of chunk c (16-byte
// loads, coalesced), so an NVFP4 block of 16 is a lane pair.  Rounding points mirror the
// unfused reference ops on bf16 tensors:  x' = bf16(x + bf16(y * gamma)),
// h = bf16((x - mean) * rstd * w + b), then the six-rule quantizer on h.
//   kMode 0: write x' (if kRes), atomically max |h| into amax_out (dynamic global scale) and
//            leave the row's {mean, rstd} in the first 8 bytes of its code row, which the
//            kMode 2 pass reads before it overwrites them with the row's codes
//   kMode 1: write x' (if kRes) and quantize h with the global scale *gs
//   kMode 2: quantize h with *gs and the row statistics left by a kMode 0 pass (no reductions)
// The kernels are issue-bound, so the parameters sit in shared memory as fp32 (no per-row
// unpacking) and the modes that reduce keep the row as fp32 pairs between the reductions.
// ---------------------------------------------------------------------------------------
VF4_DEV float bf16_bits_lo(uint32_t w) { return __uint_as_float(w << 16); }
VF4_DEV float bf16_bits_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Resident CTAs per SM (launch bound and grid) and whether the row is kept as fp32 pairs between
// the reductions; the modes that reduce keep it, at 16 warps per SM (measured at ViT-L/14 b1024:
// 24 or 32 warps with spills or re-unpacking are 2-3% slower), except the residual form at
// K > 1024, whose held row would not fit in 128 registers next to the prefetched x and y.
template <int NC, bool kRes, int kMode>
struct LnCfg {
  static constexpr int kMinBlocks = kMode == 2 ? 3 : 2;
  static constexpr bool kHold = kMode != 2 && !(kRes && NC > 4);
};

// element pair i of a lane's chunk as fp32: held, or unpacked from the raw bf16 words
template <bool kHold>
VF4_DEV unsigned long long ln_x2(const unsigned long long* vc, const uint4& xc, int i) {
  if constexpr (kHold) return vc[i];
  else return bf16x2_to_f32x2(i == 0 ? xc.x : i == 1 ? xc.y : i == 2 ? xc.z : xc.w);
}

template <int NC, bool kRes, int kMode>
__global__ void __launch_bounds__(256, (LnCfg<NC, kRes, kMode>::kMinBlocks)) ln_cast_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ gamma,
    __nv_bfloat16* __restrict__ x_out, const __nv_bfloat16* __restrict__ ln_w, const __nv_bfloat16* __restrict__ ln_b,
    float eps, int64_t M, int K, const float* __restrict__ gs_ptr, float* __restrict__ amax_out,
    uint8_t* out_packed, uint8_t* __restrict__ out_sf) {
  static_assert(!(kRes && kMode == 2), "the statistics pass runs without the residual");
  // s_wb[(4c + j) * 32 + l] = {w[e], w[e+1], b[e], b[e+1]}, e = 256c + 8l + 2j
  // s_g [(2c + j) * 32 + l] = {g[e], .., g[e+3]} as two bf16 pairs, e = 256c + 8l + 4j
  // (consecutive lanes read consecutive 16 / 8 bytes: conflict-free)
  __shared__ float4 s_wb[NC * 128];
  __shared__ uint2 s_g[kRes ? NC * 64 : 1];
  __shared__ float4 s_q[kMode != 0 ? 128 : 1];   // {dec, lo, hi} per scale byte (scale_entry)
  if constexpr (kMode != 0) {
    const float gsv = *gs_ptr;
    for (int i = threadIdx.x; i < 128; i += blockDim.x) s_q[i] = scale_entry((uint32_t)i, gsv);
  }
  for (int i = threadIdx.x; i < NC * 128; i += blockDim.x) {
    const int e = 256 * (i >> 7) + 8 * (i & 31) + 2 * ((i >> 5) & 3);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (e < K) {
      v.x = __bfloat162float(ln_w[e]);
      v.y = __bfloat162float(ln_w[e + 1]);
      v.z = __bfloat162float(ln_b[e]);
      v.w = __bfloat162float(ln_b[e + 1]);
    }
    s_wb[i] = v;
  }
  if constexpr (kRes) {
    for (int i = threadIdx.x; i < NC * 64; i += blockDim.x) {
      const int e = 256 * (i >> 6) + 8 * (i & 31) + 4 * ((i >> 5) & 1);
      uint2 v = make_uint2(0x3F803F80u, 0x3F803F80u);   // 1.0 pairs
      if (gamma && e < K) {
        const uint32_t g0 = __bfloat16_as_ushort(gamma[e]), g1 = __bfloat16_as_ushort(gamma[e + 1]),
                       g2 = __bfloat16_as_ushort(gamma[e + 2]), g3 = __bfloat16_as_ushort(gamma[e + 3]);
        v = make_uint2(g0 | (g1 << 16), g2 | (g3 << 16));
      }
      s_g[i] = v;
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp_g = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t Mp = (M + 127) & ~int64_t(127);
  const int ncb = K / 64;
  const int64_t code_ld = K / 2;
  float gs = 1.f, s_enc = 1.f;
  if constexpr (kMode != 0) {
    gs = *gs_ptr;
    s_enc = __fdiv_rn(1.0f, gs);
  }
  // Raw bf16 words (and, in kMode 2, the row statistics) of the next row are loaded while the
  // current row is processed.
  uint4 nx[NC], ny[kRes ? NC : 1];
  float2 nst = make_float2(0.f, 0.f);
  auto fetch = [&](int64_t row) {
    if (row < M) {
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int e0 = 256 * c + 8 * lane;
        if (e0 < K) {
          nx[c] = __ldg(reinterpret_cast<const uint4*>(x + row * K + e0));
          if constexpr (kRes) ny[c] = __ldg(reinterpret_cast<const uint4*>(y + row * K + e0));
        }
      }
      // the statistics share their bytes with this row's codes, which this kernel writes:
      // a coherent load, not the read-only path
      if constexpr (kMode == 2) nst = __ldcg(reinterpret_cast<const float2*>(out_packed + row * code_ld));
    }
  };
  float lane_amax = 0.f;
  fetch(warp_g);
  for (int64_t row = warp_g; row < Mp; row += nwarps) {
    uint4 cx[NC], cy[kRes ? NC : 1];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      cx[c] = nx[c];
      if constexpr (kRes) cy[c] = ny[c];
    }
    const float2 cst = nst;
    fetch(row + nwarps);
    if (row >= M) {  // zero the scale padding rows of the last 128-row tile
      if constexpr (kMode != 0) {
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const int e0 = 256 * c + 8 * lane;
          if (e0 < K && (lane & 7) == 0) {
            const int col = e0 / 16;
            *reinterpret_cast<uint32_t*>(out_sf + ((row >> 7) * ncb + (col >> 2)) * 512 + (row & 31) * 16 +
                                         ((row >> 5) & 3) * 4) = 0u;
          }
        }
      }
      continue;
    }
    float mean, rstd;
    // v: the row as fp32 pairs (after the residual step when kRes), kept between the reductions
    constexpr bool kHold = LnCfg<NC, kRes, kMode>::kHold;
    unsigned long long v[kHold ? NC : 1][4];
    if constexpr (kMode == 2) {
      mean = cst.x;
      rstd = cst.y;
      __syncwarp();   // every lane has read the statistics before any lane overwrites them
    } else {
      unsigned long long sum2 = f32x2_pack(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < NC; ++c) {
        const int e0 = 256 * c + 8 * lane;
        if (e0 < K) {
          const uint32_t xw[4] = {cx[c].x, cx[c].y, cx[c].z, cx[c].w};
          if constexpr (kRes) {
            const uint32_t yw[4] = {cy[c].x, cy[c].y, cy[c].z, cy[c].w};
            uint32_t rw[4];
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const uint2 gg = s_g[(2 * c + jj) * 32 + lane];
              const uint32_t g2[2] = {gg.x, gg.y};
#pragma unroll
              for (int t = 0; t < 2; ++t) {
                const int i = 2 * jj + t;
                // x' = bf16(x + bf16(y * gamma)) in bf16 pair arithmetic (the same roundings)
                rw[i] = add_bf16x2(xw[i], mul_bf16x2(yw[i], g2[t]));
                if constexpr (kHold) v[c][i] = bf16x2_to_f32x2(rw[i]);
              }
            }
            *reinterpret_cast<uint4*>(x_out + row * K + e0) = make_uint4(rw[0], rw[1], rw[2], rw[3]);
            if constexpr (!kHold) cx[c] = make_uint4(rw[0], rw[1], rw[2], rw[3]);   // x' replaces x
          } else if constexpr (kHold) {
#pragma unroll
            for (int i = 0; i < 4; ++i) v[c][i] = bf16x2_to_f32x2(xw[i]);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) sum2 = add_f32x2(sum2, ln_x2<kHold>(v[kHold ? c : 0], cx[c], i));
        }
      }
      float s0, s1;
      f32x2_unpack(sum2, &s0, &s1);
      float sum = s0 + s1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      mean = sum / (float)K;
      const unsigned long long nm2 = f32x2_pack(-mean, -mean);
      unsigned long long sq2 = f32x2_pack(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < NC; ++c)
        if (256 * c + 8 * lane < K) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const unsigned long long d2 = add_f32x2(ln_x2<kHold>(v[kHold ? c : 0], cx[c], i), nm2);
            sq2 = fma_f32x2(d2, d2, sq2);
          }
        }
      f32x2_unpack(sq2, &s0, &s1);
      float sq = s0 + s1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      rstd = rsqrtf(sq / (float)K + eps);
      if constexpr (kMode == 0)
        if (lane == 0) *reinterpret_cast<float2*>(out_packed + row * code_ld) = make_float2(mean, rstd);
    }
    const unsigned long long nmean2 = f32x2_pack(-mean, -mean), rstd2 = f32x2_pack(rstd, rstd);
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int e0 = 256 * c + 8 * lane;
      const bool in = e0 < K;   // warp-uniform per (c, lane group of 8) -> shuffles stay converged
      float h[8];
      float am = 0.f;
      if (in) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 wb = s_wb[(4 * c + i) * 32 + lane];
          // h = (x - mean) * rstd * w + b, rounded to bf16 (kMode 0 rounds the maximum only:
          // rounding is monotone, so max |bf16(h)| = bf16(max |h|))
          const unsigned long long hf = fma_f32x2(mul_f32x2(add_f32x2(ln_x2<kHold>(v[kHold ? c : 0], cx[c], i), nmean2), rstd2), f32x2_pack(wb.x, wb.y),
                                                  f32x2_pack(wb.z, wb.w));
          if constexpr (kMode == 0) {
            float h0, h1;
            f32x2_unpack(hf, &h0, &h1);
            am = max3f(am, fabsf(h0), fabsf(h1));
          } else {
            const uint32_t hb = bf16x2_round(hf);
            h[2 * i] = __uint_as_float(hb << 16);
            h[2 * i + 1] = __uint_as_float(hb & 0xFFFF0000u);
          }
        }
        if constexpr (kMode != 0) {
          am = max3f(fabsf(h[0]), fabsf(h[1]), fabsf(h[2]));
          am = max3f(am, fabsf(h[3]), fabsf(h[4]));
          am = max3f(am, fabsf(h[5]), fabsf(h[6]));
          am = fmaxf(am, fabsf(h[7]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) h[i] = 0.f;
      }
      if constexpr (kMode == 0) {
        lane_amax = fmaxf(lane_amax, am);
      } else {
        const float bam = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        const uint32_t sf = six_code(bam, s_enc);
        const uint32_t codes = encode8_bracket_q(h, s_q[sf], 0x1p17f);   // h is bf16-rounded
        if (in) *reinterpret_cast<uint32_t*>(out_packed + row * code_ld + e0 / 2) = codes;
        // scale bytes of SF columns 16c + 4g .. +3 live in lanes 8g, 8g+2, 8g+4, 8g+6 (a lane pair
        // holds one block's byte): each lane places its byte, two xor-shuffles OR the four together
        uint32_t w = sf << (8 * ((lane >> 1) & 3));
        w |= __shfl_xor_sync(0xffffffffu, w, 2);
        w |= __shfl_xor_sync(0xffffffffu, w, 4);
        if (in && (lane & 7) == 0) {
          const int col = e0 / 16;
          *reinterpret_cast<uint32_t*>(out_sf + ((row >> 7) * ncb + (col >> 2)) * 512 + (row & 31) * 16 +
                                       ((row >> 5) & 3) * 4) = w;
        }
      }
    }
  }
  if constexpr (kMode == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lane_amax = fmaxf(lane_amax, __shfl_xor_sync(0xffffffffu, lane_amax, o));
    lane_amax = __bfloat162float(__float2bfloat16_rn(lane_amax));
    if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(amax_out), __float_as_uint(lane_amax));
  }
}

template <int NC, bool kRes, int kMode>
static void launch_ln_one(const void* x, const void* y, const void* gamma, void* x_out, const void* w, const void* b,
                          float eps, int64_t M, int K, const float* gs, float* amax, uint8_t* op, uint8_t* sf,
                          cudaStream_t s) {
  // one resident wave: every warp walks its rows with the next row's loads in flight
  const int64_t Mp = (M + 127) & ~int64_t(127);
  const int64_t per_wave = (int64_t)num_sms() * LnCfg<NC, kRes, kMode>::kMinBlocks;
  const int64_t need = (Mp * 32 + 255) / 256;
  const int grid = (int)(need < per_wave ? (need < 1 ? 1 : need) : per_wave);
  ln_cast_kernel<NC, kRes, kMode><<<grid, 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(y),
      static_cast<const __nv_bfloat16*>(gamma), static_cast<__nv_bfloat16*>(x_out),
      static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(b), eps, M, K, gs, amax, op, sf);
}

template <int NC>
static void launch_ln(bool res, int mode, const void* x, const void* y, const void* gamma, void* x_out,
                      const void* w, const void* b, float eps, int64_t M, int K, const float* gs, float* amax,
                      uint8_t* op, uint8_t* sf, cudaStream_t s) {
  if (res && mode == 0) launch_ln_one<NC, true, 0>(x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s);
  else if (res) launch_ln_one<NC, true, 1>(x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s);
  else if (mode == 0) launch_ln_one<NC, false, 0>(x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s);
  else if (mode == 1) launch_ln_one<NC, false, 1>(x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s);
  else launch_ln_one<NC, false, 2>(x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s);
}

static void dispatch_ln(int nc, bool res, int mode, const void* x, const void* y, const void* gamma, void* x_out,
                        const void* w, const void* b, float eps, int64_t M, int K, const float* gs, float* amax,
                        uint8_t* op, uint8_t* sf, cudaStream_t s) {
  switch (nc) {
    case 1: launch_ln<1>(res, mode, x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s); break;
    case 2: launch_ln<2>(res, mode, x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s); break;
    case 3: launch_ln<3>(res, mode, x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s); break;
    case 4: launch_ln<4>(res, mode, x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s); break;
    default: launch_ln<5>(res, mode, x, y, gamma, x_out, w, b, eps, M, K, gs, amax, op, sf, s); break;
  }
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

namespace vf4 {
// Pairs of elements through the epilogue's packed erf-GELU; an odd tail element pairs with itself.
__global__ void __launch_bounds__(256) gelu_erf_kernel(const float* __restrict__ x, int64_t n,
                                                       float* __restrict__ out) {
  const int64_t pairs = (n + 1) / 2;
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < pairs; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = 2 * t;
    const float a = x[i], b = i + 1 < n ? x[i + 1] : a;
    float ga, gb;
    f32x2_unpack(gelu_erf_x2(f32x2_pack(a, b)), &ga, &gb);
    out[i] = ga;
    if (i + 1 < n) out[i + 1] = gb;
  }
}
}  // namespace vf4

int vf4_gelu_erf_f32(const float* x, int64_t n, float* out, vf4_stream_t stream) {
  if (int st = vf4::check_device()) return st;
  if (n < 0 || (n > 0 && (!x || !out))) return vf4::fail(VF4_ERR_ARG, "vf4_gelu_erf_f32: bad arguments");
  if (n == 0) return VF4_OK;
  const int64_t pairs = (n + 1) / 2;
  const int grid = (int)((pairs + 255) / 256 < 148 * 16 ? (pairs + 255) / 256 : 148 * 16);
  vf4::gelu_erf_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(x, n, out);
  return vf4::launch_status("vf4_gelu_erf_f32");
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

int vf4_ln_cast_nvfp4(const void* x, const void* y, const void* gamma, void* x_out, const void* ln_w,
                      const void* ln_b, float eps, int64_t M, int64_t K, const float* gs, uint8_t* out_packed,
                      uint8_t* out_sf, float* gs_out, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (M < 0 || K <= 0 || K % 64 != 0 || K > 1280)
    return fail(VF4_ERR_UNSUPPORTED, "vf4_ln_cast_nvfp4: need K %% 64 == 0 and K <= 1280 (K=%lld)", (long long)K);
  if (!ln_w || !ln_b || (M > 0 && (!x || !out_packed || !out_sf)) || (y && !x_out) || (!gs && !gs_out))
    return fail(VF4_ERR_ARG, "vf4_ln_cast_nvfp4: missing pointer");
  const void* ps[] = {x, y, gamma, x_out, ln_w, ln_b, out_packed, out_sf};
  for (const void* p : ps)
    if (p && !aligned16(p)) return fail(VF4_ERR_ALIGN, "vf4_ln_cast_nvfp4: pointers must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int nc = (int)((K + 255) / 256);
  const bool res = y != nullptr;
  if (gs) {
    if (gs_out && gs_out != gs && cudaMemcpyAsync(gs_out, gs, 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return fail(VF4_ERR_CUDA, "vf4_ln_cast_nvfp4: gs copy failed");
    dispatch_ln(nc, res, 1, x, y, gamma, x_out, ln_w, ln_b, eps, M, (int)K, gs, nullptr, out_packed, out_sf, s);
    return launch_status("vf4_ln_cast_nvfp4");
  }
  // dynamic global scale: pass 1 (residual write + amax of the normalised rows), scale, pass 2
  if (cudaMemsetAsync(gs_out, 0, 4, s) != cudaSuccess) return fail(VF4_ERR_CUDA, "vf4_ln_cast_nvfp4: memset");
  // (pass 1 leaves each row's mean and rstd in its code row for pass 2)
  dispatch_ln(nc, res, 0, x, y, gamma, x_out, ln_w, ln_b, eps, M, (int)K, nullptr, gs_out, out_packed, nullptr, s);
  global_scale_kernel<<<1, 32, 0, s>>>(gs_out, 6.f * 448.f, gs_out);
  dispatch_ln(nc, false, 2, res ? x_out : x, nullptr, nullptr, nullptr, ln_w, ln_b, eps, M, (int)K, gs_out, nullptr,
              out_packed, out_sf, s);
  return launch_status("vf4_ln_cast_nvfp4");
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

int vf4_cast_nvfp4_split(const void* x_main, int64_t rows_main, const void* x_tail, int64_t rows_tail,
                         int64_t n_img, int64_t K, const float* gs, float* gs_out, uint8_t* out_packed,
                         uint8_t* out_sf_swizzled, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (n_img <= 0 || rows_main <= 0 || rows_tail <= 0 || K <= 0 || K % 64 != 0 ||
      n_img * (rows_main + rows_tail) * (K / 16) + 1024ll * 256 >= (1ll << 31))
    return fail(VF4_ERR_ARG, "vf4_cast_nvfp4_split: bad sizes (n=%lld main=%lld tail=%lld K=%lld)", (long long)n_img,
                (long long)rows_main, (long long)rows_tail, (long long)K);
  if (!x_main || !x_tail || !out_packed || !out_sf_swizzled || (!gs && !gs_out))
    return fail(VF4_ERR_ARG, "vf4_cast_nvfp4_split: null pointer");
  if (!aligned16(x_main) || !aligned16(x_tail) || (reinterpret_cast<uintptr_t>(out_packed) & 7u) ||
      (reinterpret_cast<uintptr_t>(out_sf_swizzled) & 3u))
    return fail(VF4_ERR_ALIGN, "vf4_cast_nvfp4_split: misaligned pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const float* use_gs = gs;
  if (!gs) {   // dynamic global over both parts
    if (cudaMemsetAsync(gs_out, 0, sizeof(float), s) != cudaSuccess)
      return fail(VF4_ERR_CUDA, "vf4_cast_nvfp4_split: memset failed");
    dispatch_amax<__nv_bfloat16>(x_main, n_img * rows_main, K, K, 0, nullptr, gs_out, s);
    dispatch_amax<__nv_bfloat16>(x_tail, n_img * rows_tail, K, K, 0, nullptr, gs_out, s);
    global_scale_kernel<<<1, 32, 0, s>>>(gs_out, 6.f * 448.f, gs_out);
    use_gs = gs_out;
  } else if (gs_out && gs_out != gs) {
    if (cudaMemcpyAsync(gs_out, gs, sizeof(float), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
      return fail(VF4_ERR_CUDA, "vf4_cast_nvfp4_split: gs copy failed");
  }
  const int64_t rows_out = rows_main + rows_tail, M = n_img * rows_out;
  const int64_t ncb = K / 64;
  if (M % 128) {   // scale words of the last row block's padding rows stay zero
    if (cudaMemsetAsync(out_sf_swizzled + (M / 128) * ncb * 512, 0, (size_t)ncb * 512, s) != cudaSuccess)
      return fail(VF4_ERR_CUDA, "vf4_cast_nvfp4_split: memset failed");
  }
  const int64_t nb4 = K / 16;
  cast_rows_kernel<<<grid_for(n_img * rows_main * nb4), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x_main), n_img * rows_main, rows_main, K, use_gs, rows_out, 0, out_packed,
      out_sf_swizzled);
  cast_rows_kernel<<<grid_for(n_img * rows_tail * nb4), 256, 0, s>>>(
      static_cast<const __nv_bfloat16*>(x_tail), n_img * rows_tail, rows_tail, K, use_gs, rows_out, rows_main,
      out_packed, out_sf_swizzled);
  return launch_status("vf4_cast_nvfp4_split");
}

}  // extern "C"
