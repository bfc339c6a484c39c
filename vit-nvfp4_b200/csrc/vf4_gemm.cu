// Block-scaled NVFP4 GEMM on sm_100a tensor cores (tcgen05.mma kind::mxf4nvf4).
//
//   D[m, n] = gs_a * gs_b * sum_k A[m, k] * B[n, k]      (E2M1 operands, UE4M3 scales / 16)
//
// Replaces torch._scaled_mm_v2 (BlockWise1x16 + TensorWise) used by the reference in
// src/vit_nvfp4/nvfp4/backends/torch_scaled_mm.py:14-46, and fuses the bias add
// (gemm.py:36-37) and the fc1 "+b1 -> GELU -> NVFP4 cast" step (fused_mlp.py:47-51).
//
// Structure (persistent, one CTA per SM, 320 threads):
//   warp 0      TMA producer: A/B tiles (128-byte swizzle) + the tile's 512-byte scale atoms
//               (plain bulk copies: the operand scale layout is already the MMA's layout)
//   warp 1      TMEM allocator and MMA issuer: tcgen05.cp scale atoms -> TMEM, one
//               tcgen05.mma per K=64 block, tcgen05.commit releases smem stages / hands
//               the accumulator to the epilogue
//   warps 2..9  epilogue: tcgen05.ld the 128 x BN fp32 accumulator (two warps per TMEM lane
//               quadrant, each half of the columns), release TMEM, then scale / bias /
//               GELU / NVFP4-quantize from registers and store
// Every wait is bounded (mbar_wait); a timeout records a device error and unwinds.
#include <stdlib.h>
#include <string.h>

#include "vf4_common.cuh"
#include "vf4_host.h"

namespace vf4 {

static __device__ int g_gemm_err;

int gemm_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_gemm_err, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_gemm_err, &z, sizeof(int));
  }
  return v;
}

// Self-test of the bounded waits every kernel uses: one thread waits on an mbarrier of its own that
// nothing ever arrives on, with the caller's limit instead of the production one.  The wait must
// give up, record kDevErrTimeoutFull in this file's error word and let the kernel return.
__global__ void wait_selftest_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_limit(smem_u32(&bar), 0, &g_gemm_err, kDevErrTimeoutFull, limit_ns);
}

__host__ __device__ constexpr bool epi_gelu(int e) { return e == VF4_EPI_GELU_NVFP4 || e == VF4_EPI_GELU_ERF_NVFP4; }

// The bf16 epilogues of the 128x256 tile stage 32 rows x 16 columns (1 KB) per warp so that a
// fourth pipeline stage fits; the GELU epilogue keeps 3 stages (its staging is 2 KB per warp) and
// the fp32 epilogue stores directly.
// With a B scale image (kRepB: the 128x256 tile and a caller-built image, vf4_b_scale_image) the
// stage holds B's scale atoms four times over -- per K64 block [atom of rows 0-127 x4][atom of rows
// 128-255 x4], 4 KB, one bulk copy of the image per stage -- so that one 128x256b tcgen05.cp (lane l
// reads row l: atom row l % 32 of each half) fills the 8 scale columns the MMA reads, where two
// 32x128b.warpx4 copies were needed: each copy costs the tensor pipe 25-45 clocks whatever its
// size.  That region leads the stage (a 16 KB block at its 1024-byte-aligned start); it costs the
// fourth stage, which measured no faster than three.
template <int BN, int EPI = VF4_EPI_BIAS, bool kF32 = false, bool REP = false>
struct GemmCfg {
  static constexpr bool kGeluEpi = EPI == VF4_EPI_GELU_NVFP4 || EPI == VF4_EPI_GELU_ERF_NVFP4;
  static constexpr int BM = 128;
  static constexpr int KB_PER_STAGE = 4;                   // 4 x K64 MMAs = 256 elements = 128 B
  static constexpr bool kRepB = REP && BN == 256;
  static constexpr int STAGES = kRepB ? 3 : BN == 256 ? (kGeluEpi ? 3 : 4) : 4;
  static constexpr int EPI_CW = BN == 256 ? 16 : 64;        // bf16 staging chunk (columns)
  static constexpr int A_BYTES = BM * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int SFA_BYTES = KB_PER_STAGE * 512;
  static constexpr int SFB_BYTES = kRepB ? KB_PER_STAGE * 4096 : (BN / 128) * KB_PER_STAGE * 512;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  // offsets inside a stage (A and B 1024-byte aligned for the 128-byte swizzle)
  static constexpr int SFB_OFF = kRepB ? 0 : A_BYTES + B_BYTES + SFA_BYTES;
  static constexpr int A_OFF = kRepB ? SFB_BYTES : 0;
  static constexpr int B_OFF = A_OFF + A_BYTES;
  static constexpr int SFA_OFF = B_OFF + B_BYTES;
  static constexpr int ACC_STAGES = BN == 256 ? 1 : 2;
  static constexpr int SFA_TCOL = 256;                      // TMEM columns of the scale slots
  static constexpr int SFA_SLOT = KB_PER_STAGE * 4;         // 4 columns per K64 block (M=128)
  static constexpr int SFB_TCOL = SFA_TCOL + 2 * SFA_SLOT;
  static constexpr int SFB_PER_KB = BN / 32;                // 4 (N=128) or 8 (N=256) columns
  static constexpr int SFB_SLOT = KB_PER_STAGE * SFB_PER_KB;
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 320;
  static constexpr int EPI_WARP_BYTES = kGeluEpi ? 32 * BN / 4 : (kF32 ? 0 : 32 * EPI_CW * 2);
  static constexpr int EPI_BYTES = 8 * EPI_WARP_BYTES;
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 2 * ACC_STAGES + 1) + 16;
  static constexpr int CONST_OFF = (STAGES * STAGE_BYTES + EPI_BYTES + BAR_BYTES + 15) / 16 * 16;
  static constexpr int CONST_BYTES = kGeluEpi ? 512 : 0;   // GELU: the scale reciprocal table
  static constexpr int SMEM = 1024 + CONST_OFF + CONST_BYTES;
  static_assert(ACC_STAGES * BN <= SFA_TCOL, "accumulators overlap the scale slots");
  static_assert(SFB_TCOL + 2 * SFB_SLOT <= TMEM_COLS, "TMEM overflow");
  static_assert(STAGE_BYTES % 1024 == 0, "stage must keep 1024-byte alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

struct GemmParams {
  const uint8_t* a_sf;
  const uint8_t* b_sf;
  const uint8_t* b_img;   // B scale image (vf4_b_scale_image) or NULL
  const float* a_gs;
  const float* b_gs;
  int M, N, K;
  int n_kb;     // ceil(K / 64): K64 blocks == scale column-blocks of A and B
  int n_rb_b;   // ceil(N / 128): scale row-blocks of B
  int n_rb_a;   // ceil(M / 128): scale row-blocks of A
  int tiles_m, tiles_n;
  const __nv_bfloat16* bias;
  void* out;
  const float* epi_gs;
  uint8_t* out_packed;
  uint8_t* out_sf;
  int out_ncb;  // scale column-blocks of the NVFP4 output (N / 64)
  const __nv_bfloat16* res;     // VF4_EPI_BIAS_RESIDUAL: residual (M, N) and LayerScale (N,) or NULL
  const __nv_bfloat16* gamma;
};

VF4_DEV float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
VF4_DEV float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// The multiplier that takes a GELU value to E2M1 units for every E4M3 scale byte b of the
// GELU-NVFP4 epilogue: RN(s_enc / e4m3(b)) with s_enc = RN(1 / gs), the "total scale" of the
// reference's fused Triton cast (nvfp4/triton_cast.py:327-330, global_scale = 1 / per_tensor_scale
// at :163); filled by the epilogue threads et = 0..127 before their first tile.
VF4_DEV void fill_rcp_tab(float* tab, int et, float s_enc) {
  if (et >= 0 && et < 128) tab[et] = __fdiv_rn(s_enc, e4m3_to_f32((uint32_t)et));
}

// NVFP4 "six" cast and store of one warp's 32-row slab of GELU outputs: row row0 + lane, columns
// [col0, col0 + NC); make_h(blk, col, h) writes the 16 fp32 values of the slab's block blk (columns
// col .. col + 15).  The cast is the Triton cast's arithmetic (triton_cast.py:318-340): block scale
// e4m3(min(RN(amax / 6) * s_enc, 448)), values times rcp_tab[scale byte] = RN(s_enc / scale),
// nearest-even E2M1.  Packed codes (NC/2 bytes per row) are staged in shared memory with the 64-byte
// (NC = 128) or 32-byte (NC = 64) swizzle, so a warp's 16-byte stores spread over all banks, and
// stored by TMA; the 4-byte scale words go straight to the 128x4-tiled layout.
template <int NC, class MakeH>
VF4_DEV void nvfp4_slab_store(MakeH&& make_h, const GemmParams& p, const CUtensorMap* tmOut, int row0, int col0,
                              int lane, float esenc, uint32_t ebuf, uint8_t* ebuf_g, const float* rcp_tab) {
  const int64_t row = (int64_t)row0 + lane;
  if (lane == 0) bulk_wait_read();
  __syncwarp();
#pragma unroll
  for (int g4 = 0; g4 < NC / 64; ++g4) {
    uint32_t sfw = 0;
    uint64_t pk[4];
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int blk = g4 * 4 + b;
      const int col = col0 + blk * 16;
      uint64_t packed = 0;
      if (col < p.N) {
        float h[16];
        make_h(blk, col, h);
        const float bs_f = fminf(__fmul_rn(div6_rn(fmaxf(amax16(h), 1e-12f)), esenc), 448.f);
        const uint32_t sf = f32_to_e4m3(bs_f);
        packed = encode16_inv(h, rcp_tab[sf], sf == 0u);
        if (row < p.M) sfw |= sf << (8 * b);
      }
      pk[b] = packed;
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int c = g4 * 2 + hh;   // 16-byte chunk of the row
      const int cs = NC == 128 ? (c ^ ((lane >> 1) & 3)) : (c ^ ((lane >> 2) & 1));
      *reinterpret_cast<uint4*>(ebuf_g + lane * (NC / 2) + (cs << 4)) =
          make_uint4((uint32_t)pk[2 * hh], (uint32_t)(pk[2 * hh] >> 32), (uint32_t)pk[2 * hh + 1],
                     (uint32_t)(pk[2 * hh + 1] >> 32));
    }
    const int c0 = (col0 >> 4) + g4 * 4;  // first scale column of this group (multiple of 4)
    if (col0 + g4 * 64 < p.N && row < (((int64_t)p.M + 127) & ~int64_t(127))) {
      int64_t off = ((row >> 7) * p.out_ncb + (c0 >> 2)) * 512 + (row & 31) * 16 + ((row >> 5) & 3) * 4;
      *reinterpret_cast<uint32_t*>(p.out_sf + off) = sfw;  // rows >= M write the zero padding
    }
  }
  fence_async_shared();
  __syncwarp();
  if (lane == 0 && col0 < p.N) {
    tma_store_2d(tmOut, ebuf, col0 / 2, row0);
    bulk_commit();
  }
}

// Epilogue for one warp's 32-row slab of a tile: v holds this lane's NC accumulator columns
// [col0, col0 + NC) of row row0 + lane; ebuf is the warp's 4 KB staging buffer.
template <int NC, int EPI, bool kF32, int CW = 64>
VF4_DEV void epilogue_slab(const uint32_t* v, const GemmParams& p, const CUtensorMap* tmOut, int row0,
                           int col0, int lane, float alpha, float egs, float esenc, uint32_t ebuf,
                           uint8_t* ebuf_g, const float* rcp_tab = nullptr, const float* bias_f = nullptr) {
  const int64_t row = (int64_t)row0 + lane;
  if constexpr (!epi_gelu(EPI) && kF32) {
    if (row < p.M) {
#pragma unroll
      for (int g = 0; g < NC / 8; ++g) {
        const int col = col0 + g * 8;
        if (col < p.N) {
          float y[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) y[i] = __uint_as_float(v[g * 8 + i]) * alpha;
          if (EPI == VF4_EPI_BIAS && p.bias) {
            uint4 bw = __ldg(reinterpret_cast<const uint4*>(p.bias + col));
            const uint32_t b4[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              y[2 * i] += __uint_as_float(b4[i] << 16);
              y[2 * i + 1] += __uint_as_float(b4[i] & 0xFFFF0000u);
            }
          }
          float4* o = reinterpret_cast<float4*>(static_cast<float*>(p.out) + row * p.N + col);
          o[0] = make_float4(y[0], y[1], y[2], y[3]);
          o[1] = make_float4(y[4], y[5], y[6], y[7]);
        }
      }
    }
  } else if constexpr (!epi_gelu(EPI)) {
    // bf16 out: each CW-column chunk of the warp's 32x(NC) slab is staged in shared memory with
    // the 2*CW-byte swizzle (16-byte piece j of row r at j ^ (r%8) for 128-byte rows, j ^ ((r/2)%4)
    // for 64-byte rows, j ^ ((r/4)%2) for 32-byte rows) and written by one TMA store
#pragma unroll
    for (int c = 0; c < NC / CW; ++c) {
      const int colc = col0 + c * CW;
      if (colc < p.N) {
        if (lane == 0) bulk_wait_read();      // the previous store has left the buffer
        __syncwarp();
#pragma unroll
        for (int j = 0; j < CW / 8; ++j) {
          const int col = colc + j * 8;
          // bf16 pair arithmetic with the reference's roundings: RN(acc * alpha) (the bf16 GEMM
          // output), + b in bf16, then for the residual form RN(y * gamma) and RN(x + that); each
          // bf16 pair op rounds the exact result once, as torch's bf16 ops do (fp32 op, one rounding)
          const unsigned long long alpha2 = f32x2_pack(alpha, alpha);
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = bf16x2_round(mul_f32x2(f32x2_pack(__uint_as_float(v[c * CW + j * 8 + 2 * i]),
                                                     __uint_as_float(v[c * CW + j * 8 + 2 * i + 1])), alpha2));
          if (EPI != VF4_EPI_NONE && p.bias && col < p.N) {
            const uint4 bw = __ldg(reinterpret_cast<const uint4*>(p.bias + col));
            const uint32_t b4[4] = {bw.x, bw.y, bw.z, bw.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = add_bf16x2(w[i], b4[i]);
          }
          if constexpr (EPI == VF4_EPI_BIAS_RESIDUAL) {
            // x + ls(y); this lane's 8 residual values are 16 contiguous bytes of its row
            uint4 rw = make_uint4(0, 0, 0, 0);
            if (row < p.M && col < p.N) rw = *reinterpret_cast<const uint4*>(p.res + row * p.N + col);
            const uint32_t r4[4] = {rw.x, rw.y, rw.z, rw.w};
            uint32_t g4[4] = {0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u};   // 1.0 pairs
            if (p.gamma && col < p.N) {
              const uint4 gw = __ldg(reinterpret_cast<const uint4*>(p.gamma + col));
              g4[0] = gw.x; g4[1] = gw.y; g4[2] = gw.z; g4[3] = gw.w;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) w[i] = add_bf16x2(r4[i], mul_bf16x2(w[i], g4[i]));
          }
          const int js = CW == 64 ? (j ^ (lane & 7)) : CW == 32 ? (j ^ ((lane >> 1) & 3)) : (j ^ ((lane >> 2) & 1));
          *reinterpret_cast<uint4*>(ebuf_g + lane * (2 * CW) + js * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(tmOut, ebuf, colc, row0);   // rows >= M and columns >= N are clipped
          bulk_commit();
        }
      }
    }
  } else {
    // GELU -> NVFP4 "six" cast of the fc1 output (fused_mlp.py:47-51).
    //  * VF4_EPI_GELU_ERF_NVFP4 follows the reference's steps: the GEMM result rounded to bf16,
    //    + b1 in bf16 (gemm_packed's bf16 output, then y1 + b1), erf-GELU in fp32 on that bf16
    //    value (the Triton cast's apply_gelu, triton_cast.py:302-303), then the cast.
    //  * VF4_EPI_GELU_NVFP4: fp32 acc * gs_a * gs_b + b1 without roundings, tanh-form GELU.
    // Element pairs go through the packed fp32 ops (fma / mul.rn.f32x2, the scalar ops' roundings);
    // bias_f, when the caller staged the bias in shared memory, holds fp32 values (tanh form) or
    // bf16 pairs (erf form).
    const unsigned long long alpha2 = f32x2_pack(alpha, alpha);
    nvfp4_slab_store<NC>(
        [&](int blk, int col, float* h) {
          if constexpr (EPI == VF4_EPI_GELU_ERF_NVFP4) {
            uint32_t bw[8];
            const bool has_bias = p.bias != nullptr;
            if (bias_f) {
              const uint4* bp = reinterpret_cast<const uint4*>(bias_f) + blk * 2;
              const uint4 b0 = bp[0], b1 = bp[1];
              bw[0] = b0.x; bw[1] = b0.y; bw[2] = b0.z; bw[3] = b0.w;
              bw[4] = b1.x; bw[5] = b1.y; bw[6] = b1.z; bw[7] = b1.w;
            } else if (has_bias) {
              const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col);
              const uint4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
              bw[0] = b0.x; bw[1] = b0.y; bw[2] = b0.z; bw[3] = b0.w;
              bw[4] = b1.x; bw[5] = b1.y; bw[6] = b1.z; bw[7] = b1.w;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              uint32_t y1 = bf16x2_round(mul_f32x2(
                  f32x2_pack(__uint_as_float(v[blk * 16 + 2 * i]), __uint_as_float(v[blk * 16 + 2 * i + 1])), alpha2));
              if (has_bias) y1 = add_bf16x2(y1, bw[i]);
              f32x2_unpack(gelu_erf_x2(bf16x2_to_f32x2(y1)), &h[2 * i], &h[2 * i + 1]);
            }
          } else {
            unsigned long long t2[8];
            if (bias_f) {
              const float4* bp = reinterpret_cast<const float4*>(bias_f + blk * 16);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float4 bb = bp[i];
                t2[2 * i] = f32x2_pack(bb.x, bb.y);
                t2[2 * i + 1] = f32x2_pack(bb.z, bb.w);
              }
            } else if (p.bias) {
              const uint4* bp = reinterpret_cast<const uint4*>(p.bias + col);
              uint4 b0 = __ldg(bp), b1 = __ldg(bp + 1);
              const uint32_t bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
              for (int i = 0; i < 8; ++i) t2[i] = bf16x2_to_f32x2(bw[i]);
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) t2[i] = 0ull;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const unsigned long long a2 = fma_f32x2(
                  f32x2_pack(__uint_as_float(v[blk * 16 + 2 * i]), __uint_as_float(v[blk * 16 + 2 * i + 1])), alpha2,
                  t2[i]);
              f32x2_unpack(gelu_tanh_x2(a2), &h[2 * i], &h[2 * i + 1]);
            }
          }
        },
        p, tmOut, row0, col0, lane, esenc, ebuf, ebuf_g, rcp_tab);
  }
}

template <int BN, int EPI, bool kF32, bool REP>
__global__ void __launch_bounds__(320, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmOut, const GemmParams p) {
  using C = GemmCfg<BN, EPI, kF32, REP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t epi0 = base + C::STAGES * C::STAGE_BYTES;   // epilogue staging buffers
  const uint32_t bar0 = epi0 + C::EPI_BYTES;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + C::ACC_STAGES + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * C::STAGES + 2 * C::ACC_STAGES);
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(gbase + C::STAGES * C::STAGE_BYTES + C::EPI_BYTES +
                                  8 * (2 * C::STAGES + 2 * C::ACC_STAGES + 1));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = &g_gemm_err;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < C::ACC_STAGES; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);
    }
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
    if (!kF32) tma_prefetch(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  const int tiles = p.tiles_m * p.tiles_n;
  const int n_st = (p.n_kb + C::KB_PER_STAGE - 1) / C::KB_PER_STAGE;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const int mb = tile / p.tiles_n, nb = tile - mb * p.tiles_n;
        for (int st = 0; st < n_st; ++st, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int kb0 = st * C::KB_PER_STAGE;
          const int nkb = min(C::KB_PER_STAGE, p.n_kb - kb0);
          const uint32_t sf_bytes = (uint32_t)nkb * 512u;
          mbar_arrive_expect_tx(full_bar(s), C::A_BYTES + C::B_BYTES + sf_bytes * (1 + (C::kRepB ? 8 : BN / 128)));
          const uint32_t stg = base + s * C::STAGE_BYTES;
          const uint32_t sa = stg + C::A_OFF, sb = stg + C::B_OFF, ssfa = stg + C::SFA_OFF, ssfb = stg + C::SFB_OFF;
          tma_load_2d(sa, &tmA, st * 128, mb * 128, full_bar(s));
          tma_load_2d(sb, &tmB, st * 128, nb * BN, full_bar(s));
          bulk_load(ssfa, p.a_sf + ((int64_t)mb * p.n_kb + kb0) * 512, sf_bytes, full_bar(s));
#pragma unroll
          for (int j = 0; j < BN / 128; ++j) {
            int rb = nb * (BN / 128) + j;
            if (rb >= p.n_rb_b) rb = nb * (BN / 128);  // N tail: finite stand-in, columns discarded
            if constexpr (C::kRepB) {   // the image's [kb][half][copy][512 B] blocks of this N tile
              if (j == 0)
                bulk_load(ssfb, p.b_img + ((int64_t)nb * p.n_kb + kb0) * 4096, (uint32_t)nkb * 4096u, full_bar(s));
            } else {
              bulk_load(ssfb + j * C::KB_PER_STAGE * 512, p.b_sf + ((int64_t)rb * p.n_kb + kb0) * 512, sf_bytes,
                        full_bar(s));
            }
          }
        }
      }
      // wait (bounded) for our own copies still in flight before the CTA can retire
      for (int k = it - C::STAGES < 0 ? 0 : it - C::STAGES; k < it; ++k)
        mbar_wait(full_bar(k % C::STAGES), (uint32_t)(k / C::STAGES) & 1u, err, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_mxf4nvf4(BN);
    int it = 0, lt = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++lt) {
      const int acc = lt % C::ACC_STAGES;
      const uint32_t aph = (uint32_t)(lt / C::ACC_STAGES) & 1u;
      if (!mbar_wait(tempty_bar(acc), aph ^ 1u, err, kDevErrTimeoutTmem)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + (uint32_t)(acc * BN);
      for (int st = 0; st < n_st; ++st, ++it) {
        const int s = it % C::STAGES;
        const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
        if (!mbar_wait(full_bar(s), ph, err, kDevErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const int nkb = min(C::KB_PER_STAGE, p.n_kb - st * C::KB_PER_STAGE);
          const uint32_t slot = (uint32_t)(it & 1);
          const uint32_t sfa_t = tmem + C::SFA_TCOL + slot * C::SFA_SLOT;
          const uint32_t sfb_t = tmem + C::SFB_TCOL + slot * C::SFB_SLOT;
          const uint32_t stg = base + s * C::STAGE_BYTES;
          const uint32_t sa = stg + C::A_OFF, sb = stg + C::B_OFF, ssfa = stg + C::SFA_OFF, ssfb = stg + C::SFB_OFF;
          // scale copies of K-block kb are issued right before its MMA (the tensor pipe runs
          // copies and MMAs in issue order; interleaving lets the copies overlap earlier MMAs)
          for (int kb = 0; kb < nkb; ++kb) {
            tmem_cp_32x128b_x4(sfa_t + kb * 4, smem_desc(ssfa + kb * 512, 0, 128, 0));
            if constexpr (C::kRepB) {
              // 128 rows of 32 bytes: the two 16-byte halves 2048 bytes apart, 8-row groups 128 apart
              tmem_cp_128x256b(sfb_t + kb * C::SFB_PER_KB, smem_desc(ssfb + kb * 4096, 2048, 128, 0));
            } else {
#pragma unroll
              for (int j = 0; j < BN / 128; ++j)
                tmem_cp_32x128b_x4(sfb_t + kb * C::SFB_PER_KB + j * 4,
                                   smem_desc(ssfb + j * C::KB_PER_STAGE * 512 + kb * 512, 0, 128, 0));
            }
            const uint64_t ad = smem_desc(sa + kb * 32, 16, 1024, 2);
            const uint64_t bd = smem_desc(sb + kb * 32, 16, 1024, 2);
            mma_mxf4nvf4(d_tmem, ad, bd, idesc, sfa_t + kb * 4, sfb_t + kb * C::SFB_PER_KB,
                         (st > 0 || kb > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(s));
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) tc_commit(tfull_bar(acc));
      __syncwarp();
    }
    // every tcgen05 op issued above completes before TMEM is released
    if (lane == 0) {
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, err, kDevErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    constexpr int NC = BN / 2;  // accumulator columns per thread
    const int q = warp & 3;     // TMEM lane quadrant this warp may access
    const int half = (warp - 2) >> 2;
    const float alpha = __ldg(p.a_gs) * __ldg(p.b_gs);
    float egs = 1.f, esenc = 1.f;
    if constexpr (epi_gelu(EPI)) {
      egs = __ldg(p.epi_gs);
      esenc = __fdiv_rn(1.0f, egs);
    }
    float* rcp_tab = reinterpret_cast<float*>(gbase + C::CONST_OFF);
    if constexpr (epi_gelu(EPI)) {
      fill_rcp_tab(rcp_tab, threadIdx.x - 64, esenc);
      named_bar_sync(1, 256);
    }
    int lt = 0;
    for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++lt) {
      const int mb = tile / p.tiles_n, nb = tile - mb * p.tiles_n;
      const int acc = lt % C::ACC_STAGES;
      const uint32_t aph = (uint32_t)(lt / C::ACC_STAGES) & 1u;
      if (!mbar_wait(tfull_bar(acc), aph, err, kDevErrTimeoutTmem)) break;
      tc_fence_after();
      uint32_t v[NC];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + half * NC);
#pragma unroll
      for (int c = 0; c < NC / 32; ++c) tmem_ld_32x32b_x32(taddr + c * 32, v + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));

      epilogue_slab<NC, EPI, kF32, C::EPI_CW>(v, p, &tmOut, mb * 128 + q * 32, nb * BN + half * NC, lane, alpha,
                                               egs, esenc,
                                   epi0 + (uint32_t)(warp - 2) * C::EPI_WARP_BYTES,
                                   gbase + C::STAGES * C::STAGE_BYTES + (warp - 2) * C::EPI_WARP_BYTES, rcp_tab);
    }
    if (lane == 0) bulk_wait_all();   // stores issued by this warp complete before the CTA retires
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ---------------------------------------------------------------------------------------
// Weight-stationary variant for K <= 1024 (n_kb <= 16).  Each CTA keeps one 256-wide N tile
// (nb = blockIdx.x % tiles_n) and walks M tiles mb = blockIdx.x / tiles_n + k * (gridDim.x /
// tiles_n): the B tile for the whole K is loaded into shared memory once and B's scale factors
// are copied into TMEM once, so the pipeline streams only A (+ its scales), each K64 step issues
// one scale copy instead of three, and shared-memory traffic per MMA drops from ~190 to ~120 B/clk.
// At any moment the CTAs of one "mb group" share their A row block through L2.
// TMEM: accumulator [0, 256), resident SFB [256, 256 + 8 n_kb), SFA slots [384, 416).
// ---------------------------------------------------------------------------------------
// EW epilogue warps: 16, each 64 accumulator columns of one lane quadrant (the launcher's choice;
// the GELU-NVFP4 epilogue needs the warps to keep up with the MMAs, and the bf16 epilogues drain
// the accumulator sooner with four warps per quadrant than with two: measured 1.4-2.7% faster at
// ViT-L/14 qkv and proj); 8 warps of 128 columns is the other configuration the template supports.
// The CTA's whole B tile (256 rows x K <= 1024, up to 128 KB) stays in shared memory; the four
// pipeline stages carry A (and its scales) only.  The epilogue staging is 1 KB per warp for 16
// warps (bf16 chunks of 16 columns, 32-byte swizzle; 32 rows x 32 bytes of codes for GELU-NVFP4)
// or 2 KB for 8 (chunks of 32 columns, 64-byte swizzle) and shares its shared memory with the B-scale staging,
// which tcgen05.cp reads before the first MMA: the staging is first written after the first
// tile's MMAs (and so those copies) have completed.
template <int EW, bool kGelu>
struct GemmWsCfg {
  static constexpr int BN = 256, BM = 128, KB_PER_STAGE = 4, STAGES = 4;
  static constexpr int ROWB = 32 * KB_PER_STAGE;                 // bytes of K per row and stage
  static constexpr uint32_t LAYOUT = ROWB == 64 ? 4u : 2u;       // SWIZZLE_64B / SWIZZLE_128B
  static constexpr int A_BYTES = BM * ROWB, B_BYTES = BN * ROWB, SFA_BYTES = KB_PER_STAGE * 512;
  static constexpr int STAGE_BYTES = A_BYTES + SFA_BYTES;        // B stays resident, stages carry A
  static constexpr int MAX_KB = 16;
  static constexpr int B_RES_BYTES = (MAX_KB / KB_PER_STAGE) * B_BYTES;   // the CTA's B tile, all of K
  static constexpr int SFB_RES_BYTES = 2 * MAX_KB * 512;
  static constexpr int SFB_TCOL = 256, SFA_TCOL = 384, SFA_SLOT = KB_PER_STAGE * 4;
  static constexpr int TMEM_COLS = 512, THREADS = 64 + 32 * EW;
  static constexpr int NC = BN / (EW / 4);                  // accumulator columns per epilogue thread
  static constexpr int EPI_CW = EW == 16 ? 16 : 32;           // bf16 staging chunk (columns)
  static constexpr int EPI_WARP_BYTES = kGelu ? 32 * NC / 2 : 32 * EPI_CW * 2;
  static constexpr int EPI_BYTES = EW * EPI_WARP_BYTES;
  static constexpr int SHARED_BYTES = EPI_BYTES > SFB_RES_BYTES ? EPI_BYTES : SFB_RES_BYTES;
  static constexpr int NBAR = 2 * STAGES + 2 + 1 + 1;   // full/empty, tfull/tempty, drain, sfb
  static constexpr int CONST_OFF = B_RES_BYTES + STAGES * STAGE_BYTES + SHARED_BYTES + 8 * NBAR + 16;
  static constexpr int CONST_BYTES = kGelu ? 512 + 4 * BN : 0;   // GELU: reciprocal table + fp32 bias
  static constexpr int SMEM = 1024 + CONST_OFF + CONST_BYTES;
  static_assert(CONST_OFF % 16 == 0, "table alignment");
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
  static_assert(EPI_BYTES % 1024 == 0, "staging alignment");
  static_assert(SFA_TCOL + 2 * SFA_SLOT <= TMEM_COLS, "TMEM overflow");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

template <int EPI, bool kF32, int EW>
__global__ void __launch_bounds__(64 + 32 * EW, 1)
    gemm_nvfp4_ws_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmOut, const GemmParams p) {
  using C = GemmWsCfg<EW, epi_gelu(EPI)>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t b_res = base;                                   // the CTA's B tile, all of K
  const uint32_t stage0 = base + C::B_RES_BYTES;
  const uint32_t sfb_res = stage0 + C::STAGES * C::STAGE_BYTES;
  const uint32_t epi0 = sfb_res;   // shared with the B-scale staging (see GemmWsCfg)
  const uint32_t bar0 = epi0 + C::SHARED_BYTES;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  const uint32_t tfull_bar = bar0 + 8u * (2 * C::STAGES), tempty_bar = tfull_bar + 8, drain_bar = tfull_bar + 16,
                 sfb_bar = tfull_bar + 24;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + (bar0 - base) + 8 * C::NBAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = &g_gemm_err;
  const int nb = blockIdx.x % p.tiles_n;
  const int mb0 = blockIdx.x / p.tiles_n, mstep = gridDim.x / p.tiles_n;
  const int n_st = (p.n_kb + C::KB_PER_STAGE - 1) / C::KB_PER_STAGE;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, EW);
    mbar_init(drain_bar, 1);
    mbar_init(sfb_bar, 1);
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
    if (!kF32) tma_prefetch(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      // this CTA's B tile and B scales for all of K, once: scale row blocks 2 nb and 2 nb + 1
      // (N tail: a finite stand-in for the second; B rows >= N are zero-filled by TMA)
      const uint32_t sfb_bytes = (uint32_t)p.n_kb * 512u;
      mbar_arrive_expect_tx(sfb_bar, 2 * sfb_bytes + (uint32_t)n_st * C::B_BYTES);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        int rb = nb * 2 + j;
        if (rb >= p.n_rb_b) rb = nb * 2;
        bulk_load(sfb_res + j * sfb_bytes, p.b_sf + (int64_t)rb * p.n_kb * 512, sfb_bytes, sfb_bar);
      }
      for (int st = 0; st < n_st; ++st)
        tma_load_2d(b_res + st * C::B_BYTES, &tmB, st * C::ROWB, nb * BN, sfb_bar);
      int it = 0;
      bool ok = true;
      for (int mb = mb0; mb < p.tiles_m && ok; mb += mstep) {
        for (int st = 0; st < n_st; ++st, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int kb0 = st * C::KB_PER_STAGE;
          const int nkb = min(C::KB_PER_STAGE, p.n_kb - kb0);
          const uint32_t sf_bytes = (uint32_t)nkb * 512u;
          mbar_arrive_expect_tx(full_bar(s), C::A_BYTES + sf_bytes);
          const uint32_t sa = stage0 + s * C::STAGE_BYTES;
          const uint32_t ssfa = sa + C::A_BYTES;
          tma_load_2d(sa, &tmA, st * C::ROWB, mb * 128, full_bar(s));
          bulk_load(ssfa, p.a_sf + ((int64_t)mb * p.n_kb + kb0) * 512, sf_bytes, full_bar(s));
        }
      }
      for (int k = it - C::STAGES < 0 ? 0 : it - C::STAGES; k < it; ++k)
        mbar_wait(full_bar(k % C::STAGES), (uint32_t)(k / C::STAGES) & 1u, err, kDevErrTimeoutFull);
      mbar_wait(sfb_bar, 0, err, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_mxf4nvf4(BN);
    const uint32_t sfb_t = tmem + C::SFB_TCOL;
    bool ok = mbar_wait(sfb_bar, 0, err, kDevErrTimeoutFull);
    tc_fence_after();
    if (ok && lane == 0) {
      for (int kb = 0; kb < p.n_kb; ++kb)
#pragma unroll
        for (int j = 0; j < 2; ++j)
          tmem_cp_32x128b_x4(sfb_t + kb * 8 + j * 4,
                             smem_desc(sfb_res + (uint32_t)(j * p.n_kb + kb) * 512u, 0, 128, 0));
    }
    __syncwarp();
    int it = 0, lt = 0;
    for (int mb = mb0; mb < p.tiles_m && ok; mb += mstep, ++lt) {
      if (!mbar_wait(tempty_bar, ((uint32_t)lt & 1u) ^ 1u, err, kDevErrTimeoutTmem)) break;
      tc_fence_after();
      for (int st = 0; st < n_st; ++st, ++it) {
        const int s = it % C::STAGES;
        const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
        if (!mbar_wait(full_bar(s), ph, err, kDevErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const int kb0 = st * C::KB_PER_STAGE;
          const int nkb = min(C::KB_PER_STAGE, p.n_kb - kb0);
          const uint32_t sfa_t = tmem + C::SFA_TCOL + (uint32_t)(it & 1) * C::SFA_SLOT;
          const uint32_t sa = stage0 + s * C::STAGE_BYTES;
          const uint32_t sb = b_res + st * C::B_BYTES;
          const uint32_t ssfa = sa + C::A_BYTES;
          for (int kb = 0; kb < nkb; ++kb) {
            tmem_cp_32x128b_x4(sfa_t + kb * 4, smem_desc(ssfa + kb * 512, 0, 128, 0));
            const uint64_t ad = smem_desc(sa + kb * 32, 16, 8 * C::ROWB, C::LAYOUT);
            const uint64_t bd = smem_desc(sb + kb * 32, 16, 8 * C::ROWB, C::LAYOUT);
            mma_mxf4nvf4(tmem, ad, bd, idesc, sfa_t + kb * 4, sfb_t + (kb0 + kb) * 8, (st > 0 || kb > 0) ? 1u : 0u);
          }
          tc_commit(empty_bar(s));
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) tc_commit(tfull_bar);
      __syncwarp();
    }
    if (lane == 0) {
      tc_commit(drain_bar);
      mbar_wait(drain_bar, 0, err, kDevErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    constexpr int NC = C::NC;
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;   // which NC-column slice of the tile
    const float alpha = __ldg(p.a_gs) * __ldg(p.b_gs);
    float egs = 1.f, esenc = 1.f;
    if constexpr (epi_gelu(EPI)) {
      egs = __ldg(p.epi_gs);
      esenc = __fdiv_rn(1.0f, egs);
    }
    // GELU: the scale reciprocal table and this CTA's bias columns (one N tile for all its tiles)
    float* rcp_tab = reinterpret_cast<float*>(gbase + C::CONST_OFF);
    float* bias_f = rcp_tab + 128;
    if constexpr (epi_gelu(EPI)) {
      const int et = threadIdx.x - 64;
      fill_rcp_tab(rcp_tab, et, esenc);
      if constexpr (EPI == VF4_EPI_GELU_ERF_NVFP4) {   // bf16 pairs (the erf form adds b1 in bf16)
        if (et < BN / 2) {
          const int col = nb * BN + 2 * et;
          const uint32_t lo = (p.bias && col < p.N) ? (uint32_t)__bfloat16_as_ushort(p.bias[col]) : 0u;
          const uint32_t hi = (p.bias && col + 1 < p.N) ? (uint32_t)__bfloat16_as_ushort(p.bias[col + 1]) : 0u;
          reinterpret_cast<uint32_t*>(bias_f)[et] = lo | (hi << 16);
        }
      } else if (et < BN) {
        const int col = nb * BN + et;
        bias_f[et] = (p.bias && col < p.N) ? __bfloat162float(p.bias[col]) : 0.f;
      }
      named_bar_sync(1, 32 * EW);
    }
    int lt = 0;
    for (int mb = mb0; mb < p.tiles_m; mb += mstep, ++lt) {
      if (!mbar_wait(tfull_bar, (uint32_t)lt & 1u, err, kDevErrTimeoutTmem)) break;
      tc_fence_after();
      uint32_t v[NC];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(part * NC);
#pragma unroll
      for (int c = 0; c < NC / 32; ++c) tmem_ld_32x32b_x32(taddr + c * 32, v + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar);
      if constexpr (EPI == VF4_EPI_GELU_ERF_NVFP4) {
        // The reference's bf16 values x = RN(RN(acc * alpha) + b1) first, for the whole slab: the
        // slab then lives in NC/2 registers of bf16 pairs through the GELU and the cast.
        const unsigned long long alpha2 = f32x2_pack(alpha, alpha);
        const uint4* bp = reinterpret_cast<const uint4*>(bias_f) + part * NC / 8;
        uint32_t y[NC / 2];
#pragma unroll
        for (int i = 0; i < NC / 8; ++i) {
          const uint4 bb = bp[i];
          const uint32_t b4[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int e = 8 * i + 2 * k;
            const uint32_t r = bf16x2_round(mul_f32x2(f32x2_pack(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), alpha2));
            y[4 * i + k] = p.bias ? add_bf16x2(r, b4[k]) : r;
          }
        }
        nvfp4_slab_store<NC>(
            [&](int blk, int, float* h) {
#pragma unroll
              for (int i = 0; i < 8; ++i) f32x2_unpack(gelu_erf_x2(bf16x2_to_f32x2(y[blk * 8 + i])), &h[2 * i], &h[2 * i + 1]);
            },
            p, &tmOut, mb * 128 + q * 32, nb * BN + part * NC, lane, esenc,
            epi0 + (uint32_t)(warp - 2) * C::EPI_WARP_BYTES, gbase + (epi0 - base) + (warp - 2) * C::EPI_WARP_BYTES,
            rcp_tab);
        continue;
      }
      epilogue_slab<NC, EPI, kF32, C::EPI_CW>(v, p, &tmOut, mb * 128 + q * 32, nb * BN + part * NC, lane, alpha,
                                               egs, esenc,
                                   epi0 + (uint32_t)(warp - 2) * C::EPI_WARP_BYTES,
                                   gbase + (epi0 - base) + (warp - 2) * C::EPI_WARP_BYTES, rcp_tab,
                                   !epi_gelu(EPI) ? nullptr
                                   : EPI == VF4_EPI_GELU_ERF_NVFP4 ? bias_f + part * NC / 2   // bf16 pairs
                                                                   : bias_f + part * NC);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}


// ---------------------------------------------------------------------------------------
// CTA-pair variant: a cluster of 2 CTAs computes a 256 x 256 tile with cta_group::2 MMAs.
// Each CTA TMA-loads its own 128 rows of A and its own 128-row half of B (no multicast), plus the
// scale atoms (its SFA row-block and both SFB row-blocks).  A forwarder warp in each CTA waits on
// its own "full" barrier and arrives on the leader's pair barrier; the leader (cluster rank 0)
// issues the scale copies and MMAs for both CTAs and multicast-commits stage releases and the
// accumulator hand-off to both CTAs' barriers; every epilogue warp of both CTAs releases TMEM by
// arriving on the leader's barrier.  Per CTA and K64 step the shared-memory traffic is 8 KB of
// TMA writes + 8 KB of MMA reads, within the SM's 128 B/clk (the 1-CTA 128x256 tile needs 24 KB).
// Warps: 0 producer, 1 TMEM allocator + MMA issuer (leader), 2 forwarder, 3..10 epilogue.
// ---------------------------------------------------------------------------------------
struct Gemm2Cfg {
  static constexpr int BN = 256;
  static constexpr int KB_PER_STAGE = 4;
  static constexpr int STAGES = 5;
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = 128 * 128;     // this CTA's half of the 256 B rows
  static constexpr int SFA_BYTES = KB_PER_STAGE * 512;
  static constexpr int SFB_BYTES = 2 * KB_PER_STAGE * 512;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  static constexpr int SFA_TCOL = 256, SFA_SLOT = KB_PER_STAGE * 4;
  static constexpr int SFB_TCOL = SFA_TCOL + 2 * SFA_SLOT, SFB_PER_KB = 8, SFB_SLOT = KB_PER_STAGE * SFB_PER_KB;
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 352;
  static constexpr int EPI_WARP_BYTES = 4096, EPI_BYTES = 8 * EPI_WARP_BYTES;
  static constexpr int NBAR = 3 * STAGES + 3;
  static constexpr int CONST_OFF = STAGES * STAGE_BYTES + EPI_BYTES + 8 * NBAR + 16;
  static constexpr int SMEM = 1024 + CONST_OFF + 512;   // + the GELU scale reciprocal table
  static_assert(CONST_OFF % 16 == 0, "table alignment");
  static_assert(STAGE_BYTES % 1024 == 0, "stage alignment");
  static_assert(SFB_TCOL + 2 * SFB_SLOT <= TMEM_COLS, "TMEM overflow");
};

template <int EPI, bool kF32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(352, 1)
    gemm_nvfp4_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmOut, const GemmParams p) {
  using C = Gemm2Cfg;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t epi0 = base + C::STAGES * C::STAGE_BYTES;
  const uint32_t bar0 = epi0 + C::EPI_BYTES;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };                 // own TMA completion
  auto pair_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };   // leader: both CTAs' data ready
  auto empty_bar = [&](int s) { return bar0 + 8u * (2 * C::STAGES + s); };
  const uint32_t tfull_bar = bar0 + 8u * (3 * C::STAGES);
  const uint32_t tempty_bar = tfull_bar + 8, drain_bar = tfull_bar + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + C::STAGES * C::STAGE_BYTES + C::EPI_BYTES + 8 * C::NBAR);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  int* err = &g_gemm_err;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(pair_bar(s), 2);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull_bar, 1);
    mbar_init(tempty_bar, 16);
    mbar_init(drain_bar, 1);
    fence_mbar_init();
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
    if (!kF32) tma_prefetch(&tmOut);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), C::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles = p.tiles_m * p.tiles_n;   // tiles_m counts 256-row tiles here
  const int n_st = (p.n_kb + C::KB_PER_STAGE - 1) / C::KB_PER_STAGE;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs) {
        const int pm = tile / p.tiles_n, nb = tile - pm * p.tiles_n;
        int rba = pm * 2 + (int)rank;
        if (rba >= p.n_rb_a) rba = p.n_rb_a - 1;   // M tail: A rows are zero-filled, scales unused
        for (int st = 0; st < n_st; ++st, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!mbar_wait(empty_bar(s), ph ^ 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int kb0 = st * C::KB_PER_STAGE;
          const int nkb = min(C::KB_PER_STAGE, p.n_kb - kb0);
          const uint32_t sf_bytes = (uint32_t)nkb * 512u;
          mbar_arrive_expect_tx(full_bar(s), C::A_BYTES + C::B_BYTES + 3 * sf_bytes);
          const uint32_t sa = base + s * C::STAGE_BYTES;
          const uint32_t sb = sa + C::A_BYTES;
          const uint32_t ssfa = sb + C::B_BYTES;
          const uint32_t ssfb = ssfa + C::SFA_BYTES;
          tma_load_2d(sa, &tmA, st * 128, pm * 256 + (int)rank * 128, full_bar(s));
          tma_load_2d(sb, &tmB, st * 128, nb * BN + (int)rank * 128, full_bar(s));
          bulk_load(ssfa, p.a_sf + ((int64_t)rba * p.n_kb + kb0) * 512, sf_bytes, full_bar(s));
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            int rb = nb * 2 + j;
            if (rb >= p.n_rb_b) rb = nb * 2;   // N tail: finite stand-in, columns discarded
            bulk_load(ssfb + j * C::KB_PER_STAGE * 512, p.b_sf + ((int64_t)rb * p.n_kb + kb0) * 512, sf_bytes,
                      full_bar(s));
          }
        }
      }
      for (int k = it - C::STAGES < 0 ? 0 : it - C::STAGES; k < it; ++k)
        mbar_wait(full_bar(k % C::STAGES), (uint32_t)(k / C::STAGES) & 1u, err, kDevErrTimeoutFull);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------------ forwarder (both CTAs)
    if (lane == 0) {
      const uint32_t n_iter = (uint32_t)((tiles - pair + npairs - 1) / npairs) * (uint32_t)n_st;
      for (uint32_t it = 0; it < (pair < tiles ? n_iter : 0u); ++it) {
        const int s = it % C::STAGES;
        if (!mbar_wait(full_bar(s), (it / C::STAGES) & 1u, err, kDevErrTimeoutFull)) break;
        mbar_arrive_remote(mapa_shared(pair_bar(s), 0));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (leader) {
      constexpr uint32_t idesc = idesc_mxf4nvf4(BN, 256);
      int it = 0, lt = 0;
      bool ok = true;
      for (int tile = pair; tile < tiles && ok; tile += npairs, ++lt) {
        if (!mbar_wait_cluster(tempty_bar, ((uint32_t)lt & 1u) ^ 1u, err, kDevErrTimeoutTmem)) break;
        tc_fence_after();
        for (int st = 0; st < n_st; ++st, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait_cluster(pair_bar(s), (uint32_t)(it / C::STAGES) & 1u, err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const int nkb = min(C::KB_PER_STAGE, p.n_kb - st * C::KB_PER_STAGE);
            const uint32_t slot = (uint32_t)(it & 1);
            const uint32_t sfa_t = tmem + C::SFA_TCOL + slot * C::SFA_SLOT;
            const uint32_t sfb_t = tmem + C::SFB_TCOL + slot * C::SFB_SLOT;
            const uint32_t sa = base + s * C::STAGE_BYTES;
            const uint32_t sb = sa + C::A_BYTES;
            const uint32_t ssfa = sb + C::B_BYTES;
            const uint32_t ssfb = ssfa + C::SFA_BYTES;
            for (int kb = 0; kb < nkb; ++kb) {
              tmem_cp_32x128b_x4_pair(sfa_t + kb * 4, smem_desc(ssfa + kb * 512, 0, 128, 0));
#pragma unroll
              for (int j = 0; j < 2; ++j)
                tmem_cp_32x128b_x4_pair(sfb_t + kb * C::SFB_PER_KB + j * 4,
                                        smem_desc(ssfb + j * C::KB_PER_STAGE * 512 + kb * 512, 0, 128, 0));
              const uint64_t ad = smem_desc(sa + kb * 32, 16, 1024, 2);
              const uint64_t bd = smem_desc(sb + kb * 32, 16, 1024, 2);
              mma_mxf4nvf4_pair(tmem, ad, bd, idesc, sfa_t + kb * 4, sfb_t + kb * C::SFB_PER_KB,
                                (st > 0 || kb > 0) ? 1u : 0u);
            }
            tc_commit_pair(empty_bar(s), 3);
          }
          __syncwarp();
        }
        if (!ok) break;
        if (lane == 0) tc_commit_pair(tfull_bar, 3);
        __syncwarp();
      }
      if (lane == 0) {
        tc_commit_pair(drain_bar, 1);
        mbar_wait(drain_bar, 0, err, kDevErrTimeoutDrain);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------------ epilogue (both CTAs)
    constexpr int NC = BN / 2;
    const int q = warp & 3;
    const int half = (warp - 3) >> 2;
    const float alpha = __ldg(p.a_gs) * __ldg(p.b_gs);
    float egs = 1.f, esenc = 1.f;
    if constexpr (epi_gelu(EPI)) {
      egs = __ldg(p.epi_gs);
      esenc = __fdiv_rn(1.0f, egs);
    }
    float* rcp_tab = reinterpret_cast<float*>(gbase + C::CONST_OFF);
    if constexpr (epi_gelu(EPI)) {
      fill_rcp_tab(rcp_tab, threadIdx.x - 96, esenc);
      named_bar_sync(1, 256);
    }
    const uint32_t tempty_leader = mapa_shared(tempty_bar, 0);
    int lt = 0;
    for (int tile = pair; tile < tiles; tile += npairs, ++lt) {
      const int pm = tile / p.tiles_n, nb = tile - pm * p.tiles_n;
      if (!mbar_wait(tfull_bar, (uint32_t)lt & 1u, err, kDevErrTimeoutTmem)) break;
      tc_fence_after();
      uint32_t v[NC];
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(half * NC);
#pragma unroll
      for (int c = 0; c < NC / 32; ++c) tmem_ld_32x32b_x32(taddr + c * 32, v + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_leader);
      epilogue_slab<NC, EPI, kF32>(v, p, &tmOut, pm * 256 + (int)rank * 128 + q * 32, nb * BN + half * NC, lane,
                                   alpha, egs, esenc, epi0 + (uint32_t)(warp - 3) * C::EPI_WARP_BYTES,
                                   gbase + C::STAGES * C::STAGE_BYTES + (warp - 3) * C::EPI_WARP_BYTES, rcp_tab);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, C::TMEM_COLS);
}

static int make_kmajor_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t kbytes, int box_rows,
                           int box_bytes = 128) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)kbytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kbytes};
  cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VF4_OK;
}

// Output map for the TMA-store epilogue: bf16 (M, N) with 64x32 boxes and the 128-byte swizzle,
// or packed FP4 codes (M, N/2) bytes with (BN/4)x32 boxes and the BN/4-byte swizzle.
static int make_out_map(CUtensorMap* m, void* ptr, int64_t rows, int64_t cols, bool fp4, int bn, int cw = 64) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int64_t rowbytes = fp4 ? cols / 2 : cols * 2;
  cuuint64_t dims[2] = {(cuuint64_t)(fp4 ? cols / 2 : cols), (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)rowbytes};
  cuuint32_t box[2] = {(cuuint32_t)(fp4 ? bn / 4 : cw), 32u};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = enc(m, fp4 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   fp4 ? (bn == 256 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B)
                       : (cw == 64 ? CU_TENSOR_MAP_SWIZZLE_128B
                                   : cw == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_32B),
                   CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled (output) failed (%d)", (int)r);
  return VF4_OK;
}

template <int BN, int EPI, bool kF32, bool REP>
static int launch_gemm_t(const uint8_t* a, const uint8_t* b, GemmParams& p, cudaStream_t s) {
  using C = GemmCfg<BN, EPI, kF32, REP>;
  CUtensorMap ta, tb, to;
  memset(&to, 0, sizeof(to));
  if (int st = make_kmajor_map(&ta, a, p.M, p.K / 2, 128)) return st;
  if (int st = make_kmajor_map(&tb, b, p.N, p.K / 2, BN)) return st;
  if (epi_gelu(EPI)) {
    if (int st = make_out_map(&to, p.out_packed, p.M, p.N, true, BN)) return st;
  } else if (!kF32) {
    if (int st = make_out_map(&to, p.out, p.M, p.N, false, BN, C::EPI_CW)) return st;
  }
  auto kern = gemm_nvfp4_kernel<BN, EPI, kF32, REP>;
  if (int st = smem_optin(kern, C::SMEM)) return st;
  p.tiles_m = (p.M + 127) / 128;
  p.tiles_n = (p.N + BN - 1) / BN;
  int tiles = p.tiles_m * p.tiles_n;
  int grid = tiles < num_sms() ? tiles : num_sms();
  kern<<<grid, C::THREADS, C::SMEM, s>>>(ta, tb, to, p);
  return launch_status("vf4_gemm_nvfp4");
}

template <int BN, int EPI, bool kF32>
static int launch_gemm(const uint8_t* a, const uint8_t* b, GemmParams& p, cudaStream_t s) {
  if constexpr (BN == 256) {
    if (p.b_img) return launch_gemm_t<BN, EPI, kF32, true>(a, b, p, s);
  }
  return launch_gemm_t<BN, EPI, kF32, false>(a, b, p, s);
}

template <int EPI, bool kF32>
static int launch_gemm_pair(const uint8_t* a, const uint8_t* b, GemmParams& p, cudaStream_t s) {
  using C = Gemm2Cfg;
  CUtensorMap ta, tb, to;
  memset(&to, 0, sizeof(to));
  if (int st = make_kmajor_map(&ta, a, p.M, p.K / 2, 128)) return st;
  if (int st = make_kmajor_map(&tb, b, p.N, p.K / 2, 128)) return st;
  if (epi_gelu(EPI)) {
    if (int st = make_out_map(&to, p.out_packed, p.M, p.N, true, C::BN)) return st;
  } else if (!kF32) {
    if (int st = make_out_map(&to, p.out, p.M, p.N, false, C::BN)) return st;
  }
  auto kern = gemm_nvfp4_pair_kernel<EPI, kF32>;
  if (int st = smem_optin(kern, C::SMEM)) return st;
  p.tiles_m = (p.M + 255) / 256;
  p.tiles_n = (p.N + C::BN - 1) / C::BN;
  const int tiles = p.tiles_m * p.tiles_n;
  const int max_pairs = num_sms() / 2;
  const int pairs = tiles < max_pairs ? tiles : max_pairs;
  kern<<<2 * pairs, C::THREADS, C::SMEM, s>>>(ta, tb, to, p);
  return launch_status("vf4_gemm_nvfp4 (CTA pair)");
}

static int dispatch_gemm_pair(const uint8_t* a, const uint8_t* b, GemmParams& p, int epi, int f32, cudaStream_t s) {
  if (epi == VF4_EPI_GELU_NVFP4) return launch_gemm_pair<VF4_EPI_GELU_NVFP4, false>(a, b, p, s);
  if (epi == VF4_EPI_GELU_ERF_NVFP4) return launch_gemm_pair<VF4_EPI_GELU_ERF_NVFP4, false>(a, b, p, s);
  if (epi == VF4_EPI_BIAS_RESIDUAL) return launch_gemm_pair<VF4_EPI_BIAS_RESIDUAL, false>(a, b, p, s);
  if (epi == VF4_EPI_BIAS)
    return f32 ? launch_gemm_pair<VF4_EPI_BIAS, true>(a, b, p, s) : launch_gemm_pair<VF4_EPI_BIAS, false>(a, b, p, s);
  return f32 ? launch_gemm_pair<VF4_EPI_NONE, true>(a, b, p, s) : launch_gemm_pair<VF4_EPI_NONE, false>(a, b, p, s);
}

template <int EPI, bool kF32>
static int launch_gemm_ws(const uint8_t* a, const uint8_t* b, GemmParams& p, cudaStream_t s) {
  constexpr int EW = 16;
  using C = GemmWsCfg<EW, epi_gelu(EPI)>;
  CUtensorMap ta, tb, to;
  memset(&to, 0, sizeof(to));
  if (int st = make_kmajor_map(&ta, a, p.M, p.K / 2, 128, C::ROWB)) return st;
  if (int st = make_kmajor_map(&tb, b, p.N, p.K / 2, C::BN, C::ROWB)) return st;
  if (epi_gelu(EPI)) {   // each warp stores 32 rows x NC/2 bytes of codes: the map of a 2*NC-wide tile
    if (int st = make_out_map(&to, p.out_packed, p.M, p.N, true, 2 * C::NC)) return st;
  } else if (!kF32) {
    if (int st = make_out_map(&to, p.out, p.M, p.N, false, C::BN, C::EPI_CW)) return st;
  }
  auto kern = gemm_nvfp4_ws_kernel<EPI, kF32, EW>;
  if (int st = smem_optin(kern, C::SMEM)) return st;
  p.tiles_m = (p.M + 127) / 128;
  p.tiles_n = (p.N + C::BN - 1) / C::BN;
  const int groups = num_sms() / p.tiles_n;   // CTAs per N tile
  kern<<<groups * p.tiles_n, C::THREADS, C::SMEM, s>>>(ta, tb, to, p);
  return launch_status("vf4_gemm_nvfp4 (resident B scales)");
}

static int dispatch_gemm_ws(const uint8_t* a, const uint8_t* b, GemmParams& p, int epi, int f32, cudaStream_t s) {
  if (epi == VF4_EPI_GELU_NVFP4) return launch_gemm_ws<VF4_EPI_GELU_NVFP4, false>(a, b, p, s);
  if (epi == VF4_EPI_GELU_ERF_NVFP4) return launch_gemm_ws<VF4_EPI_GELU_ERF_NVFP4, false>(a, b, p, s);
  if (epi == VF4_EPI_BIAS_RESIDUAL) return launch_gemm_ws<VF4_EPI_BIAS_RESIDUAL, false>(a, b, p, s);
  if (epi == VF4_EPI_BIAS)
    return f32 ? launch_gemm_ws<VF4_EPI_BIAS, true>(a, b, p, s) : launch_gemm_ws<VF4_EPI_BIAS, false>(a, b, p, s);
  return f32 ? launch_gemm_ws<VF4_EPI_NONE, true>(a, b, p, s) : launch_gemm_ws<VF4_EPI_NONE, false>(a, b, p, s);
}

template <int BN>
static int dispatch_gemm(const uint8_t* a, const uint8_t* b, GemmParams& p, int epi, int f32,
                         cudaStream_t s) {
  if (epi == VF4_EPI_GELU_NVFP4) return launch_gemm<BN, VF4_EPI_GELU_NVFP4, false>(a, b, p, s);
  if (epi == VF4_EPI_GELU_ERF_NVFP4) return launch_gemm<BN, VF4_EPI_GELU_ERF_NVFP4, false>(a, b, p, s);
  if (epi == VF4_EPI_BIAS_RESIDUAL) return launch_gemm<BN, VF4_EPI_BIAS_RESIDUAL, false>(a, b, p, s);
  if (epi == VF4_EPI_BIAS) {
    return f32 ? launch_gemm<BN, VF4_EPI_BIAS, true>(a, b, p, s)
               : launch_gemm<BN, VF4_EPI_BIAS, false>(a, b, p, s);
  }
  return f32 ? launch_gemm<BN, VF4_EPI_NONE, true>(a, b, p, s)
             : launch_gemm<BN, VF4_EPI_NONE, false>(a, b, p, s);
}

}  // namespace vf4

using namespace vf4;

static int gemm_entry(const uint8_t* a_packed, const uint8_t* a_sf, const float* a_gs, const uint8_t* b_packed,
                      const uint8_t* b_sf, const float* b_gs, int64_t M, int64_t N, int64_t K, const void* bias,
                      int epilogue, void* out, int out_dtype, const float* epi_gs, uint8_t* out_packed,
                      uint8_t* out_sf, const void* residual, const void* gamma, vf4_stream_t stream,
                      const uint8_t* b_img = nullptr) {
  if (int st = check_device()) return st;
  if (M < 0 || N <= 0 || K <= 0) return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4: bad sizes M=%lld N=%lld K=%lld",
                                             (long long)M, (long long)N, (long long)K);
  if (M > (int64_t)INT32_MAX / 2 || N > 65535 * 128 || K > (1 << 20))
    return fail(VF4_ERR_UNSUPPORTED, "vf4_gemm_nvfp4: sizes too large");
  if (K % 32 != 0 || N % 16 != 0)
    return fail(VF4_ERR_UNSUPPORTED, "vf4_gemm_nvfp4: need K %% 32 == 0 and N %% 16 == 0 (K=%lld N=%lld)",
                (long long)K, (long long)N);
  if (epilogue < VF4_EPI_NONE || epilogue > VF4_EPI_BIAS_RESIDUAL)
    return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4: bad epilogue %d", epilogue);
  if (!a_packed || !a_sf || !a_gs || !b_packed || !b_sf || !b_gs)
    return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4: null operand");
  if (!aligned16(a_packed) || !aligned16(b_packed) || !aligned16(a_sf) || !aligned16(b_sf) ||
      (bias && !aligned16(bias)))
    return fail(VF4_ERR_ALIGN, "vf4_gemm_nvfp4: operands, scales and bias must be 16-byte aligned");
  if (b_img && !aligned16(b_img)) return fail(VF4_ERR_ALIGN, "vf4_gemm_nvfp4_ex: b_image must be 16-byte aligned");
  if (epilogue == VF4_EPI_BIAS_RESIDUAL) {
    if (!residual) return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4_residual: residual is NULL");
    if (!aligned16(residual) || (gamma && !aligned16(gamma)))
      return fail(VF4_ERR_ALIGN, "vf4_gemm_nvfp4_residual: residual and gamma must be 16-byte aligned");
  }
  if (epi_gelu(epilogue)) {
    if (N % 64 != 0) return fail(VF4_ERR_UNSUPPORTED, "vf4_gemm_nvfp4: GELU-NVFP4 epilogue needs N %% 64 == 0");
    if (!epi_gs || !out_packed || !out_sf) return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4: GELU-NVFP4 outputs missing");
    if ((reinterpret_cast<uintptr_t>(out_packed) & 7u) || (reinterpret_cast<uintptr_t>(out_sf) & 3u))
      return fail(VF4_ERR_ALIGN, "vf4_gemm_nvfp4: out_packed 8-byte / out_sf 4-byte alignment");
  } else {
    if (!out) return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4: out is NULL");
    if (out_dtype != VF4_BF16 && out_dtype != VF4_F32) return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4: bad out_dtype");
    if (!aligned16(out)) return fail(VF4_ERR_ALIGN, "vf4_gemm_nvfp4: out must be 16-byte aligned");
  }
  if (M == 0) return VF4_OK;
  GemmParams p{};
  p.a_sf = a_sf;
  p.b_sf = b_sf;
  p.b_img = b_img;
  p.a_gs = a_gs;
  p.b_gs = b_gs;
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.n_kb = (int)((K + 63) / 64);
  p.n_rb_b = (int)((N + 127) / 128);
  p.n_rb_a = (int)((M + 127) / 128);
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.out = out;
  p.epi_gs = epi_gs;
  p.out_packed = out_packed;
  p.out_sf = out_sf;
  p.out_ncb = (int)((N / 16 + 3) / 4);
  p.res = static_cast<const __nv_bfloat16*>(residual);
  p.gamma = static_cast<const __nv_bfloat16*>(gamma);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const char* mode = getenv("VF4_GEMM_TILE");   // "pair" selects the CTA-pair 256x256 kernel
  if (N >= 256 && M > 128 && mode && mode[0] == 'p')
    return dispatch_gemm_pair(a_packed, b_packed, p, epilogue, out_dtype == VF4_F32, s);
  // resident-B-scales kernel: K <= 1024, at least one CTA per N tile and one M tile per CTA
  // (VF4_GEMM_TILE=stream selects the plain streaming kernel)
  const bool ws_ok = N >= 256 && p.n_kb <= 16 && (N + 255) / 256 <= num_sms() &&
                     (M + 127) / 128 >= num_sms() / ((N + 255) / 256) && !(mode && mode[0] == 's');
  if (ws_ok) return dispatch_gemm_ws(a_packed, b_packed, p, epilogue, out_dtype == VF4_F32, s);
  if (N >= 256) return dispatch_gemm<256>(a_packed, b_packed, p, epilogue, out_dtype == VF4_F32, s);
  return dispatch_gemm<128>(a_packed, b_packed, p, epilogue, out_dtype == VF4_F32, s);
}

extern "C" int vf4_selftest_wait_timeout(uint64_t limit_ns, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (limit_ns == 0 || limit_ns > 1000000000ull)
    return fail(VF4_ERR_ARG, "vf4_selftest_wait_timeout: limit must be in (0, 1 s]");
  wait_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns);
  return launch_status("vf4_selftest_wait_timeout");
}

extern "C" int vf4_gemm_nvfp4(const uint8_t* a_packed, const uint8_t* a_sf, const float* a_gs,
                              const uint8_t* b_packed, const uint8_t* b_sf, const float* b_gs,
                              int64_t M, int64_t N, int64_t K, const void* bias, int epilogue,
                              void* out, int out_dtype, const float* epi_gs, uint8_t* out_packed,
                              uint8_t* out_sf, vf4_stream_t stream) {
  if (epilogue == VF4_EPI_BIAS_RESIDUAL)
    return fail(VF4_ERR_ARG, "vf4_gemm_nvfp4: the residual epilogue is vf4_gemm_nvfp4_residual");
  return gemm_entry(a_packed, a_sf, a_gs, b_packed, b_sf, b_gs, M, N, K, bias, epilogue, out, out_dtype, epi_gs,
                    out_packed, out_sf, nullptr, nullptr, stream);
}

extern "C" int vf4_gemm_nvfp4_residual(const uint8_t* a_packed, const uint8_t* a_sf, const float* a_gs,
                                       const uint8_t* b_packed, const uint8_t* b_sf, const float* b_gs,
                                       int64_t M, int64_t N, int64_t K, const void* bias, const void* residual,
                                       const void* gamma, void* out, vf4_stream_t stream) {
  return gemm_entry(a_packed, a_sf, a_gs, b_packed, b_sf, b_gs, M, N, K, bias, VF4_EPI_BIAS_RESIDUAL, out, VF4_BF16,
                    nullptr, nullptr, nullptr, residual, gamma, stream);
}

// B scale image: for every 256-row tile tn of B and K64 block kb, 4 KB = [rows 0-127 atom x4][rows
// 128-255 atom x4] of the 512-byte to_blocked atoms (a tile past N repeats its first atom: finite
// scales for columns the epilogue discards).  One thread per 16 bytes.
__global__ void b_scale_image_kernel(const uint8_t* __restrict__ sf, int n_rb, int n_kb, int64_t words,
                                     uint8_t* __restrict__ img) {
  const int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (w >= words) return;
  const int64_t a = w >> 5;                     // 512-byte block of the image
  const int j = (int)((a >> 2) & 1);
  const int64_t tk = a >> 3;                    // tn * n_kb + kb
  const int kb = (int)(tk % n_kb), tn = (int)(tk / n_kb);
  int rb = 2 * tn + j;
  if (rb >= n_rb) rb = 2 * tn;
  reinterpret_cast<uint4*>(img)[w] =
      __ldg(reinterpret_cast<const uint4*>(sf + ((int64_t)rb * n_kb + kb) * 512) + (w & 31));
}

extern "C" int64_t vf4_b_scale_image_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0) return 0;
  return (N + 255) / 256 * ((K + 63) / 64) * 4096;
}

extern "C" int vf4_b_scale_image(const uint8_t* b_sf, int64_t N, int64_t K, uint8_t* image, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (N <= 0 || K <= 0 || N > 65535 * 128 || K > (1 << 20)) return fail(VF4_ERR_ARG, "vf4_b_scale_image: bad sizes");
  if (!b_sf || !image) return fail(VF4_ERR_ARG, "vf4_b_scale_image: null pointer");
  if (!aligned16(b_sf) || !aligned16(image)) return fail(VF4_ERR_ALIGN, "vf4_b_scale_image: 16-byte alignment");
  const int64_t words = vf4_b_scale_image_bytes(N, K) / 16;
  b_scale_image_kernel<<<(unsigned)((words + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      b_sf, (int)((N + 127) / 128), (int)((K + 63) / 64), words, image);
  return launch_status("vf4_b_scale_image");
}

extern "C" int vf4_gemm_nvfp4_ex(const uint8_t* a_packed, const uint8_t* a_sf, const float* a_gs,
                                 const uint8_t* b_packed, const uint8_t* b_sf, const uint8_t* b_image,
                                 const float* b_gs, int64_t M, int64_t N, int64_t K, const void* bias, int epilogue,
                                 void* out, int out_dtype, const float* epi_gs, uint8_t* out_packed, uint8_t* out_sf,
                                 const void* residual, const void* gamma, vf4_stream_t stream) {
  return gemm_entry(a_packed, a_sf, a_gs, b_packed, b_sf, b_gs, M, N, K, bias, epilogue, out, out_dtype, epi_gs,
                    out_packed, out_sf, residual, gamma, stream, b_image);
}
