// Low-precision attention for ViT on sm_100a: QK^T and PV as tcgen05 MMAs.
//
// NVFP4 routes follow the reference's emulated quant_sdpa(qk='nvfp4', pv='nvfp4', smooth_k,
// smooth_v) (src/vit_nvfp4/nvfp4/attention.py:53-86):
//   k~ = k - mean_S(k);  S = deq(Q) deq(K~)^T * scale;  P = softmax(S);
//   v~ = v - mean_S(v);  out = deq(P) deq(V~) + mean_S(v)
// with Q, K~ quantized along the head dim and V~ along tokens (16-element NVFP4 blocks, E4M3
// block scales, "six" rule, ties-down codes) under the reference's tensor-wide global scales
// (or, with VF4_ATTN_HEAD_GLOBALS, per (image, head)).  Two deliberate differences: P uses the
// fixed global 1/(6*448) instead of the amax of the whole P tensor, and P is quantized before
// the 1/rowsum (P = exp(S - max) lies in [0, 1] with the row max exactly 1; the output is
// divided by the row sum), so a tile's probabilities need one pass over its scores for the
// maximum and one for P.
// The FP8 routes (quant_sdpa(qk='fp8', pv='fp8'), the reference's default arguments) and the
// bf16 route of blocks the reference leaves unconverted are described at their kernels below.
#include <mutex>

#include "vf4_common.cuh"
#include "vf4_host.h"

namespace vf4 {

static __device__ int g_attn_err;

int attn_device_error(int clear) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_attn_err, sizeof(int));
  if (clear) {
    int z = 0;
    cudaMemcpyToSymbol(g_attn_err, &z, sizeof(int));
  }
  return v;
}

constexpr int kScalStride = 4 + 128;   // per head: gs_q, gs_k, gs_v, pad, mean_v[128]
constexpr float kInv2688 = 1.0f / 2688.0f;

struct AttnGeom {
  int B, H, S, D;
  int S_pad, Dp, Dv, nc;
  int64_t BH;
  int64_t q_head, vt_head, qsf_head, vsf_head;  // bytes per head
  int64_t off_q, off_k, off_v, off_qsf, off_ksf, off_vsf, off_scal, total;
};

static int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

static AttnGeom make_geom(int64_t B, int64_t H, int64_t S, int64_t D) {
  AttnGeom g{};
  g.B = (int)B;
  g.H = (int)H;
  g.S = (int)S;
  g.D = (int)D;
  g.S_pad = (int)align_up(S, 128);
  g.Dp = D <= 64 ? 64 : 128;
  g.Dv = g.Dp;
  g.nc = g.S_pad / 128;
  g.BH = B * H;
  g.q_head = (int64_t)g.S_pad * g.Dp / 2;
  g.vt_head = (int64_t)g.Dv * g.S_pad / 2;
  g.qsf_head = (int64_t)(g.S_pad / 128) * (g.Dp / 64) * 512;
  g.vsf_head = (int64_t)(g.S_pad / 64) * 512;
  int64_t o = 0;
  g.off_q = o;   o = align_up(o + g.BH * g.q_head, 1024);
  g.off_k = o;   o = align_up(o + g.BH * g.q_head, 1024);
  g.off_v = o;   o = align_up(o + g.BH * g.vt_head, 1024);
  g.off_qsf = o; o = align_up(o + g.BH * g.qsf_head, 1024);
  g.off_ksf = o; o = align_up(o + g.BH * g.qsf_head, 1024);
  g.off_vsf = o; o = align_up(o + g.BH * g.vsf_head, 1024);
  g.off_scal = o; o = align_up(o + g.BH * kScalStride * 4, 1024);
  g.total = o;
  return g;
}

// ---------------------------------------------------------------------------------------
// Kernel 1: per-(b,h) smoothing, global scales and NVFP4 packing
// ---------------------------------------------------------------------------------------
VF4_DEV void load8(const __nv_bfloat16* p, float* v) {
  uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

VF4_DEV float block_max(float m, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) r = fmaxf(r, red[i]);
  return r;
}

VF4_DEV float warp_max(float m) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  return m;
}

// ---------------------------------------------------------------------------------------
// Per-head statistics for the reference's tensor-wide global scales (attention.py:28-50 takes one
// amax over the whole q, k~ and v~ tensors): column means of k and v per (b, h), written to
// `stats` (mu_k[Dp], mu_v[Dp] per head), and atomic maxima over all heads of |q|, |k - mu_k|,
// |v - mu_v| into amax3[0..2] (non-negative floats compare like their bit patterns).  The
// centred maxima come from column max / min: rounding is monotone, so max_s |x_s - m| =
// max(|max x - m|, |min x - m|) exactly.  One read of q, k and v; 256 threads per head.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) attn_stats_kernel(const __nv_bfloat16* __restrict__ q,
                                                         const __nv_bfloat16* __restrict__ k,
                                                         const __nv_bfloat16* __restrict__ v, int64_t sb,
                                                         int64_t sh, int64_t ss, int H, int S, int D, int Dp,
                                                         int smooth, float* __restrict__ stats,
                                                         float* __restrict__ amax3) {
  extern __shared__ float part[];   // [8 warps][6][D] (or [6][rpi][D]): k sum/max/min, v sum/max/min
  __shared__ float red[3][8];
  const int head = blockIdx.x;
  const int b = head / H, h = head - b * H;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int D8 = D / 8, rpi = 256 / D8, active = rpi * D8;
  const bool lanes_share = 32 % D8 == 0;   // every lane of a warp on whole rows (D = 16, 32, 64, 128)
  const int j = t % D8, r0 = t / D8;
  const int64_t off = (int64_t)b * sb + (int64_t)h * sh + 8 * j;
  float ks[8], kx[8], kn[8], vs[8], vx[8], vn[8], qm = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    ks[e] = vs[e] = 0.f;
    kx[e] = vx[e] = -INFINITY;
    kn[e] = vn[e] = INFINITY;
  }
  if (t < active) {
    // two rows per iteration: six 16-byte loads in flight per thread
    for (int r = r0; r < S; r += 2 * rpi) {
      const bool two = r + rpi < S;
      float a[2][8], c[2][8], u[2][8];
      load8(q + off + (int64_t)r * ss, a[0]);
      load8(k + off + (int64_t)r * ss, c[0]);
      load8(v + off + (int64_t)r * ss, u[0]);
      if (two) {
        load8(q + off + (int64_t)(r + rpi) * ss, a[1]);
        load8(k + off + (int64_t)(r + rpi) * ss, c[1]);
        load8(v + off + (int64_t)(r + rpi) * ss, u[1]);
      }
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        if (m == 1 && !two) break;   // the means keep a fixed summation order: row r, then r + rpi
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          qm = fmaxf(qm, fabsf(a[m][e]));
          ks[e] += c[m][e];
          kx[e] = fmaxf(kx[e], c[m][e]);
          kn[e] = fminf(kn[e], c[m][e]);
          vs[e] += u[m][e];
          vx[e] = fmaxf(vx[e], u[m][e]);
          vn[e] = fminf(vn[e], u[m][e]);
        }
      }
    }
    if (!lanes_share) {
      const int RD = rpi * D;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = r0 * D + 8 * j + e;
        part[i] = ks[e];
        part[RD + i] = kx[e];
        part[2 * RD + i] = kn[e];
        part[3 * RD + i] = vs[e];
        part[4 * RD + i] = vx[e];
        part[5 * RD + i] = vn[e];
      }
    }
  }
  if (lanes_share) {
    // the lanes of a warp holding chunk j (lane % D8 == j) combine by shuffles, then lanes
    // [0, D8) write the warp's partials part[w][6][D]: a fixed order, deterministic means
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      for (int o = D8; o < 32; o <<= 1) {
        ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], o);
        vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], o);
        kx[e] = fmaxf(kx[e], __shfl_xor_sync(0xffffffffu, kx[e], o));
        kn[e] = fminf(kn[e], __shfl_xor_sync(0xffffffffu, kn[e], o));
        vx[e] = fmaxf(vx[e], __shfl_xor_sync(0xffffffffu, vx[e], o));
        vn[e] = fminf(vn[e], __shfl_xor_sync(0xffffffffu, vn[e], o));
      }
    }
    if (lane < D8) {
      float* pw = part + w * 6 * D;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        pw[8 * lane + e] = ks[e];
        pw[D + 8 * lane + e] = kx[e];
        pw[2 * D + 8 * lane + e] = kn[e];
        pw[3 * D + 8 * lane + e] = vs[e];
        pw[4 * D + 8 * lane + e] = vx[e];
        pw[5 * D + 8 * lane + e] = vn[e];
      }
    }
  }
  qm = warp_max(qm);
  if (lane == 0) red[0][w] = qm;
  __syncthreads();
  float ak = 0.f, av = 0.f;
  if (t < D) {
    float sk = 0.f, xk = -INFINITY, nk = INFINITY, sv = 0.f, xv = -INFINITY, nv = INFINITY;
    if (lanes_share) {
      for (int ww = 0; ww < 8; ++ww) {
        const float* pw = part + ww * 6 * D;
        sk += pw[t];
        xk = fmaxf(xk, pw[D + t]);
        nk = fminf(nk, pw[2 * D + t]);
        sv += pw[3 * D + t];
        xv = fmaxf(xv, pw[4 * D + t]);
        nv = fminf(nv, pw[5 * D + t]);
      }
    } else {
      const int RD = rpi * D;
      for (int r = 0; r < rpi; ++r) {   // fixed order: deterministic means
        const int i = r * D + t;
        sk += part[i];
        xk = fmaxf(xk, part[RD + i]);
        nk = fminf(nk, part[2 * RD + i]);
        sv += part[3 * RD + i];
        xv = fmaxf(xv, part[4 * RD + i]);
        nv = fminf(nv, part[5 * RD + i]);
      }
    }
    // smooth bit 0 / 1 off: that mean is 0 (no centring, and the maximum is of |k| / |v| itself)
    const float mk = (smooth & 1) ? __fdiv_rn(sk, (float)S) : 0.f, mv = (smooth & 2) ? __fdiv_rn(sv, (float)S) : 0.f;
    stats[(int64_t)head * 2 * Dp + t] = mk;
    stats[(int64_t)head * 2 * Dp + Dp + t] = mv;
    ak = fmaxf(fabsf(xk - mk), fabsf(nk - mk));
    av = fmaxf(fabsf(xv - mv), fabsf(nv - mv));
  } else if (t < Dp) {
    stats[(int64_t)head * 2 * Dp + t] = 0.f;
    stats[(int64_t)head * 2 * Dp + Dp + t] = 0.f;
  }
  ak = warp_max(ak);
  av = warp_max(av);
  if (lane == 0) {
    red[1][w] = ak;
    red[2][w] = av;
  }
  __syncthreads();
  if (t < 3) {
    float m = 0.f;
    for (int i = 0; i < 8; ++i) m = fmaxf(m, red[t][i]);
    atomicMax(reinterpret_cast<unsigned int*>(amax3) + t, __float_as_uint(m));
  }
}

// Head dim 64 form of attn_stats_kernel (the fused route): threads 0-127 take k and |q|, threads
// 128-255 take v, each thread 8 columns of rows t/8 + 16 i, two rows per trip; the lanes of a warp
// that hold the same 8 columns combine by shuffles, the four warps of a tensor through shared
// memory in a fixed order (deterministic means); three CTAs per SM.
__global__ void __launch_bounds__(256, 3) attn_stats64_kernel(const __nv_bfloat16* __restrict__ q,
                                                              const __nv_bfloat16* __restrict__ k,
                                                              const __nv_bfloat16* __restrict__ v, int64_t sb,
                                                              int64_t sh, int64_t ss, int H, int S, int smooth,
                                                              float* __restrict__ stats, float* __restrict__ amax3) {
  __shared__ float part[8][3][64];   // per warp: sum, max, min of its tensor's 64 columns
  __shared__ float qred[4], ared[4];
  const int head = blockIdx.x;
  const int b = head / H, h = head - b * H;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const bool is_v = t >= 128;
  const int tt = t & 127, j = tt & 7;
  const int64_t off = (int64_t)b * sb + (int64_t)h * sh + 8 * j;
  const __nv_bfloat16* x = is_v ? v : k;
  float sm[8], mx[8], mn[8], qm = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    sm[e] = 0.f;
    mx[e] = -INFINITY;
    mn[e] = INFINITY;
  }
  // rows tt/8 + 16 i; the raw 16-byte words of the next pair of rows are loaded before the current
  // pair is accumulated (two pairs of loads in flight per thread), in the same summation order
  auto fetch = [&](int r, uint4* cw, uint4* aw) {
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int rr = r + 16 * m;
      const bool in = rr < S;
      cw[m] = in ? __ldg(reinterpret_cast<const uint4*>(x + off + (int64_t)rr * ss)) : make_uint4(0, 0, 0, 0);
      if (!is_v) aw[m] = in ? __ldg(reinterpret_cast<const uint4*>(q + off + (int64_t)rr * ss)) : make_uint4(0, 0, 0, 0);
    }
  };
  uint4 cw[2], aw[2], cn[2], an[2];
  int r = tt >> 3;
  fetch(r, cw, aw);
  for (; r < S; r += 32) {
    if (r + 32 < S) fetch(r + 32, cn, an);
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      if (r + 16 * m >= S) break;   // fixed summation order per thread: row r, then r + 16
      const uint32_t cv[4] = {cw[m].x, cw[m].y, cw[m].z, cw[m].w}, av[4] = {aw[m].x, aw[m].y, aw[m].z, aw[m].w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float c = (e & 1) ? __uint_as_float(cv[e >> 1] & 0xFFFF0000u) : __uint_as_float(cv[e >> 1] << 16);
        if (!is_v) {
          const float a = (e & 1) ? __uint_as_float(av[e >> 1] & 0xFFFF0000u) : __uint_as_float(av[e >> 1] << 16);
          qm = fmaxf(qm, fabsf(a));
        }
        sm[e] += c;
        mx[e] = fmaxf(mx[e], c);
        mn[e] = fminf(mn[e], c);
      }
    }
    cw[0] = cn[0];
    cw[1] = cn[1];
    aw[0] = an[0];
    aw[1] = an[1];
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) {
#pragma unroll
    for (int o = 8; o < 32; o <<= 1) {
      sm[e] += __shfl_xor_sync(0xffffffffu, sm[e], o);
      mx[e] = fmaxf(mx[e], __shfl_xor_sync(0xffffffffu, mx[e], o));
      mn[e] = fminf(mn[e], __shfl_xor_sync(0xffffffffu, mn[e], o));
    }
  }
  if (lane < 8) {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      part[w][0][8 * lane + e] = sm[e];
      part[w][1][8 * lane + e] = mx[e];
      part[w][2][8 * lane + e] = mn[e];
    }
  }
  qm = warp_max(qm);
  if (lane == 0 && w < 4) qred[w] = qm;
  __syncthreads();
  float am = 0.f;
  if (t < 128) {   // t < 64: column t of k; 64 <= t < 128: column t - 64 of v
    const int c = t & 63, w0 = t < 64 ? 0 : 4;
    float su = 0.f, xx = -INFINITY, nn = INFINITY;
    for (int ww = w0; ww < w0 + 4; ++ww) {
      su += part[ww][0][c];
      xx = fmaxf(xx, part[ww][1][c]);
      nn = fminf(nn, part[ww][2][c]);
    }
    const float mean = (smooth & (t < 64 ? 1 : 2)) ? __fdiv_rn(su, (float)S) : 0.f;   // smooth-K / smooth-V
    stats[(int64_t)head * 128 + t] = mean;
    am = fmaxf(fabsf(xx - mean), fabsf(nn - mean));
  }
  am = warp_max(am);
  if (lane == 0 && w < 4) ared[w] = am;   // warps 0-1: k columns, 2-3: v columns
  __syncthreads();
  if (t < 3) {
    const float m = t == 0 ? fmaxf(fmaxf(qred[0], qred[1]), fmaxf(qred[2], qred[3]))
                           : fmaxf(ared[2 * (t - 1)], ared[2 * (t - 1) + 1]);
    atomicMax(reinterpret_cast<unsigned int*>(amax3) + t, __float_as_uint(m));
  }
}

__global__ void __launch_bounds__(256) attn_prep_kernel(const __nv_bfloat16* __restrict__ q,
                                                        const __nv_bfloat16* __restrict__ k,
                                                        const __nv_bfloat16* __restrict__ v, int64_t sb,
                                                        int64_t sh, int64_t ss, AttnGeom g,
                                                        uint8_t* __restrict__ ws,
                                                        const float* __restrict__ stats,
                                                        const float* __restrict__ amax3) {
  __shared__ float part[2][2048];
  __shared__ float mu[2][128];
  __shared__ float red[8];
  const int bh = blockIdx.x;
  const int b = bh / g.H, h = bh - b * g.H;
  const __nv_bfloat16* qh = q + b * sb + h * sh;
  const __nv_bfloat16* kh = k + b * sb + h * sh;
  const __nv_bfloat16* vh = v + b * sb + h * sh;
  const int S = g.S, D = g.D, D8 = D / 8;
  const int rpi = 256 / D8, active = rpi * D8;
  const int t = threadIdx.x, c8 = t % D8, r0 = t / D8;

  float aq = 0.f, ak = 0.f, av = 0.f;
  if (stats) {   // tensor-wide globals: means and amaxes from attn_stats_kernel
    if (t < D) {
      mu[0][t] = stats[(int64_t)bh * 2 * g.Dp + t];
      mu[1][t] = stats[(int64_t)bh * 2 * g.Dp + g.Dp + t];
    }
    aq = amax3[0];
    ak = amax3[1];
    av = amax3[2];
    __syncthreads();
  } else {
  // pass A: column sums of k and v, amax of q
  float sk[8], sv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) sk[i] = sv[i] = 0.f;
  if (t < active) {
    for (int r = r0; r < S; r += rpi) {
      float a[8], bk[8], bv[8];
      load8(qh + r * ss + c8 * 8, a);
      load8(kh + r * ss + c8 * 8, bk);
      load8(vh + r * ss + c8 * 8, bv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        aq = fmaxf(aq, fabsf(a[i]));
        sk[i] += bk[i];
        sv[i] += bv[i];
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      part[0][r0 * D + c8 * 8 + i] = sk[i];
      part[1][r0 * D + c8 * 8 + i] = sv[i];
    }
  }
  __syncthreads();
  if (t < D) {
    float a = 0.f, bb = 0.f;
    for (int r = 0; r < rpi; ++r) {  // fixed order: deterministic means
      a += part[0][r * D + t];
      bb += part[1][r * D + t];
    }
    mu[0][t] = __fdiv_rn(a, (float)S);
    mu[1][t] = __fdiv_rn(bb, (float)S);
  }
  aq = block_max(aq, red);  // contains __syncthreads: mu visible afterwards

  // pass B: amax of the centred k and v
  if (t < active) {
    for (int r = r0; r < S; r += rpi) {
      float bk[8], bv[8];
      load8(kh + r * ss + c8 * 8, bk);
      load8(vh + r * ss + c8 * 8, bv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ak = fmaxf(ak, fabsf(bk[i] - mu[0][c8 * 8 + i]));
        av = fmaxf(av, fabsf(bv[i] - mu[1][c8 * 8 + i]));
      }
    }
  }
  ak = block_max(ak, red);
  av = block_max(av, red);
  }
  const float gs_q = __fdiv_rn(fmaxf(aq, 1e-12f), 2688.f);
  const float gs_k = __fdiv_rn(fmaxf(ak, 1e-12f), 2688.f);
  const float gs_v = __fdiv_rn(fmaxf(av, 1e-12f), 2688.f);
  float* scal = reinterpret_cast<float*>(ws + g.off_scal) + (int64_t)bh * kScalStride;
  if (t == 0) {
    scal[0] = gs_q;
    scal[1] = gs_k;
    scal[2] = gs_v;
    scal[3] = 0.f;
  }
  if (t < 128) scal[4 + t] = t < D ? mu[1][t] : 0.f;
  const float se_q = __fdiv_rn(1.f, gs_q), se_k = __fdiv_rn(1.f, gs_k), se_v = __fdiv_rn(1.f, gs_v);

  const int lane = t & 31;
  // pass C: Q and K~ along the head dim -> (S_pad, Dp/2) packed + (S_pad x Dp/16) tiled scales
  {
    const int nblk = g.Dp / 16, dblk = D / 16;
    const int ncb = g.Dp / 64;
    const int total = g.S_pad * nblk;
    uint8_t* qp = ws + g.off_q + (int64_t)bh * g.q_head;
    uint8_t* kp = ws + g.off_k + (int64_t)bh * g.q_head;
    uint8_t* qsf = ws + g.off_qsf + (int64_t)bh * g.qsf_head;
    uint8_t* ksf = ws + g.off_ksf + (int64_t)bh * g.qsf_head;
    for (int i0 = t & ~31; i0 < total; i0 += 256) {
      const int i = i0 + lane;
      const int r = i / nblk, bb = i - r * nblk;
      const bool in = i < total;
      const bool valid = in && r < S && bb < dblk;
      uint32_t sfq = 0, sfk = 0;
      uint64_t pq = 0, pk = 0;
      if (valid) {
        float x[16];
        load8(qh + r * ss + bb * 16, x);
        load8(qh + r * ss + bb * 16 + 8, x + 8);
        BlockQ z = quantize_block<false>(x, gs_q, se_q, 0x1p17f);   // raw bf16 values
        pq = z.packed;
        sfq = z.sf;
        load8(kh + r * ss + bb * 16, x);
        load8(kh + r * ss + bb * 16 + 8, x + 8);
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = x[e] - mu[0][bb * 16 + e];
        z = quantize_block<false>(x, gs_k, se_k);
        pk = z.packed;
        sfk = z.sf;
      }
      if (in) {
        *reinterpret_cast<uint64_t*>(qp + (int64_t)r * (g.Dp / 2) + bb * 8) = pq;
        *reinterpret_cast<uint64_t*>(kp + (int64_t)r * (g.Dp / 2) + bb * 8) = pk;
      }
      uint32_t wq = sfq << (8 * (bb & 3)), wk = sfk << (8 * (bb & 3));
      wq |= __shfl_xor_sync(0xffffffffu, wq, 1);
      wq |= __shfl_xor_sync(0xffffffffu, wq, 2);
      wk |= __shfl_xor_sync(0xffffffffu, wk, 1);
      wk |= __shfl_xor_sync(0xffffffffu, wk, 2);
      if (in && (bb & 3) == 0) {
        const int64_t off = sf_swizzle_offset(r, bb, ncb);
        *reinterpret_cast<uint32_t*>(qsf + off) = wq;
        *reinterpret_cast<uint32_t*>(ksf + off) = wk;
      }
    }
  }
  // pass D: V~^T along tokens -> (Dv, S_pad/2) packed + (128 x S_pad/16) tiled scales
  {
    const int nblk = g.S_pad / 16;
    const int ncb = g.S_pad / 64;
    const int total = 128 * nblk;  // scale rows are padded to 128
    uint8_t* vp = ws + g.off_v + (int64_t)bh * g.vt_head;
    uint8_t* vsf = ws + g.off_vsf + (int64_t)bh * g.vsf_head;
    for (int i0 = t & ~31; i0 < total; i0 += 256) {
      const int i = i0 + lane;
      const int d = i / nblk, tb = i - d * nblk;
      const bool in = i < total;
      uint32_t sf = 0;
      uint64_t pv = 0;
      if (in && d < D) {
        float x[16];
        const float m = mu[1][d];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int tok = tb * 16 + e;
          x[e] = tok < S ? __bfloat162float(vh[(int64_t)tok * ss + d]) - m : 0.f;
        }
        BlockQ z = quantize_block<false>(x, gs_v, se_v);
        pv = z.packed;
        sf = z.sf;
      }
      if (in && d < g.Dv) *reinterpret_cast<uint64_t*>(vp + (int64_t)d * (g.S_pad / 2) + tb * 8) = pv;
      uint32_t w = sf << (8 * (tb & 3));
      w |= __shfl_xor_sync(0xffffffffu, w, 1);
      w |= __shfl_xor_sync(0xffffffffu, w, 2);
      if (in && (tb & 3) == 0) *reinterpret_cast<uint32_t*>(vsf + sf_swizzle_offset(d, tb, ncb)) = w;
    }
  }
}

// ---------------------------------------------------------------------------------------
// Kernel 2: attention forward (long sequences).  Persistent: each CTA takes whole heads (the
// B*H heads strided over the grid) and runs all query tiles of a head against that head's K~ and
// V~^T, which are loaded into shared memory once per head.
//   warp 0      loads: K~, V~^T and their scales once per head; Q and its scales per 128-query
//               tile (the next tile's Q is loaded as soon as the current tile's last QK^T MMA has
//               run)
//   warp 1      TMEM allocation, then the MMAs: per 128-key chunk S = Q K~^T into one of two
//               TMEM score buffers (pass 1, then again in pass 2), and O = P V~ per chunk
//   warps 2-9   softmax: two warps per TMEM lane quadrant, each owning 64 of a chunk's 128 key
//               columns.  Pass 1: row max (and min, for a negative scale); the two halves combine
//               through shared memory.  Pass 2: P = exp(s - max) in [0, 1] and its row sums, NVFP4
//               with the fixed global 1/2688 (each half writes its 64 keys' codes and one K64
//               scale word) into one of two P buffers.  Epilogue: O * gs_v / (2688 rowsum) +
//               mean(v) -> bf16.
// Every wait is bounded; a give-up records the device error and unwinds.
// ---------------------------------------------------------------------------------------
VF4_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int DP>
struct AttnCfg {
  static constexpr int DV = DP;
  static constexpr int ROWB = DP / 2;                 // bytes per Q/K row
  static constexpr int KB = DP / 64;                  // K64 blocks of QK^T
  static constexpr int QBYTES = 128 * ROWB;
  static constexpr int VBYTES = DV * 64;              // V~^T chunk: DV rows x 128 keys
  static constexpr int PBYTES = 128 * 64;             // P chunk: 128 rows x 128 keys
  static constexpr uint32_t QK_LAYOUT = DP == 64 ? 6u : 4u;   // SWIZZLE_32B / SWIZZLE_64B
  static constexpr uint32_t QK_SBO = 8 * ROWB;
  // TMEM columns: two score buffers, O, and the scale slots
  static constexpr int T_S = 0, T_O = 256, T_QSF = 256 + DV, T_KSF = T_QSF + 4 * KB;
  static constexpr int T_PSF = T_KSF + 4 * KB, T_VSF = T_PSF + 8;
  static constexpr int TMEM_COLS = 512;
  static constexpr int SOFTMAX_WARPS = 8;
  static constexpr int THREADS = 64 + 32 * SOFTMAX_WARPS;
  static_assert(T_VSF + 8 <= TMEM_COLS, "TMEM overflow");
};

struct AttnSmem {
  uint32_t q, k, v, p, qsf, ksf, vsf, psf, red, bar, total;
};

template <int DP>
static AttnSmem attn_smem_layout(int nc, int S_pad) {
  using C = AttnCfg<DP>;
  AttnSmem s{};
  uint32_t o = 0;
  s.q = o;   o += C::QBYTES;
  s.k = o;   o += nc * C::QBYTES;
  s.v = o;   o += nc * C::VBYTES;
  s.p = o;   o += 2 * C::PBYTES;
  s.qsf = o; o += C::KB * 512;
  s.ksf = o; o += nc * C::KB * 512;
  s.vsf = o; o += (S_pad / 64) * 512;
  s.psf = o; o += 2 * 1024;
  s.red = o; o += 128 * 2 * 8;           // per row and key half: running max and sum
  s.bar = o; o += 256;
  s.total = o + 1024;  // slack for aligning the base to 1024
  return s;
}

template <int DP>
__global__ void __launch_bounds__(AttnCfg<DP>::THREADS, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const AttnGeom g, const uint8_t* __restrict__ ws,
                    const AttnSmem L, float scale, __nv_bfloat16* __restrict__ out, int64_t osb, int64_t osh,
                    int64_t oss) {
  using C = AttnCfg<DP>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar = base + L.bar;
  const uint32_t kv_full = bar, kv_free = bar + 8, q_full = bar + 16, q_free = bar + 24, o_full = bar + 32,
                 o_free = bar + 40, drain = bar + 48;
  auto s_full = [&](int i) { return bar + 56 + 8u * i; };
  auto s_free = [&](int i) { return bar + 72 + 8u * i; };
  auto p_full = [&](int i) { return bar + 88 + 8u * i; };
  auto p_free = [&](int i) { return bar + 104 + 8u * i; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L.bar + 128);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nc = g.nc, S = g.S;
  int* err = &g_attn_err;
  constexpr int NSW = C::SOFTMAX_WARPS;

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_free, 1);
    mbar_init(q_full, 1);
    mbar_init(q_free, 1);
    mbar_init(o_full, 1);
    mbar_init(o_free, NSW);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), NSW);
      mbar_init(p_full(i), NSW);
      mbar_init(p_free(i), 1);
    }
    fence_mbar_init();
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
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
    if (lane == 0) {
      // ------------------------------------------------------------ loads
      const uint32_t qsf_bytes = C::KB * 512, ksf_bytes = nc * C::KB * 512, vsf_bytes = (g.S_pad / 64) * 512;
      uint32_t hc = 0, tcnt = 0;
      bool ok = true;
      for (int64_t bh = blockIdx.x; bh < g.BH && ok; bh += gridDim.x, ++hc) {
        if (!(ok = mbar_wait(kv_free, (hc & 1u) ^ 1u, err, kDevErrTimeoutEmpty))) break;
        mbar_arrive_expect_tx(kv_full, nc * (C::QBYTES + C::VBYTES) + ksf_bytes + vsf_bytes);
        for (int j = 0; j < nc; ++j) {
          tma_load_2d(base + L.k + j * C::QBYTES, &tmK, 0, (int)(bh * g.S_pad + j * 128), kv_full);
          tma_load_2d(base + L.v + j * C::VBYTES, &tmV, j * 64, (int)(bh * C::DV), kv_full);
        }
        bulk_load(base + L.ksf, ws + g.off_ksf + bh * g.qsf_head, ksf_bytes, kv_full);
        bulk_load(base + L.vsf, ws + g.off_vsf + bh * g.vsf_head, vsf_bytes, kv_full);
        for (int qt = 0; qt < nc; ++qt, ++tcnt) {
          if (!(ok = mbar_wait(q_free, (tcnt & 1u) ^ 1u, err, kDevErrTimeoutEmpty))) break;
          mbar_arrive_expect_tx(q_full, C::QBYTES + qsf_bytes);
          tma_load_2d(base + L.q, &tmQ, 0, (int)(bh * g.S_pad + qt * 128), q_full);
          bulk_load(base + L.qsf, ws + g.off_qsf + bh * g.qsf_head + (int64_t)qt * C::KB * 512, qsf_bytes, q_full);
        }
      }
      // our own copies still in flight complete before the CTA retires (bounded)
      if (hc > 0) mbar_wait(kv_full, (hc - 1) & 1u, err, kDevErrTimeoutFull);
      if (tcnt > 0) mbar_wait(q_full, (tcnt - 1) & 1u, err, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issue
      constexpr uint32_t id_s = idesc_mxf4nvf4(128);
      constexpr uint32_t id_o = idesc_mxf4nvf4(C::DV);
      const uint32_t t_o = tmem + C::T_O, t_qsf = tmem + C::T_QSF, t_ksf = tmem + C::T_KSF;
      const uint32_t t_psf = tmem + C::T_PSF, t_vsf = tmem + C::T_VSF;
      uint32_t hc = 0, tcnt = 0, sc = 0, pc = 0;
      bool ok = true;
      auto issue_s = [&](int j) -> bool {   // S chunk j into score buffer sc & 1
        const int b = (int)(sc & 1u);
        if (!mbar_wait(s_free(b), ((sc >> 1) & 1u) ^ 1u, err, kDevErrTimeoutEmpty)) return false;
        tc_fence_after();
        for (int kb = 0; kb < C::KB; ++kb)
          tmem_cp_32x128b_x4(t_ksf + kb * 4, smem_desc(base + L.ksf + (j * C::KB + kb) * 512, 0, 128, 0));
        for (int kb = 0; kb < C::KB; ++kb) {
          const uint64_t ad = smem_desc(base + L.q + kb * 32, 16, C::QK_SBO, C::QK_LAYOUT);
          const uint64_t bd = smem_desc(base + L.k + j * C::QBYTES + kb * 32, 16, C::QK_SBO, C::QK_LAYOUT);
          mma_mxf4nvf4(tmem + C::T_S + 128 * b, ad, bd, id_s, t_qsf + kb * 4, t_ksf + kb * 4, kb > 0 ? 1u : 0u);
        }
        tc_commit(s_full(b));
        ++sc;
        return true;
      };
      for (int64_t bh = blockIdx.x; bh < g.BH && ok; bh += gridDim.x, ++hc) {
        if (!(ok = mbar_wait(kv_full, hc & 1u, err, kDevErrTimeoutFull))) break;
        for (int qt = 0; qt < nc && ok; ++qt, ++tcnt) {
          if (!(ok = mbar_wait(q_full, tcnt & 1u, err, kDevErrTimeoutFull))) break;
          tc_fence_after();
          for (int kb = 0; kb < C::KB; ++kb)
            tmem_cp_32x128b_x4(t_qsf + kb * 4, smem_desc(base + L.qsf + kb * 512, 0, 128, 0));
          // pass 1: scores for the row statistics
          for (int j = 0; j < nc && ok; ++j) ok = issue_s(j);
          // pass 2: scores again, one chunk ahead of the PV products
          if (ok) ok = issue_s(0);
          // O of the previous tile has been read by the softmax warps before it is overwritten
          if (ok) ok = mbar_wait(o_free, (tcnt & 1u) ^ 1u, err, kDevErrTimeoutTmem);
          for (int j = 0; j < nc && ok; ++j) {
            if (j + 1 < nc) {
              if (!(ok = issue_s(j + 1))) break;
            } else {
              tc_commit(q_free);   // every QK^T of this tile issued: Q's buffers free once they ran
            }
            const int pb = (int)(pc & 1u);
            if (!(ok = mbar_wait(p_full(pb), (pc >> 1) & 1u, err, kDevErrTimeoutFull))) break;
            tc_fence_after();
            for (int kb = 0; kb < 2; ++kb) {
              tmem_cp_32x128b_x4(t_psf + kb * 4, smem_desc(base + L.psf + pb * 1024 + kb * 512, 0, 128, 0));
              tmem_cp_32x128b_x4(t_vsf + kb * 4, smem_desc(base + L.vsf + (2 * j + kb) * 512, 0, 128, 0));
            }
            const uint32_t pbuf = base + L.p + pb * C::PBYTES;
            for (int kb = 0; kb < 2; ++kb) {
              const uint64_t ad = smem_desc(pbuf + kb * 256, 128, 512, 0);           // interleaved, no swizzle
              const uint64_t bd = smem_desc(base + L.v + j * C::VBYTES + kb * 32, 16, 512, 4);  // SWIZZLE_64B
              mma_mxf4nvf4(t_o, ad, bd, id_o, t_psf + kb * 4, t_vsf + kb * 4, (j > 0 || kb > 0) ? 1u : 0u);
            }
            tc_commit(p_free(pb));
            ++pc;
          }
          if (ok) tc_commit(o_full);
        }
        if (ok) tc_commit(kv_free);   // this head's K~ / V~ no longer read once these MMAs ran
      }
      tc_commit(drain);
      mbar_wait(drain, 0, err, kDevErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;               // key columns [64 half, 64 half + 64) of a chunk
    const int r = quad * 32 + lane;                 // row of the query tile == TMEM lane
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    float2* red = reinterpret_cast<float2*>(gbase + L.red);   // [half][128 rows]
    uint32_t tcnt = 0, sc = 0, pc = 0;
    bool ok = true;
    uint32_t v[64];
    auto load_s = [&]() -> bool {   // this warp's 64 columns of the next score chunk
      const int b = (int)(sc & 1u);
      if (!mbar_wait(s_full(b), (sc >> 1) & 1u, err, kDevErrTimeoutFull)) return false;
      tc_fence_after();
      const uint32_t ta = tmem + lane_addr + C::T_S + 128 * b + 64 * half;
      tmem_ld_32x32b_x32(ta, v);
      tmem_ld_32x32b_x32(ta + 32, v + 32);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free(b));
      ++sc;
      return true;
    };
    for (int64_t bh = blockIdx.x; bh < g.BH && ok; bh += gridDim.x) {
      const float* scal = reinterpret_cast<const float*>(ws + g.off_scal) + bh * kScalStride;
      const float cexp = scal[0] * scal[1] * scale * 1.4426950408889634f;
      for (int qt = 0; qt < nc && ok; ++qt, ++tcnt) {
        const int tq = qt * 128 + r;                // query token
        // pass 1: the row's largest and smallest raw score over this warp's columns; fl(x * cexp) is
        // monotone in x, so the row max of the scaled scores is (cexp >= 0 ? max : min) * cexp exactly
        float m = -INFINITY, mn = INFINITY;
        for (int j = 0; j < nc && ok; ++j) {
          if (!(ok = load_s())) break;
          const int nvalid = min(64, S - j * 128 - 64 * half);   // may be <= 0 for the last chunk
          if (nvalid >= 64) {
#pragma unroll
            for (int i = 0; i < 64; i += 2) {
              m = max3f(m, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
              mn = min3f(mn, __uint_as_float(v[i]), __uint_as_float(v[i + 1]));
            }
          } else {
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (i < nvalid) {
                m = fmaxf(m, __uint_as_float(v[i]));
                mn = fminf(mn, __uint_as_float(v[i]));
              }
          }
        }
        // combine the two halves of the row
        red[half * 128 + r] = make_float2(m, mn);
        named_bar_sync(1 + quad, 64);
        const float2 o2 = red[(1 - half) * 128 + r];
        const float mr = (cexp >= 0.f ? fmaxf(m, o2.x) : fminf(mn, o2.y)) * cexp;
        named_bar_sync(1 + quad, 64);               // both halves have read red before it is reused
        float l = 0.f;
        // pass 2: P = exp(s - max) in [0, 1] (exactly 1 at the row max), its row sums, P -> NVFP4 (fixed
        // global 1/2688) into the P buffers; the 1/rowsum is applied to O
        for (int j = 0; j < nc && ok; ++j) {
          if (!(ok = load_s())) break;
          const int nvalid = min(64, S - j * 128 - 64 * half);
          const int pb = (int)(pc & 1u);
          if (!(ok = mbar_wait(p_free(pb), ((pc >> 1) & 1u) ^ 1u, err, kDevErrTimeoutEmpty))) break;
          uint8_t* pbuf = gbase + L.p + pb * C::PBYTES;
          uint32_t sfw = 0u;
#pragma unroll
          for (int blk = 0; blk < 4; ++blk) {
            uint64_t codes = 0;
            if (blk * 16 < nvalid) {
              float pv[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) {
                const int i = blk * 16 + e;
                pv[e] = i < nvalid ? ex2_approx(__fmaf_rn(__uint_as_float(v[i]), cexp, -mr)) : 0.f;
                l += pv[e];
              }
              float amax = 0.f;
#pragma unroll
              for (int e = 0; e < 16; ++e) amax = fmaxf(amax, pv[e]);
              float dec;
              const uint32_t sf = six_scale(amax, 2688.f, kInv2688, &dec);
              codes = encode16_fast(pv, dec);
              sfw |= sf << (8 * blk);
            }
            // interleaved K-major core matrices: (row group, 16-byte K chunk) at rg*512 + kc*128 + (r%8)*16
            const int gb = 4 * half + blk;          // 16-key block within the 128-key chunk
            *reinterpret_cast<uint64_t*>(pbuf + (r >> 3) * 512 + (gb >> 1) * 128 + (r & 7) * 16 + (gb & 1) * 8) = codes;
          }
          // this half's four blocks are the K64 block `half` of the chunk: one scale word
          *reinterpret_cast<uint32_t*>(gbase + L.psf + pb * 1024 + half * 512 + (r & 31) * 16 + (r >> 5) * 4) = sfw;
          fence_async_shared();
          __syncwarp();
          if (lane == 0) mbar_arrive(p_full(pb));
          ++pc;
        }
        red[half * 128 + r].x = l;
        named_bar_sync(1 + quad, 64);
        const float inv_l = 1.0f / (l + red[(1 - half) * 128 + r].x);
        named_bar_sync(1 + quad, 64);               // read before the next tile's pass 1 rewrites red
        // epilogue: this warp's half of the head dim
        if (ok && (ok = mbar_wait(o_full, tcnt & 1u, err, kDevErrTimeoutTmem))) {
          tc_fence_after();
          constexpr int DH = C::DV / 2;
          uint32_t ov[DH];
#pragma unroll
          for (int c = 0; c < DH / 32; ++c)
            tmem_ld_32x32b_x32(tmem + lane_addr + C::T_O + half * DH + c * 32, ov + c * 32);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(o_free);
          if (tq < S) {
            const float ao = kInv2688 * scal[2] * inv_l;
            const int b = (int)(bh / g.H), h = (int)(bh - (int64_t)b * g.H);
            __nv_bfloat16* o = out + b * osb + (int64_t)tq * oss + h * osh + half * DH;
#pragma unroll
            for (int d8 = 0; d8 < DH / 8; ++d8) {
              if (half * DH + d8 * 8 < g.D) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int d = d8 * 8 + 2 * e;
                  __nv_bfloat162 hv = __floats2bfloat162_rn(__uint_as_float(ov[d]) * ao + scal[4 + half * DH + d],
                                                            __uint_as_float(ov[d + 1]) * ao + scal[4 + half * DH + d + 1]);
                  w[e] = *reinterpret_cast<uint32_t*>(&hv);
                }
                *reinterpret_cast<uint4*>(o + d8 * 8) = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ---------------------------------------------------------------------------------------
// Fused attention for head dim <= 64 and S <= 320 (ViT-S/16, ViT-B/16, ViT-L/14): one kernel,
// no workspace.  Persistent CTAs (one per SM, 18 warps) walk over the B*H heads.  Per head:
//   warp 0      TMA loads of the head's q, k, v rows (bf16, 128-byte swizzle) into "raw"
//   warps 2-17  prep: column means of k and v, amax of q, k~ = k - mean, v~ = v - mean ->
//               per-head globals; Q and K~ (blocks along d) and V~^T (blocks along tokens) to
//               NVFP4 in shared memory, in the MMA's K-major core-matrix layout (8 rows x 16
//               bytes, no swizzle), with their scales in tcgen05.cp atoms.  The raw buffer is
//               released here, so the next head's loads overlap this head's tiles.
//   per 128-query tile:
//     warp 1      S = Q K~^T: mxf4nvf4 MMAs over key chunks of 256/128/64 into TMEM
//     warps 2-17  (TMEM lane quadrant x key slice) pass 1: row max; pass 2: P = exp(S - max)
//                 in [0, 1] (row max exactly 1), row sums, P -> NVFP4 (fixed global 1/2688)
//     warp 1      O = P V~ (mxf4nvf4, K = keys) into TMEM
//     warps 2-17  out = O * gs_v / (2688 * rowsum) + mean(v) -> bf16 -> TMA store
// P is quantized unnormalised and the 1/rowsum applied to O (the reference normalises P first;
// with the fixed P global both are quantizations of the same probabilities).
// Named barriers: 1 = all 16 compute warps, 2 + q = the four warps of TMEM lane quadrant q.
// ---------------------------------------------------------------------------------------
#ifndef VF4_ATTN_SLICES
#define VF4_ATTN_SLICES 3
#endif
constexpr int kSlices = VF4_ATTN_SLICES;                 // compute warps per TMEM lane quadrant
constexpr int kFusedCompute = 4 * kSlices, kFusedWarps = kFusedCompute + 2, kCT = 32 * kFusedCompute;
// TMEM columns: S (<= 320 keys), two O buffers (tile t's PV overlaps tile t+1's softmax), scales
constexpr uint32_t kFusedTmemS = 0, kFusedTmemO = 320, kFusedTmemQsf = 448, kFusedTmemKsf = 452,
                   kFusedTmemPsf = 464, kFusedTmemVsf = 484;

struct FusedGeom {
  int B, H, S, D;
  int nq, skp;          // query tiles of 128; keys padded to a multiple of 64
  int box_rows, nbox;   // raw TMA boxes per tensor
  int heads;
  int qkv_hs, out_hs;   // tensor-map dimension order (d, h, s, b) instead of (d, s, h, b)
  float scale;
  const float* stats;   // per-head means (tensor-wide globals) or NULL (per-head globals)
  const float* amax3;
  const uint8_t* images;   // packed route: per-head operand images written by attn_pack_kernel
  // In the packed route fq .. sfv are offsets inside an operand image (two image buffers at
  // img[0], img[1]; the image's last 512 bytes hold gs_q, gs_k, gs_v and mean(v)); otherwise they
  // are offsets from the shared-memory base after the raw q / k / v buffers.
  uint32_t raw_q, raw_k, raw_v, fq, fk, fv, sfq, sfk, sfv, fp, sfp, zero_end, stg, red, bar, total;
  uint32_t img[2], img_bytes, img_scal;
};

static FusedGeom make_fused_geom(int64_t B, int64_t H, int64_t S, int64_t D, float scale, bool packed = false) {
  FusedGeom g{};
  g.B = (int)B;
  g.H = (int)H;
  g.S = (int)S;
  g.D = (int)D;
  g.nq = (int)((S + 127) / 128);
  g.skp = (int)((S + 63) / 64 * 64);
  g.nbox = S <= 256 ? 1 : 2;
  g.box_rows = (int)align_up((S + g.nbox - 1) / g.nbox, 8);
  g.heads = (int)(B * H);
  g.scale = scale;
  const uint32_t rawb = packed ? 0u : (uint32_t)(g.nbox * g.box_rows * 128);
  uint32_t o = 0;
  g.raw_q = o; o += rawb;
  g.raw_k = o; o += rawb;
  g.raw_v = o; o += rawb;
  const uint32_t ops0 = o;
  g.fq = o;  o += (uint32_t)g.nq * 4096u;
  g.fk = o;  o += (uint32_t)g.skp * 32u;
  g.fv = o;  o += (uint32_t)g.skp * 32u;
  g.sfq = o; o += (uint32_t)g.nq * 512u;
  g.sfk = o; o += (uint32_t)((g.skp + 127) / 128) * 512u;
  g.sfv = o; o += (uint32_t)(g.skp / 64) * 512u;
  if (packed) {   // operand offsets become image-relative; two images, then the P buffers
    g.img_scal = o - ops0;
    g.img_bytes = (uint32_t)align_up(g.img_scal + 512u, 1024);
    for (uint32_t* f : {&g.fq, &g.fk, &g.fv, &g.sfq, &g.sfk, &g.sfv}) *f -= ops0;
    g.img[0] = ops0;
    g.img[1] = ops0 + g.img_bytes;
    o = ops0 + 2 * g.img_bytes;
  }
  g.fp = o;  o += (uint32_t)g.skp * 64u;
  g.sfp = o; o += (uint32_t)(g.skp / 64) * 512u;
  g.zero_end = o;
  o = (uint32_t)align_up(o, 1024);
  g.stg = o; o += 4 * 4096;
  g.red = o; o += 15104;
  g.bar = o; o += 128;
  g.total = o + 1024;
  return g;
}

static bool fused_ok(int64_t S, int64_t D) {
  if (D != 64 || S > 320) return false;
  return make_fused_geom(1, 1, S, D, 1.f).total <= 227u * 1024u;
}

static bool packed_ok(int64_t S, int64_t D) {
  return fused_ok(S, D) && make_fused_geom(1, 1, S, D, 1.f, true).total <= 227u * 1024u;
}

// 8 bf16 of row s, 16-byte chunk j (elements 8j..8j+7) of a 128-byte-swizzled raw tile, as fp32.
VF4_DEV void raw_load8(const uint8_t* raw, int s, int j, float* v) {
  const uint4 a = *reinterpret_cast<const uint4*>(raw + s * 128 + ((j ^ (s & 7)) << 4));
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

VF4_DEV float raw_elem(const uint8_t* raw, int s, int d) {
  const uint16_t b = *reinterpret_cast<const uint16_t*>(raw + s * 128 + (((d >> 3) ^ (s & 7)) << 4) + (d & 7) * 2);
  return __uint_as_float((uint32_t)b << 16);
}

// byte offset of (row, 8-byte half-chunk h) in a K-major core-matrix operand with sbo bytes per
// 8-row group: 16-byte chunk h/2 of the row, half h%2
VF4_DEV uint32_t cm_off(int row, int h, uint32_t sbo) {
  return (uint32_t)(row >> 3) * sbo + (uint32_t)(h >> 1) * 128u + (uint32_t)(row & 7) * 16u + (uint32_t)(h & 1) * 8u;
}

// scale-factor atom offset of (row, scale column c) for 128-row atoms of 4 columns
VF4_DEV uint32_t sf_atom_off(int row, int c) {
  return (uint32_t)(row >> 7) * 512u + (uint32_t)(row & 31) * 16u + (uint32_t)((row >> 5) & 3) * 4u + (uint32_t)c;
}

template <bool kPacked>
__global__ void __launch_bounds__(kFusedWarps * 32, 1)
    attn_fused_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                      const FusedGeom g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (base - raw0);
  const uint32_t bar = base + g.bar;
  const uint32_t raw_full = bar, raw_free = bar + 8, ops_ready = bar + 16, s_full = bar + 24, s_free = bar + 32,
                 p_full = bar + 40, drain = bar + 80;
  auto o_full = [&](int ob) { return bar + 48 + 8u * ob; };   // per O buffer
  auto o_free = [&](int ob) { return bar + 64 + 8u * ob; };
  auto img_full = [&](int i) { return bar + 96 + 8u * i; };    // packed route: operand image i landed
  auto img_free = [&](int i) { return bar + 112 + 8u * i; };   // packed route: image i no longer read
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gb + g.bar + 88);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbo_kv = (uint32_t)(g.skp / 32) * 128u;   // bytes per 8-row group of P and V~^T
  int* err = &g_attn_err;

  if (warp == 0 && lane == 0) {
    mbar_init(raw_full, 1);
    mbar_init(raw_free, kFusedCompute);
    mbar_init(ops_ready, kFusedCompute);
    mbar_init(s_full, 1);
    mbar_init(s_free, kFusedCompute);
    mbar_init(p_full, kFusedCompute);
    for (int ob = 0; ob < 2; ++ob) {
      mbar_init(o_full(ob), 1);
      mbar_init(o_free(ob), kFusedCompute);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(img_full(i), 1);
      mbar_init(img_free(i), kFusedCompute);
    }
    fence_mbar_init();
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    tma_prefetch(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp >= 2) {
    // scale atoms and P codes start at zero: padding keys, rows and head-dim columns stay zero
    for (uint32_t o = (kPacked ? g.fp : g.sfq) + 16u * (threadIdx.x - 64); o < g.zero_end; o += 16u * kCT)
      *reinterpret_cast<uint4*>(gb + o) = make_uint4(0, 0, 0, 0);
  }
  fence_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    if constexpr (kPacked) {
      // ---------------------------------------------------------- operand images (packed route)
      if (lane == 0) {
        int hi = 0;
        for (int head = blockIdx.x; head < g.heads; head += gridDim.x, ++hi) {
          const int ib = hi & 1;
          if (hi >= 2 && !mbar_wait(img_free(ib), (uint32_t)((hi >> 1) - 1) & 1u, err, kDevErrTimeoutEmpty)) break;
          mbar_arrive_expect_tx(img_full(ib), g.img_bytes);
          const uint8_t* src = g.images + (int64_t)head * g.img_bytes;
          for (uint32_t o = 0; o < g.img_bytes; o += 8192u) {
            const uint32_t n = g.img_bytes - o < 8192u ? g.img_bytes - o : 8192u;
            bulk_load(base + g.img[ib] + o, src + o, n, img_full(ib));
          }
        }
        for (int k = hi - 2 < 0 ? 0 : hi - 2; k < hi; ++k)   // own copies landed
          mbar_wait(img_full(k & 1), (uint32_t)(k >> 1) & 1u, err, kDevErrTimeoutFull);
      }
    } else if (lane == 0) {
      // ---------------------------------------------------------- raw loads
      const uint32_t bytes = 3u * (uint32_t)(g.nbox * g.box_rows) * 128u;
      int hi = 0;
      for (int head = blockIdx.x; head < g.heads; head += gridDim.x, ++hi) {
        if (hi > 0 && !mbar_wait(raw_free, (uint32_t)(hi - 1) & 1u, err, kDevErrTimeoutEmpty)) break;
        const int b = head / g.H, h = head - b * g.H;
        mbar_arrive_expect_tx(raw_full, bytes);
        for (int j = 0; j < g.nbox; ++j) {
          const uint32_t off = (uint32_t)(j * g.box_rows) * 128u;
          const int c1 = g.qkv_hs ? h : j * g.box_rows, c2 = g.qkv_hs ? j * g.box_rows : h;
          tma_load_4d(base + g.raw_q + off, &tmQ, 0, c1, c2, b, raw_full);
          tma_load_4d(base + g.raw_k + off, &tmK, 0, c1, c2, b, raw_full);
          tma_load_4d(base + g.raw_v + off, &tmV, 0, c1, c2, b, raw_full);
        }
      }
      if (hi > 0) mbar_wait(raw_full, (uint32_t)(hi - 1) & 1u, err, kDevErrTimeoutFull);   // own copies landed
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    bool ok = true;
    int hi = 0, it = 0;
    const uint32_t t_qsf = tmem + kFusedTmemQsf, t_ksf = tmem + kFusedTmemKsf;
    const uint32_t t_psf = tmem + kFusedTmemPsf, t_vsf = tmem + kFusedTmemVsf;
    const int nkb = g.skp / 64;
    for (int head = blockIdx.x; head < g.heads && ok; head += gridDim.x, ++hi) {
      if (kPacked ? !mbar_wait(img_full(hi & 1), (uint32_t)(hi >> 1) & 1u, err, kDevErrTimeoutFull)
                  : !mbar_wait(ops_ready, (uint32_t)hi & 1u, err, kDevErrTimeoutFull))
        break;
      tc_fence_after();
      const uint32_t opb = kPacked ? base + g.img[hi & 1] : base;   // operand base of this head
      if (lane == 0) {
        for (int a = 0; a < (g.skp + 127) / 128; ++a)
          tmem_cp_32x128b_x4(t_ksf + 4 * a, smem_desc(opb + g.sfk + 512 * a, 0, 128, 0));
        for (int kb = 0; kb < nkb; ++kb)
          tmem_cp_32x128b_x4(t_vsf + 4 * kb, smem_desc(opb + g.sfv + 512 * kb, 0, 128, 0));
      }
      __syncwarp();
      for (int t = 0; t < g.nq; ++t, ++it) {
        if (it > 0 && !mbar_wait(s_free, (uint32_t)(it - 1) & 1u, err, kDevErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          tmem_cp_32x128b_x4(t_qsf, smem_desc(opb + g.sfq + 512 * t, 0, 128, 0));
          const uint64_t ad = smem_desc(opb + g.fq + 4096u * t, 128, 256, 0);
          for (int n0 = 0; n0 < g.skp;) {
            const int rem = g.skp - n0;
            const int n = rem >= 256 ? 256 : (rem >= 128 ? 128 : 64);
            const uint64_t bd = smem_desc(opb + g.fk + (uint32_t)(n0 / 8) * 256u, 128, 256, 0);
            mma_mxf4nvf4(tmem + kFusedTmemS + n0, ad, bd, idesc_mxf4nvf4((uint32_t)n), t_qsf, t_ksf + (n0 / 128) * 4,
                         0u);
            n0 += n;
          }
          tc_commit(s_full);
        }
        __syncwarp();
        const int ob = it & 1, use = it >> 1;
        if (!mbar_wait(p_full, (uint32_t)it & 1u, err, kDevErrTimeoutFull) ||
            (use > 0 && !mbar_wait(o_free(ob), (uint32_t)(use - 1) & 1u, err, kDevErrTimeoutEmpty))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t t_o = tmem + kFusedTmemO + 64u * ob;
          for (int kb = 0; kb < nkb; ++kb) {
            tmem_cp_32x128b_x4(t_psf + 4 * kb, smem_desc(base + g.sfp + 512 * kb, 0, 128, 0));
            mma_mxf4nvf4(t_o, smem_desc(base + g.fp + 256u * kb, 128, sbo_kv, 0),
                         smem_desc(opb + g.fv + 256u * kb, 128, sbo_kv, 0), idesc_mxf4nvf4(64), t_psf + 4 * kb,
                         t_vsf + 4 * kb, kb > 0 ? 1u : 0u);
          }
          tc_commit(o_full(ob));
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      tc_commit(drain);
      mbar_wait(drain, 0, err, kDevErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ prep, softmax, epilogue
    const int cw = warp - 2;           // compute warp 0..15
    const int qd = warp & 3;           // TMEM lane quadrant this warp may access
    const int cs = cw >> 2;            // key slice 0..3
    const int ct = threadIdx.x - 64;   // compute thread 0..511
    const uint32_t qbar = 2u + (uint32_t)qd;
    float* red = reinterpret_cast<float*>(gb + g.red);
    float* red_kv = red;               // [2][16][64] column partial sums of k and v
    float* red_m = red + 2048;         // [4][128] row max per key slice
    float* red_l = red + 2560;         // [2][4][128] row sum per key slice, per O buffer
    float* mu = red + 3584;            // [2][64] means of k and v
    float* wmax = red + 3712;          // [3][16] per-warp amax of q, k~, v~
    float* scal = red + 3760;          // gs_q, gs_k, gs_v, 1/gs_q, 1/gs_k, 1/gs_v
    const uint8_t* rq = gb + g.raw_q;
    const uint8_t* rk = gb + g.raw_k;
    const uint8_t* rv = gb + g.raw_v;
    const int S = g.S, D = g.D;
    const int nvb = (S + 15) / 16;                      // key blocks holding real keys
    const int b0 = cs * nvb / kSlices, b1 = (cs + 1) * nvb / kSlices;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const int r = qd * 32 + lane;                       // tile row == TMEM lane
    bool ok = true;
    int hi = 0, it = 0;
    for (int head = blockIdx.x; head < g.heads; head += gridDim.x, ++hi) {
      const int b = head / g.H, h = head - b * g.H;
      float gq, gk, gv;
      const float* muv;   // mean(v) of this head
      if constexpr (kPacked) {
        if (ok) ok = mbar_wait(img_full(hi & 1), (uint32_t)(hi >> 1) & 1u, err, kDevErrTimeoutFull);
        const float* sc = reinterpret_cast<const float*>(gb + g.img[hi & 1] + g.img_scal);
        gq = sc[0];
        gk = sc[1];
        gv = sc[2];
        muv = sc + 64;
      } else {
      if (ok) ok = mbar_wait(raw_full, (uint32_t)hi & 1u, err, kDevErrTimeoutFull);
      if (g.stats) {
        // tensor-wide globals: this head's means and the global maxima were computed beforehand
        // (the first barrier: every warp has finished the previous head's epilogue, which reads mu)
        named_bar_sync(1, kCT);
        if (ct < 128) mu[ct] = g.stats[(int64_t)head * 128 + ct];
        if (ct < 3) {
          const float gsv = __fdiv_rn(fmaxf(g.amax3[ct], 1e-12f), 2688.f);
          scal[ct] = gsv;
          scal[3 + ct] = __fdiv_rn(1.0f, gsv);
        }
        named_bar_sync(1, kCT);
      } else {
      // ---- prep 1: column sums of k and v, amax of q (chunk j = ct % 8, rows ct/8 + 64i)
      {
        const int j = ct & 7;
        float ks[8], vs[8], qm = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) ks[e] = vs[e] = 0.f;
        if (ok) {
          for (int s = ct >> 3; s < S; s += kCT / 8) {
            float a[8];
            raw_load8(rq, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) qm = fmaxf(qm, fabsf(a[e]));
            raw_load8(rk, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) ks[e] += a[e];
            raw_load8(rv, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) vs[e] += a[e];
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], 8);
          ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], 16);
          vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], 8);
          vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], 16);
        }
        qm = warp_max(qm);
        if (lane < 8) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            red_kv[cw * 64 + 8 * lane + e] = ks[e];
            red_kv[(kFusedCompute + cw) * 64 + 8 * lane + e] = vs[e];
          }
        }
        if (lane == 0) wmax[cw] = qm;
      }
      named_bar_sync(1, kCT);
      if (ct < 128) {
        const int which = ct >> 6, d = ct & 63;
        float sum = 0.f;
        for (int w = 0; w < kFusedCompute; ++w) sum += red_kv[(which * kFusedCompute + w) * 64 + d];   // fixed order
        mu[which * 64 + d] = __fdiv_rn(sum, (float)S);
      }
      named_bar_sync(1, kCT);
      // ---- prep 2: amax of k - mean and v - mean
      {
        const int j = ct & 7;
        float km = 0.f, vm = 0.f;
        if (ok) {
          for (int s = ct >> 3; s < S; s += kCT / 8) {
            float a[8];
            raw_load8(rk, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) km = fmaxf(km, fabsf(a[e] - mu[8 * j + e]));
            raw_load8(rv, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) vm = fmaxf(vm, fabsf(a[e] - mu[64 + 8 * j + e]));
          }
        }
        km = warp_max(km);
        vm = warp_max(vm);
        if (lane == 0) {
          wmax[16 + cw] = km;
          wmax[32 + cw] = vm;
        }
      }
      named_bar_sync(1, kCT);
      if (ct == 0) {
        float am[3] = {0.f, 0.f, 0.f};
        for (int w = 0; w < kFusedCompute; ++w)
          for (int i = 0; i < 3; ++i) am[i] = fmaxf(am[i], wmax[16 * i + w]);
        for (int i = 0; i < 3; ++i) {
          const float gsv = __fdiv_rn(fmaxf(am[i], 1e-12f), 2688.f);
          scal[i] = gsv;
          scal[3 + i] = __fdiv_rn(1.0f, gsv);
        }
      }
      named_bar_sync(1, kCT);
      }
      gq = scal[0];
      gk = scal[1];
      gv = scal[2];
      muv = mu + 64;
      // ---- prep 3: NVFP4 operands.  Q rows [0, 128 nq) and K~ rows [0, skp): 4 column blocks
      // per row, lane quads = one row (their 4 scale bytes merge into one word).  Two items per
      // loop trip so the two quantization chains interleave (the loop bounds are multiples of 32:
      // whole warps take the same branch, as the lane-quad shuffles need).
      auto qk_block = [&](int i, const uint8_t* raw, uint32_t fo, uint32_t so, bool centre, float gs, float se,
                          float dec_max) {
        const int s = i >> 2, cb = i & 3;
        uint64_t codes = 0;
        uint32_t sf = 0;
        if (ok && s < S && cb * 16 < D) {
          float x[16];
          raw_load8(raw, s, 2 * cb, x);
          raw_load8(raw, s, 2 * cb + 1, x + 8);
          if (centre) {
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] -= mu[16 * cb + e];
          }
          const BlockQ z = quantize_block<false>(x, gs, se, dec_max);
          codes = z.packed;
          sf = z.sf;
        }
        *reinterpret_cast<uint64_t*>(gb + fo + cm_off(s, cb, 256)) = codes;
        uint32_t w = sf << (8 * cb);
        w |= __shfl_xor_sync(0xffffffffu, w, 1);
        w |= __shfl_xor_sync(0xffffffffu, w, 2);
        if (cb == 0) *reinterpret_cast<uint32_t*>(gb + so + sf_atom_off(s, 0)) = w;
      };
      for (int i = ct; i < g.nq * 512; i += 2 * kCT) {
        qk_block(i, rq, g.fq, g.sfq, false, gq, scal[3], 0x1p17f);   // raw bf16 values
        if (i + kCT < g.nq * 512) qk_block(i + kCT, rq, g.fq, g.sfq, false, gq, scal[3], 0x1p17f);
      }
      for (int i = ct; i < g.skp * 4; i += 2 * kCT) {
        qk_block(i, rk, g.fk, g.sfk, true, gk, scal[4], 2.0f);
        if (i + kCT < g.skp * 4) qk_block(i + kCT, rk, g.fk, g.sfk, true, gk, scal[4], 2.0f);
      }
      // V~^T rows d in [0, 64), token blocks tb in [0, skp/16); a warp covers 32 consecutive d of one
      // token block, so its raw reads of a token row are 64 contiguous bytes (no bank conflicts)
      {
        const int ntb = g.skp / 16;
        auto v_block = [&](int i) {
          const int tb = i >> 6, d = i & 63;
          uint64_t codes = 0;
          uint32_t sf = 0;
          if (ok && d < D && tb * 16 < S) {
            float x[16];
            const float m = mu[64 + d];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              const int s = tb * 16 + e;
              x[e] = s < S ? raw_elem(rv, s, d) - m : 0.f;
            }
            const BlockQ z = quantize_block<false>(x, gv, scal[5]);
            codes = z.packed;
            sf = z.sf;
          }
          *reinterpret_cast<uint64_t*>(gb + g.fv + cm_off(d, tb, sbo_kv)) = codes;
          gb[g.sfv + (uint32_t)(tb >> 2) * 512u + sf_atom_off(d, tb & 3)] = (uint8_t)sf;
        };
        for (int i = ct; i < 64 * ntb; i += 2 * kCT) {
          v_block(i);
          if (i + kCT < 64 * ntb) v_block(i + kCT);
        }
      }
      fence_async_shared();   // operand writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(ops_ready);
        mbar_arrive(raw_free);
      }
      }
      const float cexp = gq * gk * g.scale * 1.4426950408889634f;
      const float ofac = gv * kInv2688;
      // epilogue of tile (global index itt, local index tl): O rows of this quadrant, the slice's
      // 8-column chunks [c0, c1) of the head dim; O(itt) is complete (o_full waited by the caller)
      const int c0 = cs * 8 / kSlices, c1 = (cs + 1) * 8 / kSlices;
      auto epilogue = [&](int itt, int tl) {
        const bool act = ok && tl * 128 + qd * 32 < S;
        const int ob = itt & 1;
        constexpr int kMaxChunks = (8 + kSlices - 1) / kSlices;
        uint32_t ov[kMaxChunks][8];
        if (act) {
#pragma unroll
          for (int k = 0; k < kMaxChunks; ++k)
            if (c0 + k < c1) tmem_ld_32x32b_x8(tmem + lane_base + kFusedTmemO + 64u * ob + 8 * (c0 + k), ov[k]);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_free(ob));
        if (cs == 0 && lane == 0) bulk_wait_read();   // this quadrant's previous store left the staging
        named_bar_sync(qbar, 32 * kSlices);                     // also publishes red_l
        uint8_t* stg = gb + g.stg + qd * 4096 + lane * 128;
        if (act) {
          const float* rl = red_l + ob * (kSlices * 128);
          float lsum = 0.f;
#pragma unroll
          for (int c = 0; c < kSlices; ++c) lsum += rl[c * 128 + r];
          const float f = ofac / lsum;
#pragma unroll
          for (int k = 0; k < kMaxChunks; ++k) {
            const int c = c0 + k;
            if (c < c1) {
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int d = 8 * c + 2 * i;
                __nv_bfloat162 hv = __floats2bfloat162_rn(__fmaf_rn(__uint_as_float(ov[k][2 * i]), f, muv[d]),
                                                          __fmaf_rn(__uint_as_float(ov[k][2 * i + 1]), f, muv[d + 1]));
                w[i] = *reinterpret_cast<uint32_t*>(&hv);
              }
              *reinterpret_cast<uint4*>(stg + ((c ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
        fence_async_shared();
        named_bar_sync(qbar, 32 * kSlices);
        if (act && cs == 0 && lane == 0) {
          const int row = tl * 128 + qd * 32;
          tma_store_4d(&tmO, base + g.stg + qd * 4096, 0, g.out_hs ? h : row, g.out_hs ? row : h, b);
          bulk_commit();
        }
      };
      // ---- query tiles: softmax of tile t overlaps the PV MMA of tile t - 1, whose epilogue
      // follows (two O buffers); the head's last epilogue runs before the next head's prep
      const unsigned long long c2 = f32x2_pack(cexp, cexp);
      for (int t = 0; t < g.nq; ++t, ++it) {
        const bool active = ok && t * 128 + qd * 32 < S;
        if (ok) ok = mbar_wait(s_full, (uint32_t)it & 1u, err, kDevErrTimeoutFull);
        tc_fence_after();
        // key blocks of this warp: [b0, bu) need no masking, block bu (if < b1) holds the last real
        // key and padding; unmasked blocks go two per TMEM load so their chains interleave
        const int bu = (b1 == nvb && (S & 15)) ? b1 - 1 : b1;
        const uint32_t srow = tmem + lane_base + kFusedTmemS;
        // pass 1: row max over this warp's key blocks
        float m = -INFINITY;
        if (active && ok) {
          int bk = b0;
          for (; bk + 1 < bu; bk += 2) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(srow + 16 * bk, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) m = fmaxf(m, __uint_as_float(v[e]));
          }
          for (; bk < b1; ++bk) {
            uint32_t v[16];
            tmem_ld_32x32b_x16(srow + 16 * bk, v);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (bk < bu || 16 * bk + e < S) m = fmaxf(m, __uint_as_float(v[e]));
          }
        }
        red_m[cs * 128 + r] = m;
        named_bar_sync(qbar, 32 * kSlices);
#pragma unroll
        for (int c = 0; c < kSlices; ++c) m = fmaxf(m, red_m[c * 128 + r]);
        // the P buffer is free once the previous tile's PV has completed
        if (t > 0 && ok) ok = mbar_wait(o_full((it - 1) & 1), (uint32_t)((it - 1) >> 1) & 1u, err, kDevErrTimeoutTmem);
        // pass 2: P = 2^((s - m) * c) in [0, 1], row sums, NVFP4 P into shared memory
        const unsigned long long nmc2 = f32x2_pack(-m * cexp, -m * cexp);
        unsigned long long lsum2 = f32x2_pack(0.f, 0.f);
        // one 16-key block: exp, masking of keys >= S (limit = S - 16 bk), sum, scale, codes
        auto p_block = [&](const uint32_t* v, int bk, int limit) {
          float p[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float x0, x1;
            f32x2_unpack(fma_f32x2(f32x2_pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), c2, nmc2),
                         &x0, &x1);
            p[2 * i] = ex2_approx(x0);
            p[2 * i + 1] = ex2_approx(x1);
          }
          if (limit < 16) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (e >= limit) p[e] = 0.f;
          }
          float am = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            lsum2 = add_f32x2(lsum2, f32x2_pack(p[2 * i], p[2 * i + 1]));
            am = fmaxf(am, fmaxf(p[2 * i], p[2 * i + 1]));
          }
          float dec;
          const uint32_t sf = six_scale(am, 2688.f, kInv2688, &dec);
          *reinterpret_cast<uint64_t*>(gb + g.fp + cm_off(r, bk, sbo_kv)) = encode16_fast(p, dec);
          gb[g.sfp + (uint32_t)(bk >> 2) * 512u + sf_atom_off(r, bk & 3)] = (uint8_t)sf;
        };
        if (active && ok) {
          int bk = b0;
          for (; bk + 1 < bu; bk += 2) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(srow + 16 * bk, v);
            tmem_wait_ld();
            p_block(v, bk, 16);
            p_block(v + 16, bk + 1, 16);
          }
          for (; bk < b1; ++bk) {
            uint32_t v[16];
            tmem_ld_32x32b_x16(srow + 16 * bk, v);
            tmem_wait_ld();
            p_block(v, bk, bk < bu ? 16 : S - 16 * bk);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
        float l0, l1;
        f32x2_unpack(lsum2, &l0, &l1);
        red_l[(it & 1) * (kSlices * 128) + cs * 128 + r] = l0 + l1;
        fence_async_shared();   // P writes -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (t > 0) epilogue(it - 1, t - 1);
      }
      // the head's last tile
      if (ok) ok = mbar_wait(o_full((it - 1) & 1), (uint32_t)((it - 1) >> 1) & 1u, err, kDevErrTimeoutTmem);
      tc_fence_after();
      epilogue(it - 1, g.nq - 1);
      if constexpr (kPacked) {   // every MMA of this head completed (o_full above); scalars read
        __syncwarp();
        if (lane == 0) mbar_arrive(img_free(hi & 1));
      }
    }
    if (cs == 0 && lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

// bf16 4-D view of (b, h, s, d) element strides (sb, sh, ss, 1) with boxes of 64 x rows x one head,
// 128-byte swizzle; the s and h dimensions are ordered by increasing stride (hs = h first).
static int make_head_map(CUtensorMap* m, const void* ptr, const FusedGeom& g, int64_t sb, int64_t sh, int64_t ss,
                         int box_rows, bool hs) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {(cuuint64_t)g.D, (cuuint64_t)(hs ? g.H : g.S), (cuuint64_t)(hs ? g.S : g.H), (cuuint64_t)g.B};
  cuuint64_t strides[3] = {(cuuint64_t)(hs ? sh : ss) * 2, (cuuint64_t)(hs ? ss : sh) * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64u, hs ? 1u : (cuuint32_t)box_rows, hs ? (cuuint32_t)box_rows : 1u, 1u};
  cuuint32_t es[4] = {1u, 1u, 1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled (attention head view) failed (%d)", (int)r);
  return VF4_OK;
}

// ---------------------------------------------------------------------------------------
// Operand packing for the packed fused route: one CTA per (b, h) quantizes Q, K~ = K - mean(K) and
// V~^T = (V - mean(V))^T with the arithmetic of the fused kernel's own preparation and writes the
// head's operand image -- codes in the MMA's K-major core-matrix layout, scale atoms in the
// tcgen05.cp layout, then gs_q, gs_k, gs_v and mean(v) -- to global memory; the packed fused kernel
// bulk-copies it into shared memory unchanged.  The image is assembled in shared memory (its
// padding rows and scale-atom tails stay zero) and stored with 16-byte writes.  With tensor-wide
// globals the means and maxima come from attn_stats_kernel; otherwise this CTA computes the head's
// own (means in a fixed summation order, centred maxima from column max / min).
// Many small CTAs per SM (about 50 KB of shared memory each) keep the loads and the quantizer
// latency overlapped, which the fused kernel's 12 compute warps could not.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256, 3) attn_pack_kernel(const __nv_bfloat16* __restrict__ q,
                                                        const __nv_bfloat16* __restrict__ k,
                                                        const __nv_bfloat16* __restrict__ v, int64_t sb,
                                                        int64_t sh, int64_t ss, const FusedGeom g,
                                                        uint8_t* __restrict__ images) {
  extern __shared__ __align__(16) uint8_t img[];
  __shared__ float mu[128];          // mean(k) [0, 64), mean(v) [64, 128)
  __shared__ float scal[8];          // gs_q, gs_k, gs_v, 1/gs_q, 1/gs_k, 1/gs_v
  __shared__ float part[8][6][64];   // per-warp column partials (per-head globals)
  __shared__ __align__(16) uint32_t vstage[8][16 * 32];   // per-warp 16 v rows of 64 bf16
  const int head = blockIdx.x;
  const int b = head / g.H, h = head - b * g.H;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int S = g.S;
  const int64_t hoff = (int64_t)b * sb + (int64_t)h * sh;
  for (uint32_t o = 16u * t; o < g.img_bytes; o += 16u * 256u) *reinterpret_cast<uint4*>(img + o) = make_uint4(0, 0, 0, 0);
  if (g.stats) {
    if (t < 128) mu[t] = g.stats[(int64_t)head * 128 + t];
    if (t < 3) {
      const float gsv = __fdiv_rn(fmaxf(g.amax3[t], 1e-12f), 2688.f);
      scal[t] = gsv;
      scal[3 + t] = __fdiv_rn(1.0f, gsv);
    }
  } else {
    // per-head globals: chunk j = t % 8 of rows t / 8 + 32 i
    const int j = t & 7;
    float ks[8], kx[8], kn[8], vs[8], vx[8], vn[8], qm = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      ks[e] = vs[e] = 0.f;
      kx[e] = vx[e] = -INFINITY;
      kn[e] = vn[e] = INFINITY;
    }
    for (int r = t >> 3; r < S; r += 32) {
      float a[8], c[8], u[8];
      load8(q + hoff + (int64_t)r * ss + 8 * j, a);
      load8(k + hoff + (int64_t)r * ss + 8 * j, c);
      load8(v + hoff + (int64_t)r * ss + 8 * j, u);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        qm = fmaxf(qm, fabsf(a[e]));
        ks[e] += c[e];
        kx[e] = fmaxf(kx[e], c[e]);
        kn[e] = fminf(kn[e], c[e]);
        vs[e] += u[e];
        vx[e] = fmaxf(vx[e], u[e]);
        vn[e] = fminf(vn[e], u[e]);
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {   // lanes j, j + 8, j + 16, j + 24 hold chunk j: fixed combination order
#pragma unroll
      for (int o = 8; o <= 16; o <<= 1) {
        ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], o);
        vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], o);
        kx[e] = fmaxf(kx[e], __shfl_xor_sync(0xffffffffu, kx[e], o));
        kn[e] = fminf(kn[e], __shfl_xor_sync(0xffffffffu, kn[e], o));
        vx[e] = fmaxf(vx[e], __shfl_xor_sync(0xffffffffu, vx[e], o));
        vn[e] = fminf(vn[e], __shfl_xor_sync(0xffffffffu, vn[e], o));
      }
    }
    if (lane < 8) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        part[w][0][8 * j + e] = ks[e];
        part[w][1][8 * j + e] = kx[e];
        part[w][2][8 * j + e] = kn[e];
        part[w][3][8 * j + e] = vs[e];
        part[w][4][8 * j + e] = vx[e];
        part[w][5][8 * j + e] = vn[e];
      }
    }
    qm = warp_max(qm);
    if (lane == 0) scal[6] = 0.f;
    __syncthreads();
    if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(&scal[6]), __float_as_uint(qm));
    float ak = 0.f, av = 0.f;
    if (t < 64) {
      float sk = 0.f, xk = -INFINITY, nk = INFINITY, sv = 0.f, xv = -INFINITY, nv = INFINITY;
      for (int ww = 0; ww < 8; ++ww) {
        sk += part[ww][0][t];
        xk = fmaxf(xk, part[ww][1][t]);
        nk = fminf(nk, part[ww][2][t]);
        sv += part[ww][3][t];
        xv = fmaxf(xv, part[ww][4][t]);
        nv = fminf(nv, part[ww][5][t]);
      }
      const float mk = __fdiv_rn(sk, (float)S), mv = __fdiv_rn(sv, (float)S);
      mu[t] = mk;
      mu[64 + t] = mv;
      ak = fmaxf(fabsf(xk - mk), fabsf(nk - mk));
      av = fmaxf(fabsf(xv - mv), fabsf(nv - mv));
    }
    ak = warp_max(ak);
    av = warp_max(av);
    __shared__ float red2[2][2];   // centred maxima of k and v from warps 0, 1 (the 64 columns)
    if (lane == 0 && w < 2) {
      red2[w][0] = ak;
      red2[w][1] = av;
    }
    __syncthreads();
    if (t < 3) {
      const float am = t == 0 ? scal[6] : fmaxf(red2[0][t - 1], red2[1][t - 1]);
      const float gsv = __fdiv_rn(fmaxf(am, 1e-12f), 2688.f);
      scal[t] = gsv;
      scal[3 + t] = __fdiv_rn(1.0f, gsv);
    }
  }
  __syncthreads();
  const float gq = scal[0], gk = scal[1], gv = scal[2];
  // Q rows [0, 128 nq) and K~ rows [0, skp): 4 column blocks per row, a lane quad per row (their
  // scale bytes merge into one word); loop bounds are multiples of 256, so whole warps iterate
  auto qk_block = [&](int i, const __nv_bfloat16* src, uint32_t fo, uint32_t so, bool centre, float gs, float se,
                      float dec_max) {
    const int r = i >> 2, cb = i & 3;
    uint64_t codes = 0;
    uint32_t sf = 0;
    if (r < S) {
      float x[16];
      load8(src + hoff + (int64_t)r * ss + 16 * cb, x);
      load8(src + hoff + (int64_t)r * ss + 16 * cb + 8, x + 8);
      if (centre) {
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] -= mu[16 * cb + e];
      }
      const BlockQ z = quantize_block<false>(x, gs, se, dec_max);
      codes = z.packed;
      sf = z.sf;
    }
    *reinterpret_cast<uint64_t*>(img + fo + cm_off(r, cb, 256)) = codes;
    uint32_t wd = sf << (8 * cb);
    wd |= __shfl_xor_sync(0xffffffffu, wd, 1);
    wd |= __shfl_xor_sync(0xffffffffu, wd, 2);
    if (cb == 0) *reinterpret_cast<uint32_t*>(img + so + sf_atom_off(r, 0)) = wd;
  };
  for (int i = t; i < g.nq * 512; i += 256) qk_block(i, q, g.fq, g.sfq, false, gq, scal[3], 0x1p17f);
  for (int i = t; i < g.skp * 4; i += 256) qk_block(i, k, g.fk, g.sfk, true, gk, scal[4], 2.0f);
  // V~^T rows d in [0, 64), token blocks tb in [0, skp / 16): warp w stages the 16 v rows of its
  // token blocks (2 KB, four 16-byte loads per lane) in shared memory, then lane l quantizes the
  // columns d = 2l, 2l + 1 of the block (its reads of a row are one 4-byte word per lane)
  const uint32_t sbo_kv = (uint32_t)(g.skp / 32) * 128u;
  const int nvb = (S + 15) / 16;
  uint4* vst = reinterpret_cast<uint4*>(vstage[w]);
  uint4 vnext[4];   // the next token block's rows, loaded while this one is quantized
  auto vload = [&](int tb) {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int rr = 4 * p + (lane >> 3), r = tb * 16 + rr, c8 = lane & 7;
      vnext[p] = (tb < nvb && r < S) ? __ldg(reinterpret_cast<const uint4*>(v + hoff + (int64_t)r * ss + 8 * c8))
                                     : make_uint4(0, 0, 0, 0);
    }
  };
  vload(w);
  for (int tb = w; tb < nvb; tb += 8) {
#pragma unroll
    for (int p = 0; p < 4; ++p) vst[(4 * p + (lane >> 3)) * 8 + (lane & 7)] = vnext[p];
    vload(tb + 8);
    __syncwarp();
    float x0[16], x1[16];
    const float m0 = mu[64 + 2 * lane], m1 = mu[64 + 2 * lane + 1];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const uint32_t wd = reinterpret_cast<const uint32_t*>(vstage[w])[e * 32 + lane];
      const bool in = tb * 16 + e < S;
      x0[e] = in ? __uint_as_float(wd << 16) - m0 : 0.f;
      x1[e] = in ? __uint_as_float(wd & 0xFFFF0000u) - m1 : 0.f;
    }
    __syncwarp();   // the stage is refilled on the next trip
    const BlockQ z0 = quantize_block<false>(x0, gv, scal[5]);
    const BlockQ z1 = quantize_block<false>(x1, gv, scal[5]);
    const int d0 = 2 * lane, d1 = 2 * lane + 1;
    *reinterpret_cast<uint64_t*>(img + g.fv + cm_off(d0, tb, sbo_kv)) = z0.packed;
    *reinterpret_cast<uint64_t*>(img + g.fv + cm_off(d1, tb, sbo_kv)) = z1.packed;
    img[g.sfv + (uint32_t)(tb >> 2) * 512u + sf_atom_off(d0, tb & 3)] = (uint8_t)z0.sf;
    img[g.sfv + (uint32_t)(tb >> 2) * 512u + sf_atom_off(d1, tb & 3)] = (uint8_t)z1.sf;
  }
  if (t < 3) reinterpret_cast<float*>(img + g.img_scal)[t] = scal[t];
  if (t < 64) reinterpret_cast<float*>(img + g.img_scal)[64 + t] = mu[64 + t];
  __syncthreads();
  uint8_t* dst = images + (int64_t)head * g.img_bytes;
  for (uint32_t o = 16u * t; o < g.img_bytes; o += 16u * 256u)
    *reinterpret_cast<uint4*>(dst + o) = *reinterpret_cast<const uint4*>(img + o);
}

static int launch_fused(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                        int64_t sb, int64_t sh, int64_t ss, float scale, void* out, int64_t osb, int64_t osh,
                        int64_t oss, const float* stats, const float* amax3, cudaStream_t s,
                        uint8_t* images = nullptr) {
  const bool packed = images != nullptr;
  FusedGeom g = make_fused_geom(B, H, S, D, scale, packed);
  g.stats = stats;
  g.amax3 = amax3;
  g.images = images;
  g.qkv_hs = sh < ss;
  g.out_hs = osh < oss;
  CUtensorMap tq, tk, tv, to;
  if (int st = make_head_map(&tq, q, g, sb, sh, ss, g.box_rows, g.qkv_hs)) return st;
  if (int st = make_head_map(&tk, k, g, sb, sh, ss, g.box_rows, g.qkv_hs)) return st;
  if (int st = make_head_map(&tv, v, g, sb, sh, ss, g.box_rows, g.qkv_hs)) return st;
  if (int st = make_head_map(&to, out, g, osb, osh, oss, 32, g.out_hs)) return st;
  if (packed) {
    const int smem = (int)g.img_bytes;
    if (int st = smem_optin(attn_pack_kernel, smem)) return st;
    attn_pack_kernel<<<(unsigned)g.heads, 256, smem, s>>>(static_cast<const __nv_bfloat16*>(q),
                                                          static_cast<const __nv_bfloat16*>(k),
                                                          static_cast<const __nv_bfloat16*>(v), sb, sh, ss, g, images);
    if (int st = launch_status("vf4_attn_nvfp4 (pack)")) return st;
  }
  auto kern = packed ? attn_fused_kernel<true> : attn_fused_kernel<false>;
  if (int st = smem_optin(kern, (int)g.total)) return st;
  const int grid = g.heads < num_sms() ? g.heads : num_sms();
  kern<<<grid, kFusedWarps * 32, g.total, s>>>(tq, tk, tv, to, g);
  return launch_status(packed ? "vf4_attn_nvfp4 (fused, packed operands)" : "vf4_attn_nvfp4 (fused)");
}

// ---------------------------------------------------------------------------------------
// FP8 attention, the reference's default route quant_sdpa(qk='fp8', pv='fp8') (attention.py:53-86
// with fp8.py:6-17): every operand row is quantized to E4M3 with its own scale amax/448 — Q and
// K~ per token along d, P per query along keys, V~ per head-dim column along tokens.  The scales
// factor out of the dot products, so QK^T and PV run as plain E4M3 x E4M3 -> fp32 MMAs
// (tcgen05.mma kind::f8f6f4, K = 32 per instruction) and the scales are applied to the scores
// (per row and column) and to the output (per row and column).  P = exp(s - max) is quantized as
// e4m3(448 * P): the reference's per-row scale of the normalised P is max(P) / 448 = 1 / (448 rowsum),
// so P / scale equals 448 * exp(s - max).  Head dim 64, S <= 320, one kernel, no workspace; the
// same persistent structure as attn_fused_kernel (loader, MMA issuer, 12 compute warps), with q
// read straight from global memory during prep (only k and v are staged, to fit 8-bit operands).
// ---------------------------------------------------------------------------------------
struct Fp8Geom {
  int B, H, S, D;
  int nq, skp, box_rows, nbox, heads;
  int kv_hs, out_hs;
  int smooth;                    // bit 0: subtract mean(k), bit 1: subtract mean(v) (and add it back)
  float scale;
  const __nv_bfloat16* q;        // read directly: element (b, h, s, d) at q + b sb + h sh + s ss + d
  int64_t sb, sh, ss;
  uint32_t raw_k, raw_v, fq, fk, fv, fp, stg, scl, red, bar, total;
};

static Fp8Geom make_fp8_geom(int64_t B, int64_t H, int64_t S, int64_t D, float scale) {
  Fp8Geom g{};
  g.B = (int)B;
  g.H = (int)H;
  g.S = (int)S;
  g.D = (int)D;
  g.nq = (int)((S + 127) / 128);
  g.skp = (int)((S + 63) / 64 * 64);
  g.nbox = S <= 256 ? 1 : 2;
  g.box_rows = (int)align_up((S + g.nbox - 1) / g.nbox, 8);
  g.heads = (int)(B * H);
  g.scale = scale;
  const uint32_t rawb = (uint32_t)(g.nbox * g.box_rows * 128);
  uint32_t o = 0;
  g.raw_k = o; o += rawb;
  g.raw_v = o; o += rawb;
  g.fq = o;  o += (uint32_t)g.nq * 128u * 64u;    // Q8: rows x 64 bytes
  g.fk = o;  o += (uint32_t)g.skp * 64u;          // K8
  g.fv = o;  o += 64u * (uint32_t)g.skp;          // V8^T: 64 rows x skp bytes
  g.fp = o;  o += 128u * (uint32_t)g.skp;         // P8: 128 rows x skp bytes
  o = (uint32_t)align_up(o, 1024);
  g.stg = o; o += 4 * 4096;
  g.scl = o; o += (uint32_t)(g.nq * 128 + g.skp + 64) * 4u;   // sq, sk, sv
  o = (uint32_t)align_up(o, 16);
  g.red = o; o += 15104;
  g.bar = o; o += 128;
  g.total = o + 1024;
  return g;
}

static bool fp8_ok(int64_t S, int64_t D) {
  if (D != 64 || S > 320) return false;
  return make_fp8_geom(1, 1, S, D, 1.f).total <= 227u * 1024u;
}

// Instruction descriptor for kind::f8f6f4 with E4M3 A and B (K-major), fp32 accumulation.
__host__ __device__ constexpr uint32_t idesc_f8_e4m3(uint32_t n, uint32_t m = 128) {
  return (1u << 4)            // D format: F32
         | (0u << 7)          // A format: E4M3
         | (0u << 10)         // B format: E4M3
         | ((n >> 3) << 17) | ((m >> 4) << 24);
}

VF4_DEV void mma_f8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// Two fp32 values -> two E4M3 bytes (low byte = first value), round-to-nearest-even, saturating.
VF4_DEV uint32_t e4m3x2(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}

// 16 fp32 values times `mul` -> 16 E4M3 bytes
VF4_DEV uint4 e4m3x16(const float* x, float mul) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = e4m3x2(x[4 * i] * mul, x[4 * i + 1] * mul) | (e4m3x2(x[4 * i + 2] * mul, x[4 * i + 3] * mul) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Registers written by an asynchronous tcgen05.ld are only valid after tcgen05.wait::ld; these
// empty volatile statements keep the compiler from moving their first uses above the wait.
VF4_DEV void reg_fence16(uint32_t* v) {
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(v[i]));
}

// Pass 1 on 16 of this warp's score columns: max of acc * sk (packed multiplies, three-input max);
// kMask drops the columns >= nv (keys past S in the last chunk).
template <bool kMask>
VF4_DEV float f8l_half_max(const uint32_t* v, const float4* sk4, int nv) {
  float ma = -INFINITY, mb = -INFINITY;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 k4 = sk4[i];
    float a0, a1, a2, a3;
    f32x2_unpack(mul_f32x2(f32x2_pack(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])), f32x2_pack(k4.x, k4.y)),
                 &a0, &a1);
    f32x2_unpack(mul_f32x2(f32x2_pack(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])),
                           f32x2_pack(k4.z, k4.w)), &a2, &a3);
    if (kMask) {
      a0 = 4 * i < nv ? a0 : -INFINITY;
      a1 = 4 * i + 1 < nv ? a1 : -INFINITY;
      a2 = 4 * i + 2 < nv ? a2 : -INFINITY;
      a3 = 4 * i + 3 < nv ? a3 : -INFINITY;
    }
    ma = max3f(ma, a0, a1);
    mb = max3f(mb, a2, a3);
  }
  return fmaxf(ma, mb);
}

// Pass 2 on 16 of this warp's score columns: p = 2^(acc sk sq - max + log2 448) (sq2, nm2: sq and
// log2 448 - max in both halves), row sums accumulated in two packed pairs; kMask zeroes the columns
// >= nv.
template <bool kMask>
VF4_DEV void f8l_half_exp(const uint32_t* v, const float4* sk4, int nv, unsigned long long sq2,
                          unsigned long long nm2, float* p, unsigned long long& l2a, unsigned long long& l2b) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 k4 = sk4[i];
    float e0, e1, e2, e3;
    f32x2_unpack(fma_f32x2(mul_f32x2(f32x2_pack(__uint_as_float(v[4 * i]), __uint_as_float(v[4 * i + 1])),
                                     f32x2_pack(k4.x, k4.y)), sq2, nm2), &e0, &e1);
    f32x2_unpack(fma_f32x2(mul_f32x2(f32x2_pack(__uint_as_float(v[4 * i + 2]), __uint_as_float(v[4 * i + 3])),
                                     f32x2_pack(k4.z, k4.w)), sq2, nm2), &e2, &e3);
    p[4 * i] = ex2_approx(e0);
    p[4 * i + 1] = ex2_approx(e1);
    p[4 * i + 2] = ex2_approx(e2);
    p[4 * i + 3] = ex2_approx(e3);
    if (kMask) {
#pragma unroll
      for (int e = 0; e < 4; ++e) p[4 * i + e] = 4 * i + e < nv ? p[4 * i + e] : 0.f;
    }
    l2a = add_f32x2(l2a, f32x2_pack(p[4 * i], p[4 * i + 1]));
    l2b = add_f32x2(l2b, f32x2_pack(p[4 * i + 2], p[4 * i + 3]));
  }
}

__global__ void __launch_bounds__(kFusedWarps * 32, 1)
    attn_fp8_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                    const __grid_constant__ CUtensorMap tmO, const Fp8Geom g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (base - raw0);
  const uint32_t bar = base + g.bar;
  const uint32_t raw_full = bar, raw_free = bar + 8, ops_ready = bar + 16, s_full = bar + 24, s_free = bar + 32,
                 p_full = bar + 40, drain = bar + 80;
  auto o_full = [&](int ob) { return bar + 48 + 8u * ob; };
  auto o_free = [&](int ob) { return bar + 64 + 8u * ob; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gb + g.bar + 88);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbo_q = 4u * 128u;                          // 64-byte rows: 4 chunks per 8-row group
  const uint32_t sbo_kv = (uint32_t)(g.skp / 16) * 128u;     // skp-byte rows (P8, V8^T)
  int* err = &g_attn_err;

  if (warp == 0 && lane == 0) {
    mbar_init(raw_full, 1);
    mbar_init(raw_free, kFusedCompute);
    mbar_init(ops_ready, kFusedCompute);
    mbar_init(s_full, 1);
    mbar_init(s_free, kFusedCompute);
    mbar_init(p_full, kFusedCompute);
    for (int ob = 0; ob < 2; ++ob) {
      mbar_init(o_full(ob), 1);
      mbar_init(o_free(ob), kFusedCompute);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    tma_prefetch(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (warp >= 2) {
    // P8 starts at zero: keys >= S stay zero for the whole kernel
    for (uint32_t o = g.fp + 16u * (threadIdx.x - 64); o < g.fp + 128u * (uint32_t)g.skp; o += 16u * kCT)
      *reinterpret_cast<uint4*>(gb + o) = make_uint4(0, 0, 0, 0);
  }
  fence_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------ raw k, v loads
    if (lane == 0) {
      const uint32_t bytes = 2u * (uint32_t)(g.nbox * g.box_rows) * 128u;
      int hi = 0;
      for (int head = blockIdx.x; head < g.heads; head += gridDim.x, ++hi) {
        if (hi > 0 && !mbar_wait(raw_free, (uint32_t)(hi - 1) & 1u, err, kDevErrTimeoutEmpty)) break;
        const int b = head / g.H, h = head - b * g.H;
        mbar_arrive_expect_tx(raw_full, bytes);
        for (int j = 0; j < g.nbox; ++j) {
          const uint32_t off = (uint32_t)(j * g.box_rows) * 128u;
          const int c1 = g.kv_hs ? h : j * g.box_rows, c2 = g.kv_hs ? j * g.box_rows : h;
          tma_load_4d(base + g.raw_k + off, &tmK, 0, c1, c2, b, raw_full);
          tma_load_4d(base + g.raw_v + off, &tmV, 0, c1, c2, b, raw_full);
        }
      }
      if (hi > 0) mbar_wait(raw_full, (uint32_t)(hi - 1) & 1u, err, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    bool ok = true;
    int hi = 0, it = 0;
    const int nks = g.skp / 32;
    for (int head = blockIdx.x; head < g.heads && ok; head += gridDim.x, ++hi) {
      if (!mbar_wait(ops_ready, (uint32_t)hi & 1u, err, kDevErrTimeoutFull)) break;
      tc_fence_after();
      for (int t = 0; t < g.nq; ++t, ++it) {
        if (it > 0 && !mbar_wait(s_free, (uint32_t)(it - 1) & 1u, err, kDevErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          for (int n0 = 0; n0 < g.skp;) {
            const int rem = g.skp - n0;
            const int n = rem >= 256 ? 256 : (rem >= 128 ? 128 : 64);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {   // K = 64 = two K32 steps
              const uint64_t ad = smem_desc(base + g.fq + (uint32_t)t * 16u * sbo_q + 256u * ks, 128, sbo_q, 0);
              const uint64_t bd = smem_desc(base + g.fk + (uint32_t)(n0 / 8) * sbo_q + 256u * ks, 128, sbo_q, 0);
              mma_f8f6f4(tmem + kFusedTmemS + n0, ad, bd, idesc_f8_e4m3((uint32_t)n), ks > 0 ? 1u : 0u);
            }
            n0 += n;
          }
          tc_commit(s_full);
        }
        __syncwarp();
        const int ob = it & 1, use = it >> 1;
        if (!mbar_wait(p_full, (uint32_t)it & 1u, err, kDevErrTimeoutFull) ||
            (use > 0 && !mbar_wait(o_free(ob), (uint32_t)(use - 1) & 1u, err, kDevErrTimeoutEmpty))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t t_o = tmem + kFusedTmemO + 64u * ob;
          for (int ks = 0; ks < nks; ++ks)
            mma_f8f6f4(t_o, smem_desc(base + g.fp + 256u * ks, 128, sbo_kv, 0),
                       smem_desc(base + g.fv + 256u * ks, 128, sbo_kv, 0), idesc_f8_e4m3(64), ks > 0 ? 1u : 0u);
          tc_commit(o_full(ob));
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      tc_commit(drain);
      mbar_wait(drain, 0, err, kDevErrTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ prep, softmax, epilogue
    const int cw = warp - 2;
    const int qd = warp & 3;
    const int cs = cw >> 2;
    const int ct = threadIdx.x - 64;
    const uint32_t qbar = 2u + (uint32_t)qd;
    float* red = reinterpret_cast<float*>(gb + g.red);
    float* red_kv = red;               // [2][kFusedCompute][64] column partial sums / maxima
    float* red_m = red + 2048;         // [kSlices][128]
    float* red_l = red + 2560;         // [2][kSlices][128]
    float* mu = red + 3584;            // [2][64]
    float* sq = reinterpret_cast<float*>(gb + g.scl);   // per query row scale amax / 448
    float* sk = sq + g.nq * 128;                        // per key
    float* sv = sk + g.skp;                             // per head-dim column
    const uint8_t* rk = gb + g.raw_k;
    const uint8_t* rv = gb + g.raw_v;
    const int S = g.S;
    const int nvb = (S + 15) / 16;
    const int b0 = cs * nvb / kSlices, b1 = (cs + 1) * nvb / kSlices;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const int r = qd * 32 + lane;
    bool ok = true;
    int hi = 0, it = 0;
    for (int head = blockIdx.x; head < g.heads; head += gridDim.x, ++hi) {
      const int b = head / g.H, h = head - b * g.H;
      // ---- Q8 straight from global memory (lane quads = one row, 16 values each)
      {
        const __nv_bfloat16* qh = g.q + (int64_t)b * g.sb + (int64_t)h * g.sh;
        for (int i = ct; i < g.nq * 512; i += kCT) {
          const int s = i >> 2, cb = i & 3;
          float x[16];
          float am = 0.f;
          if (s < S) {
            load8(qh + (int64_t)s * g.ss + 16 * cb, x);
            load8(qh + (int64_t)s * g.ss + 16 * cb + 8, x + 8);
#pragma unroll
            for (int e = 0; e < 16; ++e) am = fmaxf(am, fabsf(x[e]));
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] = 0.f;
          }
          am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
          am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
          const float scl = __fdiv_rn(fmaxf(am, 1e-12f), 448.f);
          *reinterpret_cast<uint4*>(gb + g.fq + (uint32_t)(s >> 3) * sbo_q + (uint32_t)cb * 128u + (s & 7) * 16) =
              e4m3x16(x, __fdiv_rn(1.f, scl));
          if (cb == 0) sq[s] = s < S ? scl : 0.f;
        }
      }
      if (ok) ok = mbar_wait(raw_full, (uint32_t)hi & 1u, err, kDevErrTimeoutFull);
      // ---- column sums of k and v -> means (chunk j = ct % 8, rows ct/8 + (kCT/8) i)
      {
        const int j = ct & 7;
        float ks[8], vs[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) ks[e] = vs[e] = 0.f;
        if (ok) {
          for (int s = ct >> 3; s < S; s += kCT / 8) {
            float a[8];
            raw_load8(rk, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) ks[e] += a[e];
            raw_load8(rv, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) vs[e] += a[e];
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], 8);
          ks[e] += __shfl_xor_sync(0xffffffffu, ks[e], 16);
          vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], 8);
          vs[e] += __shfl_xor_sync(0xffffffffu, vs[e], 16);
        }
        if (lane < 8) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            red_kv[cw * 64 + 8 * lane + e] = ks[e];
            red_kv[(kFusedCompute + cw) * 64 + 8 * lane + e] = vs[e];
          }
        }
      }
      named_bar_sync(1, kCT);
      if (ct < 128) {
        const int which = ct >> 6, d = ct & 63;
        float sum = 0.f;
        for (int w = 0; w < kFusedCompute; ++w) sum += red_kv[(which * kFusedCompute + w) * 64 + d];
        mu[which * 64 + d] = (g.smooth & (which ? 2 : 1)) ? __fdiv_rn(sum, (float)S) : 0.f;
      }
      named_bar_sync(1, kCT);
      // ---- per-column amax of v - mean over the tokens -> sv
      {
        const int j = ct & 7;
        float vm[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) vm[e] = 0.f;
        if (ok) {
          for (int s = ct >> 3; s < S; s += kCT / 8) {
            float a[8];
            raw_load8(rv, s, j, a);
#pragma unroll
            for (int e = 0; e < 8; ++e) vm[e] = fmaxf(vm[e], fabsf(a[e] - mu[64 + 8 * j + e]));
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          vm[e] = fmaxf(vm[e], __shfl_xor_sync(0xffffffffu, vm[e], 8));
          vm[e] = fmaxf(vm[e], __shfl_xor_sync(0xffffffffu, vm[e], 16));
        }
        if (lane < 8) {
#pragma unroll
          for (int e = 0; e < 8; ++e) red_kv[cw * 64 + 8 * lane + e] = vm[e];
        }
      }
      named_bar_sync(1, kCT);
      if (ct < 64) {
        float m = 0.f;
        for (int w = 0; w < kFusedCompute; ++w) m = fmaxf(m, red_kv[w * 64 + ct]);
        sv[ct] = __fdiv_rn(fmaxf(m, 1e-12f), 448.f);
      }
      named_bar_sync(1, kCT);
      // ---- K8: per key row (lane quads), k - mean
      for (int i = ct; i < g.skp * 4; i += kCT) {
        const int s = i >> 2, cb = i & 3;
        float x[16];
        float am = 0.f;
        if (ok && s < S) {
          raw_load8(rk, s, 2 * cb, x);
          raw_load8(rk, s, 2 * cb + 1, x + 8);
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            x[e] -= mu[16 * cb + e];
            am = fmaxf(am, fabsf(x[e]));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) x[e] = 0.f;
        }
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        const float scl = __fdiv_rn(fmaxf(am, 1e-12f), 448.f);
        *reinterpret_cast<uint4*>(gb + g.fk + (uint32_t)(s >> 3) * sbo_q + (uint32_t)cb * 128u + (s & 7) * 16) =
            e4m3x16(x, __fdiv_rn(1.f, scl));
        if (cb == 0) sk[s] = s < S ? (g.scale < 0.f ? -scl : scl) : 0.f;   // the score's sign folded in
      }
      // ---- V8^T: row d, 16-token blocks; a warp covers 32 consecutive d of one token block
      {
        const int ntb = g.skp / 16;
        for (int i = ct; i < 64 * ntb; i += kCT) {
          const int tb = i >> 6, d = i & 63;
          float x[16];
          const float m = mu[64 + d];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int s = tb * 16 + e;
            x[e] = (ok && s < S) ? raw_elem(rv, s, d) - m : 0.f;
          }
          *reinterpret_cast<uint4*>(gb + g.fv + (uint32_t)(d >> 3) * sbo_kv + (uint32_t)tb * 128u + (d & 7) * 16) =
              e4m3x16(x, __fdiv_rn(1.f, sv[d]));
        }
      }
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(ops_ready);
        mbar_arrive(raw_free);
      }
      named_bar_sync(1, kCT);   // sq / sk / sv visible to every compute warp
      const float cbase = fabsf(g.scale) * 1.4426950408889634f;
      const int c0 = cs * 8 / kSlices, c1 = (cs + 1) * 8 / kSlices;
      auto epilogue = [&](int itt, int tl) {
        const bool act = ok && tl * 128 + qd * 32 < S;
        const int ob = itt & 1;
        constexpr int kMaxChunks = (8 + kSlices - 1) / kSlices;
        uint32_t ov[kMaxChunks][8];
        if (act) {
#pragma unroll
          for (int k = 0; k < kMaxChunks; ++k)
            if (c0 + k < c1) tmem_ld_32x32b_x8(tmem + lane_base + kFusedTmemO + 64u * ob + 8 * (c0 + k), ov[k]);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(o_free(ob));
        if (cs == 0 && lane == 0) bulk_wait_read();
        named_bar_sync(qbar, 32 * kSlices);
        uint8_t* stg = gb + g.stg + qd * 4096 + lane * 128;
        if (act) {
          const float* rl = red_l + ob * (kSlices * 128);
          float lsum = 0.f;
#pragma unroll
          for (int c = 0; c < kSlices; ++c) lsum += rl[c * 128 + r];
          const float f = 1.0f / (448.f * lsum);
#pragma unroll
          for (int k = 0; k < kMaxChunks; ++k) {
            const int c = c0 + k;
            if (c < c1) {
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int d = 8 * c + 2 * i;
                __nv_bfloat162 hv = __floats2bfloat162_rn(
                    __fmaf_rn(__uint_as_float(ov[k][2 * i]), f * sv[d], mu[64 + d]),
                    __fmaf_rn(__uint_as_float(ov[k][2 * i + 1]), f * sv[d + 1], mu[64 + d + 1]));
                w[i] = *reinterpret_cast<uint32_t*>(&hv);
              }
              *reinterpret_cast<uint4*>(stg + ((c ^ (lane & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
        fence_async_shared();
        named_bar_sync(qbar, 32 * kSlices);
        if (act && cs == 0 && lane == 0) {
          const int row = tl * 128 + qd * 32;
          tma_store_4d(&tmO, base + g.stg + qd * 4096, 0, g.out_hs ? h : row, g.out_hs ? row : h, b);
          bulk_commit();
        }
      };
      for (int t = 0; t < g.nq; ++t, ++it) {
        const bool active = ok && t * 128 + qd * 32 < S;
        if (ok) ok = mbar_wait(s_full, (uint32_t)it & 1u, err, kDevErrTimeoutFull);
        tc_fence_after();
        const uint32_t srow = tmem + lane_base + kFusedTmemS;
        const float c = sq[t * 128 + r] * cbase;   // real score * log2 e = acc * sk * c, c >= 0
        // pass 1: max over keys of acc * sk (c >= 0 is common to the row), 16 columns per TMEM load
        // (a second load in flight spills registers at this kernel's 128-register budget)
        float m = -INFINITY;
        if (active && ok && b0 < b1) {
          uint32_t va[16];
          auto max16 = [&](int bk, const uint32_t* v) {
            const float4* sk4 = reinterpret_cast<const float4*>(sk + 16 * bk);
            const int nv = S - 16 * bk;
            m = fmaxf(m, nv >= 16 ? f8l_half_max<false>(v, sk4, 16) : f8l_half_max<true>(v, sk4, nv));
          };
          for (int bk = b0; bk < b1; ++bk) {
            tmem_ld_32x32b_x16(srow + 16 * bk, va);
            tmem_wait_ld();
            reg_fence16(va);
            max16(bk, va);
          }
        }
        red_m[cs * 128 + r] = m;
        named_bar_sync(qbar, 32 * kSlices);
#pragma unroll
        for (int k = 0; k < kSlices; ++k) m = fmaxf(m, red_m[k * 128 + r]);
        if (t > 0 && ok) ok = mbar_wait(o_full((it - 1) & 1), (uint32_t)((it - 1) >> 1) & 1u, err, kDevErrTimeoutTmem);
        // pass 2: P = exp(s - max), row sums, P8 = e4m3(448 P)
        const float nmc = -m * c;
        float lsum = 0.f;
        if (active && ok && b0 < b1) {
          const unsigned long long c2 = f32x2_pack(c, c), nm2 = f32x2_pack(nmc, nmc);
          unsigned long long l2a = f32x2_pack(0.f, 0.f), l2b = l2a;
          uint32_t va[16];
          auto exp16 = [&](int bk, const uint32_t* v) {
            const float4* sk4 = reinterpret_cast<const float4*>(sk + 16 * bk);
            const int nv = S - 16 * bk;
            float p[16];
            if (nv >= 16)
              f8l_half_exp<false>(v, sk4, 16, c2, nm2, p, l2a, l2b);
            else
              f8l_half_exp<true>(v, sk4, nv, c2, nm2, p, l2a, l2b);
            *reinterpret_cast<uint4*>(gb + g.fp + (uint32_t)(r >> 3) * sbo_kv + (uint32_t)bk * 128u + (r & 7) * 16) =
                e4m3x16(p, 448.f);
          };
          for (int bk = b0; bk < b1; ++bk) {
            tmem_ld_32x32b_x16(srow + 16 * bk, va);
            tmem_wait_ld();
            reg_fence16(va);
            exp16(bk, va);
          }
          float la0, la1, lb0, lb1;
          f32x2_unpack(l2a, &la0, &la1);
          f32x2_unpack(l2b, &lb0, &lb1);
          lsum = (la0 + la1) + (lb0 + lb1);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);
        red_l[(it & 1) * (kSlices * 128) + cs * 128 + r] = lsum;
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (t > 0) epilogue(it - 1, t - 1);
      }
      if (ok) ok = mbar_wait(o_full((it - 1) & 1), (uint32_t)((it - 1) >> 1) & 1u, err, kDevErrTimeoutTmem);
      tc_fence_after();
      epilogue(it - 1, g.nq - 1);
      named_bar_sync(1, kCT);   // every warp is done with this head's scales before the next head's prep
    }
    if ((warp - 2) < 4 && lane == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

static int launch_fp8(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                      int64_t sb, int64_t sh, int64_t ss, float scale, void* out, int64_t osb, int64_t osh,
                      int64_t oss, int smooth, cudaStream_t s) {
  Fp8Geom g = make_fp8_geom(B, H, S, D, scale);
  g.smooth = smooth;
  g.q = static_cast<const __nv_bfloat16*>(q);
  g.sb = sb;
  g.sh = sh;
  g.ss = ss;
  g.kv_hs = sh < ss;
  g.out_hs = osh < oss;
  FusedGeom fg = make_fused_geom(B, H, S, D, scale);   // the head-view maps take D, S, H, B from it
  CUtensorMap tk, tv, to;
  if (int st = make_head_map(&tk, k, fg, sb, sh, ss, g.box_rows, g.kv_hs)) return st;
  if (int st = make_head_map(&tv, v, fg, sb, sh, ss, g.box_rows, g.kv_hs)) return st;
  if (int st = make_head_map(&to, out, fg, osb, osh, oss, 32, g.out_hs)) return st;
  if (int st = smem_optin(attn_fp8_kernel, (int)g.total)) return st;
  const int grid = g.heads < num_sms() ? g.heads : num_sms();
  attn_fp8_kernel<<<grid, kFusedWarps * 32, g.total, s>>>(tk, tv, to, g);
  return launch_status("vf4_attn_fp8");
}

// ---------------------------------------------------------------------------------------
// FP8 attention for long sequences and head dims other than 64 (ViT-H/14: head dim 80 with
// S = 257 at 224 px and S = 1025 at 448 px).  The arithmetic of attn_fp8_kernel (per-row E4M3
// Q and K~, per-column V~, P = e4m3(448 exp(s - max)), out = O sv / (448 rowsum) + mean(v)),
// split into kernels because the 8-bit operands of a long head do not fit shared memory next to
// its scores:
//   attn_fp8_colstats_kernel  one CTA per head: column means of k and v, per-column scale of V~
//                          (amax of v - mean from the column max and min)
//   attn_fp8_pack_kernel   one CTA per (head, 128-token chunk): Q8, K~8 and V~8^T written to the
//                          workspace in the MMA's K-major core-matrix layout (8 rows x 16 bytes, no
//                          swizzle) so that a plain bulk copy of a contiguous range is an operand
//                          tile; per-row scales of Q (sq) and of K~ (sk, pre-multiplied by
//                          scale * log2 e)
//   attn_fp8_long_kernel   persistent, whole heads per CTA.  K~8 and sk stay in shared memory for
//                          the head; per 128-query tile Q8 is loaded once and the V~8^T key chunks
//                          stream through a 3-stage ring.  The scores of each tile are formed twice
//                          (128-key chunks into three TMEM buffers): pass 1 takes the exact row max,
//                          pass 2 forms P, its row sums and P8, so P is quantized against the final
//                          max as the reference quantizes its normalised P.
// Warps: 0 loads (cp.async.bulk), 1 MMAs (tcgen05.mma kind::f8f6f4), 2-17 softmax (TMEM lane
// quadrant x 32-key quarter of each chunk) and the epilogue (8-column groups of the head dim).
// Every wait is bounded; a give-up records the device error and unwinds.
// ---------------------------------------------------------------------------------------
constexpr int kF8LStages = 3;                       // V~8^T chunks in flight
constexpr int kF8LSlices = 4;                       // softmax warps per TMEM lane quadrant
constexpr int kF8LSoftmax = 4 * kF8LSlices;
constexpr int kF8LWarps = 2 + kF8LSoftmax;
constexpr uint32_t kF8LSBuf = 3;                    // 128-column score buffers in TMEM, then O
constexpr uint32_t kF8LTmemS = 0, kF8LTmemO = 128 * kF8LSBuf;
static_assert(kF8LTmemO + 128 <= 512, "O (up to 128 columns) follows the score buffers in 512 columns");

struct F8LGeom {
  int B, H, S, D;
  int S_pad, nc, DK, DV;   // keys padded to 128-key chunks; QK^T contraction padded to K32 steps
  int64_t BH;
  int64_t qk_head, v_head;  // bytes per head of Q8 (= K~8) and of V~8^T
  int64_t off_q, off_k, off_v, off_sq, off_sk, off_sv, off_mu, off_muk, total;
};

static F8LGeom make_f8l_geom(int64_t B, int64_t H, int64_t S, int64_t D) {
  F8LGeom g{};
  g.B = (int)B;
  g.H = (int)H;
  g.S = (int)S;
  g.D = (int)D;
  g.S_pad = (int)align_up(S, 128);
  g.nc = g.S_pad / 128;
  g.DK = (int)align_up(D, 32);
  g.DV = (int)D;
  g.BH = B * H;
  g.qk_head = (int64_t)g.S_pad * g.DK;
  g.v_head = (int64_t)g.nc * g.DV * 128;
  int64_t o = 0;
  g.off_q = o;  o = align_up(o + g.BH * g.qk_head, 1024);
  g.off_k = o;  o = align_up(o + g.BH * g.qk_head, 1024);
  g.off_v = o;  o = align_up(o + g.BH * g.v_head, 1024);
  g.off_sq = o; o = align_up(o + g.BH * g.S_pad * 4, 1024);
  g.off_sk = o; o = align_up(o + g.BH * g.S_pad * 4, 1024);
  g.off_sv = o; o = align_up(o + g.BH * g.DV * 4, 1024);
  g.off_mu = o; o = align_up(o + g.BH * g.DV * 4, 1024);
  g.off_muk = o; o = align_up(o + g.BH * g.DV * 4, 1024);
  g.total = o;
  return g;
}

struct F8LSmem {
  uint32_t k, sk, q, v, p, red_m, red_l, bar, total;
};

static F8LSmem f8l_smem_layout(const F8LGeom& g) {
  F8LSmem s{};
  uint32_t o = 0;
  s.k = o;     o += (uint32_t)g.nc * 128u * (uint32_t)g.DK;
  s.sk = o;    o += (uint32_t)g.S_pad * 4u;
  s.q = o;     o += 128u * (uint32_t)g.DK;
  s.v = o;     o += (uint32_t)kF8LStages * (uint32_t)g.DV * 128u;
  s.p = o;     o += 2u * 128u * 128u;
  s.red_m = o; o += (uint32_t)kF8LSlices * 128u * 4u;
  s.red_l = o; o += (uint32_t)kF8LSlices * 128u * 4u;
  s.bar = o;   o += 256;
  s.total = o + 1024;   // slack for aligning the base to 1024
  return s;
}

static bool f8l_ok(int64_t S, int64_t D) {
  if (S < 1 || D < 16 || D > 128 || D % 16 != 0 || S > (1 << 20)) return false;
  return f8l_smem_layout(make_f8l_geom(1, 1, S, D)).total <= 227u * 1024u;
}

// 16 fp32 values divided by `scl` -> E4M3 bytes.  The quotients are the correctly rounded x / scl of
// the reference (Markstein's correction with inv = RN(1 / scl); quotients too small for it to hold
// are far below E4M3's smallest subnormal and encode as zero either way).
VF4_DEV uint4 e4m3x16_div(const float* x, float scl, float inv) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = e4m3x2(div_markstein(x[4 * i], scl, inv), div_markstein(x[4 * i + 1], scl, inv)) |
           (e4m3x2(div_markstein(x[4 * i + 2], scl, inv), div_markstein(x[4 * i + 3], scl, inv)) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Column statistics of one head (one CTA per head): sums of k and v, max and min of v over the
// tokens -> mean(k) (or 0 without smooth-K), mean(v) (or 0 without smooth-V) and the per-column
// scale of V~ = max_s |v_s - mean| / 448 (rounding is monotone, so that max is
// max(|max v - mean|, |min v - mean|) exactly).
__global__ void __launch_bounds__(256) attn_fp8_colstats_kernel(const __nv_bfloat16* __restrict__ k,
                                                                const __nv_bfloat16* __restrict__ v, int64_t sb,
                                                                int64_t sh, int64_t ss, const F8LGeom g, int smooth,
                                                                uint8_t* __restrict__ ws) {
  __shared__ float part[4][2048];   // per thread row-slice: column sums of k and v, max and min of v
  const int bh = blockIdx.x;
  const int b = bh / g.H, h = bh - b * g.H;
  const __nv_bfloat16* kh = k + b * sb + h * sh;
  const __nv_bfloat16* vh = v + b * sb + h * sh;
  const int S = g.S, D = g.D, D8 = D / 8;
  const int rpi = 256 / D8, active = rpi * D8;
  const int t = threadIdx.x, c8 = t % D8, r0 = t / D8;
  {
    float sk[8], sv[8], vmax[8], vmin[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sk[i] = sv[i] = 0.f;
      vmax[i] = -INFINITY;
      vmin[i] = INFINITY;
    }
    if (t < active) {
      for (int r = r0; r < S; r += rpi) {
        float bk[8], bv[8];
        load8(kh + r * ss + c8 * 8, bk);
        load8(vh + r * ss + c8 * 8, bv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          sk[i] += bk[i];
          sv[i] += bv[i];
          vmax[i] = fmaxf(vmax[i], bv[i]);
          vmin[i] = fminf(vmin[i], bv[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        part[0][r0 * D + c8 * 8 + i] = sk[i];
        part[1][r0 * D + c8 * 8 + i] = sv[i];
        part[2][r0 * D + c8 * 8 + i] = vmax[i];
        part[3][r0 * D + c8 * 8 + i] = vmin[i];
      }
    }
  }
  __syncthreads();
  if (t < D) {
    float a = 0.f, bb = 0.f, mx = -INFINITY, mn = INFINITY;
    for (int r = 0; r < rpi && r < S; ++r) {   // fixed order: deterministic means
      a += part[0][r * D + t];
      bb += part[1][r * D + t];
      mx = fmaxf(mx, part[2][r * D + t]);
      mn = fminf(mn, part[3][r * D + t]);
    }
    const float mv = (smooth & 2) ? __fdiv_rn(bb, (float)S) : 0.f;
    const float am = fmaxf(fabsf(mx - mv), fabsf(mn - mv));
    reinterpret_cast<float*>(ws + g.off_muk)[(int64_t)bh * g.DV + t] = (smooth & 1) ? __fdiv_rn(a, (float)S) : 0.f;
    reinterpret_cast<float*>(ws + g.off_mu)[(int64_t)bh * g.DV + t] = mv;
    reinterpret_cast<float*>(ws + g.off_sv)[(int64_t)bh * g.DV + t] = __fdiv_rn(fmaxf(am, 1e-12f), 448.f);
  }
}

// Operands of one 128-token chunk of one head (blockIdx.x = head * nc + chunk): Q8 and K~8 rows with
// their per-row scales (sk pre-multiplied by scale * log2 e) and the chunk of V~8^T, all in the MMA's
// K-major core-matrix layout.  Quotients x / scale correctly rounded, as the reference divides.
__global__ void __launch_bounds__(256) attn_fp8_pack_kernel(const __nv_bfloat16* __restrict__ q,
                                                            const __nv_bfloat16* __restrict__ k,
                                                            const __nv_bfloat16* __restrict__ v, int64_t sb,
                                                            int64_t sh, int64_t ss, const F8LGeom g, float scale,
                                                            uint8_t* __restrict__ ws) {
  __shared__ __align__(16) __nv_bfloat16 tile[128 * 128];   // the chunk's v rows [128][D]
  __shared__ float muk[128], muv[128], svs[128];
  const int bh = blockIdx.x / g.nc, j = blockIdx.x - bh * g.nc;
  const int b = bh / g.H, h = bh - b * g.H;
  const __nv_bfloat16* qh = q + b * sb + h * sh;
  const __nv_bfloat16* kh = k + b * sb + h * sh;
  const __nv_bfloat16* vh = v + b * sb + h * sh;
  const int S = g.S, D = g.D, D8 = D / 8;
  const int t = threadIdx.x, lane = t & 31;
  if (t < D) {
    muk[t] = reinterpret_cast<const float*>(ws + g.off_muk)[(int64_t)bh * g.DV + t];
    muv[t] = reinterpret_cast<const float*>(ws + g.off_mu)[(int64_t)bh * g.DV + t];
    svs[t] = reinterpret_cast<const float*>(ws + g.off_sv)[(int64_t)bh * g.DV + t];
  }
  // the chunk's v rows into shared memory (zeros past S) by asynchronous copies that run while the
  // Q / K~ rows below are quantized
  for (int i = t; i < 128 * D8; i += 256) {
    const int rr = i / D8, cc = i - rr * D8, tok = j * 128 + rr;
    const __nv_bfloat16* src = vh + (int64_t)(tok < S ? tok : 0) * ss + cc * 8;
    const uint32_t dst = smem_u32(tile + rr * D + cc * 8);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(tok < S ? 16 : 0)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  __syncthreads();   // the statistics above are visible to every thread
  // Q8 and K~8: 8 lanes per row (lane & 7 = 16-element chunk along d), 4 rows per warp
  {
    const int kc = lane & 7, nkc = g.DK / 16, dkc = D / 16;
    const float kmul = scale * 1.4426950408889634f;
    uint8_t* qp = ws + g.off_q + (int64_t)bh * g.qk_head + (int64_t)j * 128 * g.DK;
    uint8_t* kp = ws + g.off_k + (int64_t)bh * g.qk_head + (int64_t)j * 128 * g.DK;
    float* sq_g = reinterpret_cast<float*>(ws + g.off_sq) + (int64_t)bh * g.S_pad + j * 128;
    float* sk_g = reinterpret_cast<float*>(ws + g.off_sk) + (int64_t)bh * g.S_pad + j * 128;
    for (int rr = (t >> 5) * 4 + (lane >> 3); rr < 128; rr += 32) {
      const int r = j * 128 + rr;
      float xq[16], xk[16];
      float aq = 0.f, ak = 0.f;
      if (r < S && kc < dkc) {
        load8(qh + r * ss + 16 * kc, xq);
        load8(qh + r * ss + 16 * kc + 8, xq + 8);
        load8(kh + r * ss + 16 * kc, xk);
        load8(kh + r * ss + 16 * kc + 8, xk + 8);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          xk[e] -= muk[16 * kc + e];
          aq = fmaxf(aq, fabsf(xq[e]));
          ak = fmaxf(ak, fabsf(xk[e]));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) xq[e] = xk[e] = 0.f;
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
        aq = fmaxf(aq, __shfl_xor_sync(0xffffffffu, aq, o));
        ak = fmaxf(ak, __shfl_xor_sync(0xffffffffu, ak, o));
      }
      const float scq = __fdiv_rn(fmaxf(aq, 1e-12f), 448.f);
      const float sck = __fdiv_rn(fmaxf(ak, 1e-12f), 448.f);
      if (kc < nkc) {
        const int64_t off = (rr >> 3) * 8 * g.DK + kc * 128 + (rr & 7) * 16;
        *reinterpret_cast<uint4*>(qp + off) = e4m3x16_div(xq, scq, __frcp_rn(scq));
        *reinterpret_cast<uint4*>(kp + off) = e4m3x16_div(xk, sck, __frcp_rn(sck));
      }
      if (kc == 0) {
        sq_g[rr] = r < S ? scq : 0.f;
        sk_g[rr] = r < S ? sck * kmul : 0.f;
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();   // every thread's copies of the v rows have landed
  // V~8^T of the chunk: one (16-key block, column d) per thread, consecutive threads on consecutive d
  {
    uint8_t* vp = ws + g.off_v + (int64_t)bh * g.v_head + (int64_t)j * g.DV * 128;
    for (int i = t; i < 8 * D; i += 256) {
      const int kc = i / D, d = i - kc * D;
      const float m = muv[d], sc = svs[d];
      float x[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int rr = kc * 16 + e;
        x[e] = j * 128 + rr < S ? __bfloat162float(tile[rr * D + d]) - m : 0.f;
      }
      *reinterpret_cast<uint4*>(vp + (d >> 3) * 1024 + kc * 128 + (d & 7) * 16) = e4m3x16_div(x, sc, __frcp_rn(sc));
    }
  }
}

__global__ void __launch_bounds__(kF8LWarps * 32, 1)
    attn_fp8_long_kernel(const F8LGeom g, const uint8_t* __restrict__ ws, const F8LSmem L,
                         __nv_bfloat16* __restrict__ out, int64_t osb, int64_t osh, int64_t oss) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar = base + L.bar;
  const uint32_t kv_full = bar, kv_free = bar + 8, q_full = bar + 16, q_free = bar + 24, o_full = bar + 32,
                 o_free = bar + 40, drain = bar + 48;
  auto s_full = [&](int i) { return bar + 56 + 8u * i; };    // [4]
  auto s_free = [&](int i) { return bar + 88 + 8u * i; };    // [4]
  auto p_full = [&](int i) { return bar + 120 + 8u * i; };   // [2]
  auto p_free = [&](int i) { return bar + 136 + 8u * i; };   // [2]
  auto v_full = [&](int i) { return bar + 152 + 8u * i; };   // [4]
  auto v_free = [&](int i) { return bar + 184 + 8u * i; };   // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L.bar + 224);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nc = g.nc, S = g.S, DK = g.DK, DV = g.DV;
  const uint32_t qbytes = 128u * (uint32_t)DK, vbytes = (uint32_t)DV * 128u;
  int* err = &g_attn_err;

  if (warp == 0 && lane == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_free, 1);
    mbar_init(q_full, 1);
    mbar_init(q_free, 1);
    mbar_init(o_full, 1);
    mbar_init(o_free, kF8LSoftmax);
    mbar_init(drain, 1);
    for (int i = 0; i < (int)kF8LSBuf; ++i) {
      mbar_init(s_full(i), 1);
      mbar_init(s_free(i), kF8LSoftmax);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(p_full(i), kF8LSoftmax);
      mbar_init(p_free(i), 1);
    }
    for (int i = 0; i < kF8LStages; ++i) {
      mbar_init(v_full(i), 1);
      mbar_init(v_free(i), 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ loads
      const uint32_t skbytes = (uint32_t)g.S_pad * 4u;
      uint32_t hc = 0, tcnt = 0, vc = 0;
      bool ok = true;
      for (int64_t bh = blockIdx.x; bh < g.BH && ok; bh += gridDim.x, ++hc) {
        if (!(ok = mbar_wait(kv_free, (hc & 1u) ^ 1u, err, kDevErrTimeoutEmpty))) break;
        mbar_arrive_expect_tx(kv_full, (uint32_t)nc * qbytes + skbytes);
        for (int j = 0; j < nc; ++j)
          bulk_load(base + L.k + (uint32_t)j * qbytes, ws + g.off_k + bh * g.qk_head + (int64_t)j * qbytes, qbytes,
                    kv_full);
        bulk_load(base + L.sk, ws + g.off_sk + bh * g.S_pad * 4, skbytes, kv_full);
        for (int qt = 0; qt < nc && ok; ++qt, ++tcnt) {
          if (!(ok = mbar_wait(q_free, (tcnt & 1u) ^ 1u, err, kDevErrTimeoutEmpty))) break;
          mbar_arrive_expect_tx(q_full, qbytes);
          bulk_load(base + L.q, ws + g.off_q + bh * g.qk_head + (int64_t)qt * qbytes, qbytes, q_full);
          for (int j = 0; j < nc; ++j, ++vc) {
            const int st = (int)(vc % kF8LStages);
            if (!(ok = mbar_wait(v_free(st), ((vc / kF8LStages) & 1u) ^ 1u, err, kDevErrTimeoutEmpty))) break;
            mbar_arrive_expect_tx(v_full(st), vbytes);
            bulk_load(base + L.v + (uint32_t)st * vbytes, ws + g.off_v + bh * g.v_head + (int64_t)j * vbytes, vbytes,
                      v_full(st));
          }
        }
      }
      // our own copies still in flight complete before the CTA retires (bounded)
      if (hc > 0) mbar_wait(kv_full, (hc - 1) & 1u, err, kDevErrTimeoutFull);
      if (tcnt > 0) mbar_wait(q_full, (tcnt - 1) & 1u, err, kDevErrTimeoutFull);
      for (uint32_t n = vc > kF8LStages ? vc - kF8LStages : 0; n < vc; ++n)
        mbar_wait(v_full((int)(n % kF8LStages)), (n / kF8LStages) & 1u, err, kDevErrTimeoutFull);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issue
      const uint32_t id_s = idesc_f8_e4m3(128), id_o = idesc_f8_e4m3((uint32_t)DV);
      const uint32_t sbo_qk = 8u * (uint32_t)DK;   // bytes between 8-row core-matrix groups
      const int nks = DK / 32;
      uint32_t hc = 0, tcnt = 0, sc = 0, pc = 0, vc = 0;
      bool ok = true;
      auto issue_s = [&](int j) -> bool {   // scores of key chunk j into buffer sc % kF8LSBuf
        const int b = (int)(sc % kF8LSBuf);
        if (!mbar_wait(s_free(b), ((sc / kF8LSBuf) & 1u) ^ 1u, err, kDevErrTimeoutEmpty)) return false;
        tc_fence_after();
        for (int ks = 0; ks < nks; ++ks)
          mma_f8f6f4(tmem + kF8LTmemS + 128u * b, smem_desc(base + L.q + 256u * ks, 128, sbo_qk, 0),
                     smem_desc(base + L.k + (uint32_t)j * qbytes + 256u * ks, 128, sbo_qk, 0), id_s,
                     ks > 0 ? 1u : 0u);
        tc_commit(s_full(b));
        ++sc;
        return true;
      };
      for (int64_t bh = blockIdx.x; bh < g.BH && ok; bh += gridDim.x, ++hc) {
        if (!(ok = mbar_wait(kv_full, hc & 1u, err, kDevErrTimeoutFull))) break;
        for (int qt = 0; qt < nc && ok; ++qt, ++tcnt) {
          if (!(ok = mbar_wait(q_full, tcnt & 1u, err, kDevErrTimeoutFull))) break;
          tc_fence_after();
          for (int j = 0; j < nc && ok; ++j) ok = issue_s(j);          // pass 1
          if (ok) ok = issue_s(0);                                      // pass 2, ahead of the PV products
          if (ok) ok = mbar_wait(o_free, (tcnt & 1u) ^ 1u, err, kDevErrTimeoutTmem);
          for (int j = 0; j < nc && ok; ++j) {
            if (j + 1 < nc) {
              if (!(ok = issue_s(j + 1))) break;
            } else {
              tc_commit(q_free);   // every QK^T of this tile issued: Q's buffer is free once they ran
            }
            const int pb = (int)(pc & 1u);
            const int st = (int)(vc % kF8LStages);
            if (!(ok = mbar_wait(p_full(pb), (pc >> 1) & 1u, err, kDevErrTimeoutFull))) break;
            if (!(ok = mbar_wait(v_full(st), (vc / kF8LStages) & 1u, err, kDevErrTimeoutFull))) break;
            tc_fence_after();
            for (int ks = 0; ks < 4; ++ks)
              mma_f8f6f4(tmem + kF8LTmemO, smem_desc(base + L.p + (uint32_t)pb * 16384u + 256u * ks, 128, 1024, 0),
                         smem_desc(base + L.v + (uint32_t)st * vbytes + 256u * ks, 128, 1024, 0), id_o,
                         (j > 0 || ks > 0) ? 1u : 0u);
            tc_commit(p_free(pb));
            tc_commit(v_free(st));
            ++pc;
            ++vc;
          }
          if (ok) tc_commit(o_full);
        }
        if (ok) tc_commit(kv_free);   // this head's K~8 and sk are no longer read once these MMAs ran
      }
      tc_commit(drain);
      mbar_wait(drain, 0, err, kDevErrTimeoutDrain);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue
    const int quad = warp & 3;
    const int slice = (warp - 2) >> 2;            // key columns [32 slice, 32 slice + 32) of a chunk
    const int r = quad * 32 + lane;               // row of the query tile == TMEM lane
    const uint32_t lane_addr = (uint32_t)(quad * 32) << 16;
    float* red_m = reinterpret_cast<float*>(gbase + L.red_m);   // [slice][128]
    float* red_l = reinterpret_cast<float*>(gbase + L.red_l);
    const float* sk = reinterpret_cast<const float*>(gbase + L.sk);
    const int nlast = S - (nc - 1) * 128 - 32 * slice;   // this warp's valid keys in the last chunk
    constexpr float kLog2_448 = 8.8073549220576041f;
    uint32_t hc = 0, tcnt = 0, sc = 0, pc = 0;
    bool ok = true;
    uint32_t va[16], vb[16];
    // this warp's 32 columns of the next score chunk: the first 16 loaded and waited for, the other
    // 16 left in flight while the first are processed; finish_s waits for them and frees the buffer
    auto start_s = [&]() -> bool {
      const int b = (int)(sc % kF8LSBuf);
      if (!mbar_wait(s_full(b), (sc / kF8LSBuf) & 1u, err, kDevErrTimeoutFull)) return false;
      tc_fence_after();
      const uint32_t ta = tmem + lane_addr + kF8LTmemS + 128u * b + 32u * slice;
      tmem_ld_32x32b_x16(ta, va);
      tmem_wait_ld();
      reg_fence16(va);
      tmem_ld_32x32b_x16(ta + 16, vb);
      return true;
    };
    auto finish_s = [&]() {
      tmem_wait_ld();
      reg_fence16(vb);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free((int)(sc % kF8LSBuf)));
      ++sc;
    };
    for (int64_t bh = blockIdx.x; bh < g.BH && ok; bh += gridDim.x, ++hc) {
      if (!(ok = mbar_wait(kv_full, hc & 1u, err, kDevErrTimeoutFull))) break;
      const float* sq_g = reinterpret_cast<const float*>(ws + g.off_sq) + bh * g.S_pad;
      const float* sv_g = reinterpret_cast<const float*>(ws + g.off_sv) + bh * DV;
      const float* mu_g = reinterpret_cast<const float*>(ws + g.off_mu) + bh * DV;
      for (int qt = 0; qt < nc && ok; ++qt, ++tcnt) {
        const float sqr = sq_g[qt * 128 + r];
        // pass 1: row max of acc * sk (scores in log2 units are acc * sk * sqr, sqr > 0 for real rows)
        float m = -INFINITY;
        for (int j = 0; j < nc && ok; ++j) {
          if (!(ok = start_s())) break;
          const float4* sk4 = reinterpret_cast<const float4*>(sk + j * 128 + 32 * slice);
          const bool full = j + 1 < nc || nlast >= 32;
          const float m1 = full ? f8l_half_max<false>(va, sk4, 16) : f8l_half_max<true>(va, sk4, nlast);
          finish_s();
          const float m2 = full ? f8l_half_max<false>(vb, sk4 + 4, 16) : f8l_half_max<true>(vb, sk4 + 4, nlast - 16);
          m = max3f(m, m1, m2);
        }
        red_m[slice * 128 + r] = m;
        named_bar_sync(1 + quad, 32 * kF8LSlices);
        float mr = red_m[r];
#pragma unroll
        for (int s = 1; s < kF8LSlices; ++s) mr = fmaxf(mr, red_m[s * 128 + r]);
        // fl(x * sqr) is monotone in x for sqr >= 0, so the row max of the scores is mr * sqr exactly
        const float nmc = kLog2_448 - mr * sqr;
        // pass 2: P' = 448 exp(s - max) = 2^(acc sk sqr - max + log2 448), row sums, P8 = e4m3(P')
        const unsigned long long sq2 = f32x2_pack(sqr, sqr), nm2 = f32x2_pack(nmc, nmc);
        unsigned long long l2a = f32x2_pack(0.f, 0.f), l2b = l2a;
        for (int j = 0; j < nc && ok; ++j) {
          if (!(ok = start_s())) break;
          const int pb = (int)(pc & 1u);
          if (!(ok = mbar_wait(p_free(pb), ((pc >> 1) & 1u) ^ 1u, err, kDevErrTimeoutEmpty))) {
            finish_s();
            break;
          }
          const float4* sk4 = reinterpret_cast<const float4*>(sk + j * 128 + 32 * slice);
          const bool full = j + 1 < nc || nlast >= 32;
          // K-major core matrices of P: (row group, 16-key chunk) at rg*1024 + kc*128
          uint8_t* prow = gbase + L.p + pb * 16384 + (r >> 3) * 1024 + 2 * slice * 128 + (r & 7) * 16;
          float p[16];
          if (full)
            f8l_half_exp<false>(va, sk4, 16, sq2, nm2, p, l2a, l2b);
          else
            f8l_half_exp<true>(va, sk4, nlast, sq2, nm2, p, l2a, l2b);
          *reinterpret_cast<uint4*>(prow) = e4m3x16(p, 1.f);
          finish_s();
          if (full)
            f8l_half_exp<false>(vb, sk4 + 4, 16, sq2, nm2, p, l2a, l2b);
          else
            f8l_half_exp<true>(vb, sk4 + 4, nlast - 16, sq2, nm2, p, l2a, l2b);
          *reinterpret_cast<uint4*>(prow + 128) = e4m3x16(p, 1.f);
          fence_async_shared();
          __syncwarp();
          if (lane == 0) mbar_arrive(p_full(pb));
          ++pc;
        }
        float la0, la1, lb0, lb1;
        f32x2_unpack(l2a, &la0, &la1);
        f32x2_unpack(l2b, &lb0, &lb1);
        red_l[slice * 128 + r] = (la0 + la1) + (lb0 + lb1);
        named_bar_sync(1 + quad, 32 * kF8LSlices);
        float lr = red_l[r];
#pragma unroll
        for (int s = 1; s < kF8LSlices; ++s) lr += red_l[s * 128 + r];
        // epilogue: 8-column groups slice, slice + 4, ... of O
        if (ok && (ok = mbar_wait(o_full, tcnt & 1u, err, kDevErrTimeoutTmem))) {
          tc_fence_after();
          const int ng = DV / 8;
          uint32_t ov[4][8];
#pragma unroll
          for (int kq = 0; kq < 4; ++kq)
            if (slice + 4 * kq < ng) tmem_ld_32x32b_x8(tmem + lane_addr + kF8LTmemO + 8u * (slice + 4 * kq), ov[kq]);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(o_free);
          const int tq = qt * 128 + r;
          if (tq < S) {
            const float f = 1.0f / lr;
            const int b = (int)(bh / g.H), h = (int)(bh - (int64_t)b * g.H);
            __nv_bfloat16* o = out + b * osb + (int64_t)tq * oss + h * osh;
#pragma unroll
            for (int kq = 0; kq < 4; ++kq) {
              const int gi = slice + 4 * kq;
              if (gi < ng) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const int d = 8 * gi + 2 * e;
                  __nv_bfloat162 hv = __floats2bfloat162_rn(
                      __fmaf_rn(__uint_as_float(ov[kq][2 * e]), f * __ldg(sv_g + d), __ldg(mu_g + d)),
                      __fmaf_rn(__uint_as_float(ov[kq][2 * e + 1]), f * __ldg(sv_g + d + 1), __ldg(mu_g + d + 1)));
                  w[e] = *reinterpret_cast<uint32_t*>(&hv);
                }
                *reinterpret_cast<uint4*>(o + 8 * gi) = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

static int launch_fp8_long(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                           int64_t sb, int64_t sh, int64_t ss, float scale, void* out, int64_t osb, int64_t osh,
                           int64_t oss, int smooth, uint8_t* ws, cudaStream_t s) {
  const F8LGeom g = make_f8l_geom(B, H, S, D);
  const F8LSmem L = f8l_smem_layout(g);
  const auto* Q = static_cast<const __nv_bfloat16*>(q);
  const auto* K = static_cast<const __nv_bfloat16*>(k);
  const auto* V = static_cast<const __nv_bfloat16*>(v);
  attn_fp8_colstats_kernel<<<(unsigned)g.BH, 256, 0, s>>>(K, V, sb, sh, ss, g, smooth, ws);
  if (int st = launch_status("vf4_attn fp8 (column statistics)")) return st;
  attn_fp8_pack_kernel<<<(unsigned)(g.BH * g.nc), 256, 0, s>>>(Q, K, V, sb, sh, ss, g, scale, ws);
  if (int st = launch_status("vf4_attn fp8 (operand pack)")) return st;
  if (int st = smem_optin(attn_fp8_long_kernel, (int)L.total)) return st;
  const int grid = (int)(g.BH < num_sms() ? g.BH : num_sms());   // persistent: whole heads per CTA
  attn_fp8_long_kernel<<<grid, kF8LWarps * 32, L.total, s>>>(g, ws, L, static_cast<__nv_bfloat16*>(out), osb, osh,
                                                             oss);
  return launch_status("vf4_attn fp8 (forward)");
}

// ---------------------------------------------------------------------------------------
// bf16 attention: the route the reference keeps for blocks left in bf16 (its qattention wrapper
// and timm's Attention call torch's scaled_dot_product_attention): out = softmax(q k^T * scale) v
// with bf16 q, k, v, fp32 accumulation and an exact (whole-row) softmax.  Head dim 64, S <= 288.
// Persistent CTAs (one per SM, 16 warps) run one stream of 128-query tiles over the B*H heads:
//   warp 0       TMA loads (128-byte swizzle): K (with the head's tail query rows) into one
//                buffer, V into one of two (the next head's V lands while this head runs), Q
//                one 128-row tile at a time
//   warp 1       S = Q K^T (tcgen05.mma kind::f16; Q and K straight from the TMA tiles,
//                K-major) into TMEM, keys padded to a multiple of 16 (chunks of <= 256); the
//                next tile's S is issued as soon as the softmax has read this one, before this
//                tile's O = P V (V straight from its TMA tile as an MN-major operand) into one
//                of two O buffers; commits release Q, K and V the moment the MMAs are done
//   warps 2-13   (TMEM lane quadrant x key slice) pass 1 row max, pass 2 P = 2^((s - max) c),
//                row sums, P -> bf16 (K-major core matrices); the previous tile's epilogue
//                (O / rowsum -> bf16, each thread storing its row's 16-byte column chunks)
//                follows, across head boundaries
//   warps 14-15  query rows past the last full 128-row tile when there are at most 4 of them
//                (S = 257: one): plain FMAs over the same shared-memory K and V, overlapped
//                with the tiles (a 128-row MMA tile for one row costs a whole tile's MMA ->
//                softmax -> PV chain)
// ---------------------------------------------------------------------------------------
constexpr uint32_t kB16TmemS = 0, kB16TmemO = 320;
constexpr int kB16TailWarps = 2, kB16Warps = kFusedWarps + kB16TailWarps, kB16TailMax = 4;

struct Bf16Geom {
  int B, H, S, D;
  int nt, tail, skp;       // MMA query tiles, query rows left to the tail warps, keys padded to 16
  int box_rows, nbox, heads;
  int kv_hs;
  float scale;
  __nv_bfloat16* out;      // out element (b, h, s, d) at out + b osb + h osh + s oss + d
  int64_t osb, osh, oss;
  float* amax;             // if set: max |out| over the whole output (atomic, as uint bits)
  uint32_t qb, kb, vb[2], tqb, pb, red, bar, total;
};

static Bf16Geom make_bf16_geom(int64_t B, int64_t H, int64_t S, int64_t D, float scale) {
  Bf16Geom g{};
  g.B = (int)B;
  g.H = (int)H;
  g.S = (int)S;
  g.D = (int)D;
  g.skp = (int)align_up(S, 16);
  g.tail = (S > 128 && S % 128 != 0 && S % 128 <= kB16TailMax) ? (int)(S % 128) : 0;
  g.nt = (int)((S - g.tail + 127) / 128);
  g.nbox = g.skp <= 256 ? 1 : 2;
  g.box_rows = (int)align_up((g.skp + g.nbox - 1) / g.nbox, 8);
  g.heads = (int)(B * H);
  g.scale = scale;
  const uint32_t rawb = (uint32_t)(g.nbox * g.box_rows) * 128u;   // a multiple of 1024
  uint32_t o = 0;
  g.qb = o;     o += 128u * 128u;
  g.kb = o;     o += rawb;
  g.vb[0] = o;  o += rawb;
  g.vb[1] = o;  o += rawb;
  g.tqb = o;    o += 1024u;                       // 8 query rows (tail rows, zero past S)
  g.pb = o;     o += 256u * (uint32_t)g.skp;      // P: 128 rows x skp bf16, K-major core matrices
  o = (uint32_t)align_up(o, 16);
  g.red = o; o += (uint32_t)(3 * kSlices * 128 + kB16TailMax * (g.skp + 2 * 64 + 4)) * 4u;
  o = (uint32_t)align_up(o, 16);
  g.bar = o; o += 128;
  g.total = o + 1024;
  return g;
}

static bool bf16_attn_ok(int64_t S, int64_t D) {
  if (D != 64 || S < 1 || S > 288) return false;
  return make_bf16_geom(1, 1, S, D, 1.f).total <= 227u * 1024u;
}

// Instruction descriptor for kind::f16 with bf16 A and B, fp32 accumulation, K-major A; B K-major
// or (b_mn) MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(uint32_t n, bool b_mn, uint32_t m = 128) {
  return (1u << 4)            // D format: F32
         | (1u << 7)          // A format: BF16
         | (1u << 10)         // B format: BF16
         | ((b_mn ? 1u : 0u) << 16)
         | ((n >> 3) << 17) | ((m >> 4) << 24);
}

VF4_DEV void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

__global__ void __launch_bounds__(kB16Warps * 32, 1)
    attn_bf16_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmT,
                     const Bf16Geom g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (base - raw0);
  const uint32_t bar = base + g.bar;
  const uint32_t q_full = bar, q_free = bar + 8, k_full = bar + 16, k_free = bar + 24, s_full = bar + 32,
                 p_full = bar + 40, drain = bar + 48;
  auto v_full = [&](int sl) { return bar + 56 + 8u * sl; };
  auto v_free = [&](int sl) { return bar + 72 + 8u * sl; };
  auto o_full = [&](int ob) { return bar + 88 + 8u * ob; };
  auto o_free = [&](int ob) { return bar + 104 + 8u * ob; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gb + g.bar + 120);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t sbo_p = 16u * (uint32_t)g.skp;   // bytes per 8-row group of P
  const float c = g.scale * 1.4426950408889634f;
  const uint32_t kv_release = g.tail > 0 ? 2u : 1u;   // MMA commit (+ the tail warps)
  int* err = &g_attn_err;

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_free, 1);
    mbar_init(k_full, 1);
    mbar_init(k_free, kv_release);
    mbar_init(s_full, 1);
    mbar_init(p_full, kFusedCompute);
    mbar_init(drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(v_full(i), 1);
      mbar_init(v_free(i), kv_release);
      mbar_init(o_full(i), 1);
      mbar_init(o_free(i), kFusedCompute);
    }
    fence_mbar_init();
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    if (g.tail > 0) tma_prefetch(&tmT);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  fence_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA loads
    if (lane == 0) {
      const uint32_t kv_bytes = (uint32_t)(g.nbox * g.box_rows) * 128u;
      int hi = 0, qi = 0;
      bool ok = true;
      for (int head = blockIdx.x; head < g.heads && ok; head += gridDim.x, ++hi) {
        const int b = head / g.H, h = head - b * g.H, sl = hi & 1;
        if (hi >= 1 && !mbar_wait(k_free, (uint32_t)(hi - 1) & 1u, err, kDevErrTimeoutEmpty)) break;
        mbar_arrive_expect_tx(k_full, kv_bytes + (g.tail > 0 ? 1024u : 0u));
        for (int j = 0; j < g.nbox; ++j) {
          const int row = j * g.box_rows;
          tma_load_4d(base + g.kb + (uint32_t)row * 128u, &tmK, 0, g.kv_hs ? h : row, g.kv_hs ? row : h, b, k_full);
        }
        if (g.tail > 0) {
          const int row = g.S - g.tail;
          tma_load_4d(base + g.tqb, &tmT, 0, g.kv_hs ? h : row, g.kv_hs ? row : h, b, k_full);
        }
        for (int t = 0; t < g.nt; ++t, ++qi) {
          if (qi > 0 && !mbar_wait(q_free, (uint32_t)(qi - 1) & 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int row = t * 128;
          mbar_arrive_expect_tx(q_full, 128u * 128u);
          tma_load_4d(base + g.qb, &tmQ, 0, g.kv_hs ? h : row, g.kv_hs ? row : h, b, q_full);
          if (t == 0) {   // V of this head after its first Q tile
            if (hi >= 2 && !mbar_wait(v_free(sl), (uint32_t)((hi >> 1) - 1) & 1u, err, kDevErrTimeoutEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(v_full(sl), kv_bytes);
            for (int j = 0; j < g.nbox; ++j) {
              const int vr = j * g.box_rows;
              tma_load_4d(base + (sl ? g.vb[1] : g.vb[0]) + (uint32_t)vr * 128u, &tmV, 0, g.kv_hs ? h : vr, g.kv_hs ? vr : h, b,
                          v_full(sl));
            }
          }
        }
      }
      // no copy may still be writing shared memory when the CTA exits
      if (qi > 0) mbar_wait(q_full, (uint32_t)(qi - 1) & 1u, err, kDevErrTimeoutFull);
      if (hi > 0) {
        mbar_wait(k_full, (uint32_t)(hi - 1) & 1u, err, kDevErrTimeoutFull);
        mbar_wait(v_full((hi - 1) & 1), (uint32_t)((hi - 1) >> 1) & 1u, err, kDevErrTimeoutFull);
        if (hi > 1) mbar_wait(v_full(hi & 1), (uint32_t)((hi - 2) >> 1) & 1u, err, kDevErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    bool ok = true;
    int hi = 0, it = 0, qi = 0;
    // S = Q K^T for the Q tile in the buffer; releases Q, and K after the head's last tile
    auto issue_qk = [&](bool last) {
      const uint32_t qa = base + g.qb, kbase = base + g.kb;
      for (int n0 = 0; n0 < g.skp;) {
        const int n = g.skp - n0 >= 256 ? 256 : g.skp - n0;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(tmem + kB16TmemS + (uint32_t)n0, smem_desc(qa + 32u * kk, 16, 1024, 2),
                  smem_desc(kbase + (uint32_t)n0 * 128u + 32u * kk, 16, 1024, 2), idesc_bf16((uint32_t)n, false),
                  kk > 0 ? 1u : 0u);
        n0 += n;
      }
      tc_commit(s_full);
      tc_commit(q_free);
      if (last) tc_commit(k_free);
    };
    if ((int)blockIdx.x < g.heads) {
      ok = mbar_wait(k_full, 0, err, kDevErrTimeoutFull) && mbar_wait(q_full, 0, err, kDevErrTimeoutFull);
      tc_fence_after();
      if (ok && lane == 0) issue_qk(g.nt == 1);
      __syncwarp();
      qi = 1;
    }
    for (int head = blockIdx.x; head < g.heads && ok; head += gridDim.x, ++hi) {
      for (int t = 0; t < g.nt; ++t, ++it) {
        // P of tile it written (and its S read) by every compute warp
        if (!mbar_wait(p_full, (uint32_t)it & 1u, err, kDevErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the next tile's S first, so that its softmax overlaps this tile's PV
        const bool same = t + 1 < g.nt;
        if (same || head + (int)gridDim.x < g.heads) {
          if ((!same && !mbar_wait(k_full, (uint32_t)(hi + 1) & 1u, err, kDevErrTimeoutFull)) ||
              !mbar_wait(q_full, (uint32_t)qi & 1u, err, kDevErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) issue_qk(same ? t + 1 == g.nt - 1 : g.nt == 1);
          __syncwarp();
          ++qi;
        }
        const int ob = it & 1, use = it >> 1;
        if ((use > 0 && !mbar_wait(o_free(ob), (uint32_t)(use - 1) & 1u, err, kDevErrTimeoutEmpty)) ||
            (t == 0 && !mbar_wait(v_full(hi & 1), (uint32_t)(hi >> 1) & 1u, err, kDevErrTimeoutFull))) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t t_o = tmem + kB16TmemO + 64u * (uint32_t)ob, vbase = base + ((hi & 1) ? g.vb[1] : g.vb[0]);
          for (int kk = 0; kk < g.skp / 16; ++kk)
            mma_f16(t_o, smem_desc(base + g.pb + 256u * kk, 128, sbo_p, 0), smem_desc(vbase + 2048u * kk, 1024, 1024, 2),
                    idesc_bf16(64, true), kk > 0 ? 1u : 0u);
          tc_commit(o_full(ob));
          if (t == g.nt - 1) tc_commit(v_free(hi & 1));
        }
        __syncwarp();
      }
    }
    if (lane == 0) {
      tc_commit(drain);
      mbar_wait(drain, 0, err, kDevErrTimeoutDrain);
    }
    __syncwarp();
  } else if (warp < kFusedWarps) {
    // ------------------------------------------------------------ softmax and epilogue
    const int cw = warp - 2;
    const int qd = warp & 3;
    const int cs = cw >> 2;
    const uint32_t qbar = 2u + (uint32_t)qd;
    float* red = reinterpret_cast<float*>(gb + g.red);
    float* red_m = red;                         // [kSlices][128]
    float* red_l = red_m + kSlices * 128;       // [2][kSlices][128]
    const int S = g.S;
    const int nkb = g.skp / 16;
    const int b0 = cs * nkb / kSlices, b1 = (cs + 1) * nkb / kSlices;
    const int c0 = cs * 8 / kSlices, c1 = (cs + 1) * 8 / kSlices;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const int r = qd * 32 + lane;
    bool ok = true;
    // max |out| over this thread's stores (the amax of the proj input), kept as the bit patterns of
    // the bf16 magnitudes in two 16-bit lanes: unsigned order of non-negative bf16 bits is their
    // numeric order and a NaN (0x7FC0) sorts above +inf, so a NaN output reaches the amax as the
    // reference's torch amax would give it, instead of being dropped by a float max
    uint32_t out_max2 = 0;
    // O / rowsum -> bf16, each thread storing its row's columns of this slice straight to global
    // memory (the row sums of every slice were written before the quadrant barrier of the next
    // tile's pass 1, which this warp has passed)
    auto epilogue = [&](int itt, int head, int tl) {
      const int b = head / g.H, h = head - b * g.H;
      const int row = tl * 128 + r;
      const bool act = ok && tl * 128 + qd * 32 < S;
      const int ob = itt & 1;
      constexpr int kMaxChunks = (8 + kSlices - 1) / kSlices;
      uint32_t ov[kMaxChunks][8];
      if (act) {
#pragma unroll
        for (int k = 0; k < kMaxChunks; ++k)
          if (c0 + k < c1) tmem_ld_32x32b_x8(tmem + lane_base + kB16TmemO + 64u * ob + 8 * (c0 + k), ov[k]);
        tmem_wait_ld();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free(ob));
      if (act && row < S) {
        const float* rl = red_l + ob * (kSlices * 128);
        float lsum = 0.f;
#pragma unroll
        for (int k = 0; k < kSlices; ++k) lsum += rl[k * 128 + r];
        const float f = 1.0f / lsum;
        __nv_bfloat16* orow = g.out + (int64_t)b * g.osb + (int64_t)h * g.osh + (int64_t)row * g.oss;
#pragma unroll
        for (int k = 0; k < kMaxChunks; ++k) {
          const int cc = c0 + k;
          if (cc < c1) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __nv_bfloat162 hv = __floats2bfloat162_rn(__uint_as_float(ov[k][2 * i]) * f,
                                                        __uint_as_float(ov[k][2 * i + 1]) * f);
              w[i] = *reinterpret_cast<uint32_t*>(&hv);
              out_max2 = umax_u16x2(out_max2, w[i] & 0x7FFF7FFFu);
            }
            *reinterpret_cast<uint4*>(orow + 8 * cc) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
    };
    int it = 0, prev_head = -1, prev_t = 0;
    for (int head = blockIdx.x; head < g.heads; head += gridDim.x) {
      for (int t = 0; t < g.nt; ++t, ++it) {
        const bool active = ok && t * 128 + qd * 32 < S;
        if (ok) ok = mbar_wait(s_full, (uint32_t)it & 1u, err, kDevErrTimeoutFull);
        tc_fence_after();
        const uint32_t srow = tmem + lane_base + kB16TmemS;
        // pass 1: row max over the valid keys; 16-column TMEM loads, the next one in flight while
        // the current one is reduced
        float m = -INFINITY;
        auto max16 = [&](int u, const uint32_t* v) {
          if (16 * u + 16 <= S) {
#pragma unroll
            for (int e = 0; e < 16; e += 2) m = max3f(m, __uint_as_float(v[e]), __uint_as_float(v[e + 1]));
          } else {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (16 * u + e < S) m = fmaxf(m, __uint_as_float(v[e]));
          }
        };
        if (active && ok && b0 < b1) {
          uint32_t va[16], vb[16];
          tmem_ld_32x32b_x16(srow + 16 * b0, va);
          tmem_wait_ld();
          reg_fence16(va);
          for (int u = b0; u < b1; u += 2) {
            if (u + 1 < b1) tmem_ld_32x32b_x16(srow + 16 * (u + 1), vb);
            max16(u, va);
            tmem_wait_ld();
            reg_fence16(vb);
            if (u + 1 < b1) {
              if (u + 2 < b1) tmem_ld_32x32b_x16(srow + 16 * (u + 2), va);
              max16(u + 1, vb);
              tmem_wait_ld();
              reg_fence16(va);
            }
          }
        }
        red_m[cs * 128 + r] = m;
        named_bar_sync(qbar, 32 * kSlices);
#pragma unroll
        for (int k = 0; k < kSlices; ++k) m = fmaxf(m, red_m[k * 128 + r]);
        // P is single-buffered: the previous tile's PV must be done reading it
        if (it > 0 && ok) ok = mbar_wait(o_full((it - 1) & 1), (uint32_t)((it - 1) >> 1) & 1u, err, kDevErrTimeoutTmem);
        // pass 2: P = 2^((s - max) c), row sums, P -> bf16
        const float nmc = -m * c;
        float lsum = 0.f;
        uint8_t* prow = gb + g.pb + (uint32_t)(r >> 3) * sbo_p + (uint32_t)(r & 7) * 16u;
        const unsigned long long c2 = f32x2_pack(c, c), nmc2 = f32x2_pack(nmc, nmc);
        unsigned long long lsum2 = f32x2_pack(0.f, 0.f);
        auto exp16 = [&](int u, const uint32_t* v) {
          float p[16];
          // x = s c - m c by pairs, 2^x on the special-function unit; keys >= S give 0
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            float x0, x1;
            f32x2_unpack(fma_f32x2(f32x2_pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1])), c2, nmc2), &x0,
                         &x1);
            p[2 * i] = ex2_approx(x0);
            p[2 * i + 1] = ex2_approx(x1);
          }
          if (16 * u + 16 > S) {
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (16 * u + e >= S) p[e] = 0.f;
          }
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            lsum2 = add_f32x2(lsum2, f32x2_pack(p[2 * i], p[2 * i + 1]));
            __nv_bfloat162 pv = __floats2bfloat162_rn(p[2 * i], p[2 * i + 1]);
            w[i] = *reinterpret_cast<uint32_t*>(&pv);
          }
          *reinterpret_cast<uint4*>(prow + (uint32_t)(2 * u) * 128u) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(prow + (uint32_t)(2 * u + 1) * 128u) = make_uint4(w[4], w[5], w[6], w[7]);
        };
        if (active && ok && b0 < b1) {
          uint32_t va[16], vb[16];
          tmem_ld_32x32b_x16(srow + 16 * b0, va);
          tmem_wait_ld();
          reg_fence16(va);
          for (int u = b0; u < b1; u += 2) {
            if (u + 1 < b1) tmem_ld_32x32b_x16(srow + 16 * (u + 1), vb);
            exp16(u, va);
            tmem_wait_ld();
            reg_fence16(vb);
            if (u + 1 < b1) {
              if (u + 2 < b1) tmem_ld_32x32b_x16(srow + 16 * (u + 2), va);
              exp16(u + 1, vb);
              tmem_wait_ld();
              reg_fence16(va);
            }
          }
        }
        {
          float l0, l1;
          f32x2_unpack(lsum2, &l0, &l1);
          lsum = l0 + l1;
        }
        tc_fence_before();
        red_l[(it & 1) * (kSlices * 128) + cs * 128 + r] = lsum;
        fence_async_shared();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
        if (it > 0) epilogue(it - 1, prev_head, prev_t);
        prev_head = head;
        prev_t = t;
      }
    }
    if (it > 0) {
      if (ok) ok = mbar_wait(o_full((it - 1) & 1), (uint32_t)((it - 1) >> 1) & 1u, err, kDevErrTimeoutTmem);
      tc_fence_after();
      epilogue(it - 1, prev_head, prev_t);
    }
    if (g.amax) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, max(out_max2 & 0xFFFFu, out_max2 >> 16) << 16);
      if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(g.amax), m);
    }
  } else if (g.tail > 0) {
    // ------------------------------------------------------------ tail query rows
    const int tw = warp - kFusedWarps, tid = threadIdx.x - 32 * kFusedWarps;
    float* red = reinterpret_cast<float*>(gb + g.red) + 3 * kSlices * 128;
    float* tp = red;                                   // [kB16TailMax][skp] probabilities
    float* to = tp + kB16TailMax * g.skp;              // [2][kB16TailMax][64] partial outputs
    float* tx = to + 2 * kB16TailMax * 64;             // [2 warps][2] maxima / sums exchange
    const int S = g.S;
    constexpr uint32_t kTailBar = 6;
    constexpr int kKeys = (288 + 63) / 64;             // keys per thread
    bool ok = true;
    int hi = 0;
    uint32_t tail_max = 0;   // fp32 bits of max |out| of the tail rows (NaN propagates, as above)
    for (int head = blockIdx.x; head < g.heads; head += gridDim.x, ++hi) {
      const int b = head / g.H, h = head - b * g.H, sl = hi & 1;
      if (ok) ok = mbar_wait(k_full, (uint32_t)hi & 1u, err, kDevErrTimeoutFull);
      const uint8_t* kt = gb + g.kb;
      const uint8_t* qt = gb + g.tqb;
      float inv_l[kB16TailMax];
      for (int rr = 0; rr < g.tail; ++rr) {
        // the query row as fp32 pairs; each key's dot product by packed FMAs into two accumulators
        unsigned long long q2[32];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint4 a = *reinterpret_cast<const uint4*>(qt + rr * 128 + ((j ^ (rr & 7)) << 4));
          q2[4 * j] = bf16x2_to_f32x2(a.x);
          q2[4 * j + 1] = bf16x2_to_f32x2(a.y);
          q2[4 * j + 2] = bf16x2_to_f32x2(a.z);
          q2[4 * j + 3] = bf16x2_to_f32x2(a.w);
        }
        float s[kKeys];
        float mx = -INFINITY;
#pragma unroll
        for (int u = 0; u < kKeys; ++u) {
          const int key = tid + 64 * u;
          s[u] = -INFINITY;
          if (ok && key < S) {
            unsigned long long acc0 = f32x2_pack(0.f, 0.f), acc1 = acc0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint4 w = *reinterpret_cast<const uint4*>(kt + key * 128 + ((j ^ (key & 7)) << 4));
              acc0 = fma_f32x2(bf16x2_to_f32x2(w.x), q2[4 * j], acc0);
              acc1 = fma_f32x2(bf16x2_to_f32x2(w.y), q2[4 * j + 1], acc1);
              acc0 = fma_f32x2(bf16x2_to_f32x2(w.z), q2[4 * j + 2], acc0);
              acc1 = fma_f32x2(bf16x2_to_f32x2(w.w), q2[4 * j + 3], acc1);
            }
            float a0, a1, b0, b1;
            f32x2_unpack(acc0, &a0, &a1);
            f32x2_unpack(acc1, &b0, &b1);
            s[u] = ((a0 + a1) + (b0 + b1)) * c;
            mx = fmaxf(mx, s[u]);
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) tx[tw] = mx;
        named_bar_sync(kTailBar, 32 * kB16TailWarps);
        mx = fmaxf(tx[0], tx[1]);
        float l = 0.f;
#pragma unroll
        for (int u = 0; u < kKeys; ++u) {
          const int key = tid + 64 * u;
          const float p = (ok && key < S) ? ex2_approx(s[u] - mx) : 0.f;
          if (key < g.skp) tp[rr * g.skp + key] = p;
          l += p;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) tx[2 + tw] = l;
        named_bar_sync(kTailBar, 32 * kB16TailWarps);
        inv_l[rr] = 1.0f / (tx[2] + tx[3]);
        named_bar_sync(kTailBar, 32 * kB16TailWarps);   // tx is reused by the next row
      }
      // K (and the tail query rows) no longer needed
      if (tid == 0) mbar_arrive(k_free);
      if (ok) ok = mbar_wait(v_full(sl), (uint32_t)(hi >> 1) & 1u, err, kDevErrTimeoutFull);
      {
        // thread: head-dim quad dq = tid % 16 (dims 4 dq .. 4 dq + 3), key quarter tid / 16; the two
        // quarters of a warp are merged by a shuffle, the two warps through shared memory
        const int dq = tid & 15, kq = tid >> 4;
        const int quarter = (S + 3) / 4;
        const int j0 = kq * quarter, j1 = min(S, j0 + quarter);
        const uint8_t* vt = gb + (sl ? g.vb[1] : g.vb[0]);
        unsigned long long a[kB16TailMax][2];
#pragma unroll
        for (int rr = 0; rr < kB16TailMax; ++rr) a[rr][0] = a[rr][1] = f32x2_pack(0.f, 0.f);
        if (ok) {
          for (int j = j0; j < j1; ++j) {
            const uint2 w = *reinterpret_cast<const uint2*>(vt + j * 128 + (((dq >> 1) ^ (j & 7)) << 4) + (dq & 1) * 8);
            const unsigned long long v01 = bf16x2_to_f32x2(w.x), v23 = bf16x2_to_f32x2(w.y);
#pragma unroll
            for (int rr = 0; rr < kB16TailMax; ++rr)
              if (rr < g.tail) {
                const float p = tp[rr * g.skp + j];
                const unsigned long long pp = f32x2_pack(p, p);
                a[rr][0] = fma_f32x2(v01, pp, a[rr][0]);
                a[rr][1] = fma_f32x2(v23, pp, a[rr][1]);
              }
          }
        }
#pragma unroll
        for (int rr = 0; rr < kB16TailMax; ++rr)
          if (rr < g.tail) {
            float o[4];
            f32x2_unpack(a[rr][0], &o[0], &o[1]);
            f32x2_unpack(a[rr][1], &o[2], &o[3]);
#pragma unroll
            for (int e = 0; e < 4; ++e) o[e] += __shfl_xor_sync(0xffffffffu, o[e], 16);
            if (lane < 16) {
#pragma unroll
              for (int e = 0; e < 4; ++e) to[(tw * kB16TailMax + rr) * 64 + 4 * dq + e] = o[e];
            }
          }
      }
      named_bar_sync(kTailBar, 32 * kB16TailWarps);
      // V no longer needed
      if (tid == 0) mbar_arrive(v_free(sl));
      for (int i = tid; i < g.tail * 64; i += 32 * kB16TailWarps) {
        const int rr = i >> 6, d = i & 63;
        const int row = S - g.tail + rr;
        if (ok) {
          const __nv_bfloat16 ob = __float2bfloat16_rn((to[rr * 64 + d] + to[(kB16TailMax + rr) * 64 + d]) * inv_l[rr]);
          g.out[(int64_t)b * g.osb + (int64_t)h * g.osh + (int64_t)row * g.oss + d] = ob;
          tail_max = max(tail_max, (uint32_t)(__bfloat16_as_ushort(ob) & 0x7FFFu) << 16);
        }
      }
      named_bar_sync(kTailBar, 32 * kB16TailWarps);   // tp / to are reused by the next head
    }
    if (g.amax) {
      tail_max = __reduce_max_sync(0xffffffffu, tail_max);
      if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(g.amax), tail_max);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

static int launch_bf16(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                       int64_t sb, int64_t sh, int64_t ss, float scale, void* out, int64_t osb, int64_t osh,
                       int64_t oss, float* amax, cudaStream_t s) {
  Bf16Geom g = make_bf16_geom(B, H, S, D, scale);
  g.amax = amax;
  if (amax && cudaMemsetAsync(amax, 0, sizeof(float), s) != cudaSuccess)
    return fail(VF4_ERR_CUDA, "vf4_attn_bf16: amax reset failed");
  g.out = static_cast<__nv_bfloat16*>(out);
  g.osb = osb;
  g.osh = osh;
  g.oss = oss;
  g.kv_hs = sh < ss;
  FusedGeom fg = make_fused_geom(B, H, S, D, scale);   // the head-view maps take D, S, H, B from it
  CUtensorMap tq, tk, tv, tt;
  if (int st = make_head_map(&tq, q, fg, sb, sh, ss, 128, g.kv_hs)) return st;
  if (int st = make_head_map(&tk, k, fg, sb, sh, ss, g.box_rows, g.kv_hs)) return st;
  if (int st = make_head_map(&tv, v, fg, sb, sh, ss, g.box_rows, g.kv_hs)) return st;
  if (int st = make_head_map(&tt, q, fg, sb, sh, ss, 8, g.kv_hs)) return st;
  if (int st = smem_optin(attn_bf16_kernel, (int)g.total)) return st;
  const int grid = g.heads < num_sms() ? g.heads : num_sms();
  attn_bf16_kernel<<<grid, kB16Warps * 32, g.total, s>>>(tq, tk, tv, tt, g);
  return launch_status("vf4_attn_bf16");
}

// ---------------------------------------------------------------------------------------
// bf16 attention, two-slot form (head dim 64, S <= 256 + kB16sExtraMax): the same result as
// attn_bf16_kernel (exact whole-row softmax, P rounded to bf16 after the row sum, O / rowsum) with
// the softmax of one 128-query tile overlapping the MMAs of the next.  TMEM holds two 256-column
// slots; a slot carries one tile through
//   S = Q K^T (fp32, keys < 256)  ->  P = 2^((s - max) c) as bf16 pairs written back over the first
//   128 columns of S  ->  O = P V (kind::f16 with A = P read from tensor memory) into columns
//   128..191 of the slot, whose scores the softmax has finished with
// so the two slots alternate between the tensor core and the softmax warps.  Keys past 256 (S =
// 257, 258) are scored on the CUDA cores (64 fused multiply-adds per row and key) by the epilogue
// warps, for the tile two ahead of the one they finish, and handed to the softmax through shared
// memory; they enter PV as one more K = 16 step whose A operand (those keys' P, zero-padded) sits in
// shared memory.  Query rows past 256 (one or two) are computed whole on the CUDA cores by four
// warps of their own, from the head's K and V in shared memory, while the tiles run: a 128-row
// MMA tile for them would cost a full slot cycle.
//   warp 0       TMA: K (with the query rows past 256) and V of the head (two buffers each,
//                128-byte swizzle), Q one 128-row tile per slot
//   warp 1       TMEM allocator and MMA issuer: S of tile i + 2 as soon as the epilogue has read
//                slot i % 2, O of tile i as soon as its P is written
//   warps 2-5    softmax of slot 0 (one thread per query row, lane quadrant warp % 4)
//   warps 6-9    softmax of slot 1
//   warps 10-13  epilogue: O / rowsum -> bf16, each thread storing its row, and max |out|; the
//                scores of the keys past 256
//   warps 14-17  the rows past 256 (idle when S <= 256)
// ---------------------------------------------------------------------------------------
constexpr int kB16sExtraMax = 2, kB16sWarps = 18;
// first warp of each role (other orders of the roles measured the same)
constexpr int kB16sSoftW = 2, kB16sEpiW = 10, kB16sTailW = 14;
constexpr uint32_t kB16sBarTail = 1;   // named barrier id of the tail warps
// Working storage of the rows past 256 (floats): p [2][272], o partials [16][2][64],
// per-warp maxima and sums [4][2][2]
constexpr uint32_t kB16sTailBytes = (2 * 272 + 16 * 2 * 64 + 4 * 2 * 2) * 4;

struct B16sGeom {
  int B, H, S, D;
  int nt, extra, skp;      // MMA query tiles per head, keys (= query rows) past 256, MMA keys
  int box_rows, nbox, heads, kv_hs;
  float scale;
  __nv_bfloat16* out;
  int64_t osb, osh, oss;
  float* amax;
  uint32_t qb[2], kb[2], vb[2], pe[2], qt[2], tw, se, red, bar, total, kv_bytes;
};

static bool b16s_ok(int64_t S, int64_t D) { return D == 64 && S >= 1 && S <= 256 + kB16sExtraMax; }

static B16sGeom make_b16s_geom(int64_t B, int64_t H, int64_t S, int64_t D, float scale) {
  B16sGeom g{};
  g.B = (int)B;
  g.H = (int)H;
  g.S = (int)S;
  g.D = (int)D;
  g.nt = (int)(((S < 256 ? S : 256) + 127) / 128);
  g.extra = S > 256 ? (int)(S - 256) : 0;
  g.skp = (int)align_up(S < 256 ? S : 256, 16);
  const int rows = g.extra ? 272 : g.skp;                       // K / V rows held (>= S zero-filled)
  g.nbox = rows <= 256 ? 1 : 2;
  g.box_rows = (int)align_up((rows + g.nbox - 1) / g.nbox, 8);
  g.heads = (int)(B * H);
  g.scale = scale;
  g.kv_bytes = (uint32_t)(g.nbox * g.box_rows) * 128u;         // a multiple of 1024
  uint32_t o = 0;
  for (int i = 0; i < 2; ++i) { g.qb[i] = o; o += 128u * 128u; }
  for (int i = 0; i < 2; ++i) { g.kb[i] = o; o += g.kv_bytes; }
  for (int i = 0; i < 2; ++i) { g.vb[i] = o; o += g.kv_bytes; }
  for (int i = 0; i < 2; ++i) { g.pe[i] = o; o += g.extra ? 4096u : 0u; }   // extra keys' P: 128 x 16 bf16
  for (int i = 0; i < 2; ++i) { g.qt[i] = o; o += g.extra ? 1024u : 0u; }   // query rows 256.. (8-row box)
  g.tw = o;  o += g.extra ? kB16sTailBytes : 0u;                            // their working storage
  g.se = o;  o += g.extra ? 2u * 128u * kB16sExtraMax * 4u : 0u;  // extra keys' scores [slot][row][key]
  g.red = o; o += 2u * 128u * 4u;                                          // row sums per slot
  g.bar = o; o += 256;
  g.total = o + 1024;
  return g;
}

VF4_DEV void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}

// 32 lanes x 8 consecutive 32-bit columns from 8 registers per thread.
VF4_DEV void tmem_st_32x32b_x8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

VF4_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(kB16sWarps * 32, 1)
    attn_bf16_slots_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmT,
                           const B16sGeom g) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw0 = smem_u32(smem_raw);
  const uint32_t base = (raw0 + 1023u) & ~1023u;
  uint8_t* gb = smem_raw + (base - raw0);
  const uint32_t bar = base + g.bar;
  auto q_full = [&](int i) { return bar + 8u * i; };
  auto q_free = [&](int i) { return bar + 16u + 8u * i; };
  auto k_full = [&](int i) { return bar + 32u + 8u * i; };
  auto k_free = [&](int i) { return bar + 48u + 8u * i; };
  auto v_full = [&](int i) { return bar + 64u + 8u * i; };
  auto v_free = [&](int i) { return bar + 80u + 8u * i; };
  auto s_full = [&](int i) { return bar + 96u + 8u * i; };
  auto p_full = [&](int i) { return bar + 112u + 8u * i; };
  auto o_full = [&](int i) { return bar + 128u + 8u * i; };
  auto o_free = [&](int i) { return bar + 144u + 8u * i; };
  auto se_full = [&](int i) { return bar + 168u + 8u * i; };
  const uint32_t drain = bar + 160u;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gb + g.bar + 184);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = g.nt, S = g.S;
  // tiles of this CTA: head blockIdx.x + j * gridDim.x, query tile t, flat index i = j * nt + t
  const int my_heads = (int)blockIdx.x < g.heads ? (g.heads - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int T = my_heads * nt;
  int* err = &g_attn_err;

  if (warp == 0 && lane == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(q_full(i), 1);
      mbar_init(q_free(i), g.extra ? 5u : 1u);               // QK commit (+ the epilogue warps' Q reads)
      mbar_init(k_full(i), 1);
      // K: the last QK commit, the softmax warps' extra-key reads and the epilogue warps' rows past
      // 256; V: the last PV commit and those rows
      mbar_init(k_free(i), g.extra ? 1u + 4u * (uint32_t)nt + 4u : 1u);
      mbar_init(v_full(i), 1);
      mbar_init(v_free(i), g.extra ? 5u : 1u);
      mbar_init(s_full(i), 1);
      mbar_init(p_full(i), 4);
      mbar_init(o_full(i), 1);
      mbar_init(o_free(i), 4);
      mbar_init(se_full(i), 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    if (g.extra) tma_prefetch(&tmT);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  fence_async_shared();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  if (warp == 0) {
    // ------------------------------------------------------------ TMA loads
    if (lane == 0) {
      bool ok = true;
      int i = 0;
      for (int j = 0; j < my_heads && ok; ++j) {
        const int head = (int)blockIdx.x + j * (int)gridDim.x;
        const int b = head / g.H, h = head - b * g.H, hb = j & 1;
        if (j >= 2 && (!mbar_wait(k_free(hb), (uint32_t)((j - 2) >> 1) & 1u, err, kDevErrTimeoutEmpty) ||
                       !mbar_wait(v_free(hb), (uint32_t)((j - 2) >> 1) & 1u, err, kDevErrTimeoutEmpty)))
          break;
        mbar_arrive_expect_tx(k_full(hb), g.kv_bytes + (g.extra ? 1024u : 0u));
        for (int x = 0; x < g.nbox; ++x) {
          const int row = x * g.box_rows;
          tma_load_4d(base + g.kb[hb] + (uint32_t)row * 128u, &tmK, 0, g.kv_hs ? h : row, g.kv_hs ? row : h, b,
                      k_full(hb));
        }
        if (g.extra)   // query rows 256.. (zero past S)
          tma_load_4d(base + g.qt[hb], &tmT, 0, g.kv_hs ? h : 256, g.kv_hs ? 256 : h, b, k_full(hb));
        mbar_arrive_expect_tx(v_full(hb), g.kv_bytes);
        for (int x = 0; x < g.nbox; ++x) {
          const int row = x * g.box_rows;
          tma_load_4d(base + g.vb[hb] + (uint32_t)row * 128u, &tmV, 0, g.kv_hs ? h : row, g.kv_hs ? row : h, b,
                      v_full(hb));
        }
        for (int t = 0; t < nt; ++t, ++i) {
          const int sl = i & 1;
          if (i >= 2 && !mbar_wait(q_free(sl), (uint32_t)((i - 2) >> 1) & 1u, err, kDevErrTimeoutEmpty)) {
            ok = false;
            break;
          }
          const int row = t * 128;
          mbar_arrive_expect_tx(q_full(sl), 128u * 128u);
          tma_load_4d(base + g.qb[sl], &tmQ, 0, g.kv_hs ? h : row, g.kv_hs ? row : h, b, q_full(sl));
        }
      }
      // no copy may still be writing shared memory when the CTA exits
      for (int x = i - 2 < 0 ? 0 : i - 2; x < i; ++x)
        mbar_wait(q_full(x & 1), (uint32_t)(x >> 1) & 1u, err, kDevErrTimeoutFull);
      for (int x = my_heads - 2 < 0 ? 0 : my_heads - 2; x < my_heads; ++x) {
        mbar_wait(k_full(x & 1), (uint32_t)(x >> 1) & 1u, err, kDevErrTimeoutFull);
        mbar_wait(v_full(x & 1), (uint32_t)(x >> 1) & 1u, err, kDevErrTimeoutFull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    bool ok = true;
    // S = Q K^T of tile i into slot i % 2, once the epilogue has read that slot's previous O
    auto issue_qk = [&](int i) {
      const int j = i / nt, t = i - j * nt, sl = i & 1, hb = j & 1;
      if (i >= 2 && !mbar_wait(o_free(sl), (uint32_t)((i - 2) >> 1) & 1u, err, kDevErrTimeoutEmpty)) return false;
      if (t == 0 && !mbar_wait(k_full(hb), (uint32_t)(j >> 1) & 1u, err, kDevErrTimeoutFull)) return false;
      if (!mbar_wait(q_full(sl), (uint32_t)(i >> 1) & 1u, err, kDevErrTimeoutFull)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t qa = base + g.qb[sl], ka = base + g.kb[hb];
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_f16(tmem + 256u * (uint32_t)sl, smem_desc(qa + 32u * kk, 16, 1024, 2), smem_desc(ka + 32u * kk, 16, 1024, 2),
                  idesc_bf16((uint32_t)g.skp, false), kk > 0 ? 1u : 0u);
        tc_commit(s_full(sl));
        tc_commit(q_free(sl));
        if (t == nt - 1) tc_commit(k_free(hb));
      }
      __syncwarp();
      return true;
    };
    if (T > 0) ok = issue_qk(0);
    if (ok && T > 1) ok = issue_qk(1);
    for (int i = 0; i < T && ok; ++i) {
      const int j = i / nt, t = i - j * nt, sl = i & 1, hb = j & 1;
      if (!mbar_wait(p_full(sl), (uint32_t)(i >> 1) & 1u, err, kDevErrTimeoutFull) ||
          (t == 0 && !mbar_wait(v_full(hb), (uint32_t)(j >> 1) & 1u, err, kDevErrTimeoutFull)))
        break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t slot = tmem + 256u * (uint32_t)sl, va = base + g.vb[hb];
        const int nk = g.skp / 16;
        for (int kk = 0; kk < nk; ++kk)
          mma_f16_tmem_a(slot + 128u, slot + 8u * (uint32_t)kk, smem_desc(va + 2048u * kk, 1024, 1024, 2),
                         idesc_bf16(64, true), kk > 0 ? 1u : 0u);
        if (g.extra)
          mma_f16(slot + 128u, smem_desc(base + g.pe[sl], 128, 256, 0), smem_desc(va + 2048u * 16u, 1024, 1024, 2),
                  idesc_bf16(64, true), 1u);
        tc_commit(o_full(sl));
        if (t == nt - 1) tc_commit(v_free(hb));
      }
      __syncwarp();
      if (i + 2 < T) ok = issue_qk(i + 2);
    }
    if (lane == 0) {
      tc_commit(drain);
      mbar_wait(drain, 0, err, kDevErrTimeoutDrain);
    }
    __syncwarp();
  } else if (warp >= kB16sSoftW && warp < kB16sSoftW + 8) {
    // ------------------------------------------------------------ softmax, one slot per warp group
    const int sl = (warp - kB16sSoftW) >> 2, qd = warp & 3, r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    const uint32_t srow = tmem + lane_base + 256u * (uint32_t)sl;
    float* red_l = reinterpret_cast<float*>(gb + g.red) + sl * 128;
    const float c = g.scale * 1.4426950408889634f;
    const int keys = S < 256 ? S : 256;   // keys scored by the MMA
    const int nchunk = g.skp / 16;
    bool ok = true;
    for (int i = sl; i < T; i += 2) {
      const int t = i - i / nt * nt;
      const bool wact = t * 128 + qd * 32 < S;   // any query row of this warp's quadrant valid
      if (ok) ok = mbar_wait(s_full(sl), (uint32_t)(i >> 1) & 1u, err, kDevErrTimeoutFull);
      tc_fence_after();
      float se[kB16sExtraMax];
#pragma unroll
      for (int e = 0; e < kB16sExtraMax; ++e) se[e] = -INFINITY;
      float lsum = 0.f;
      if (ok && wact) {
        // pass 1: row max over the valid keys
        float m = -INFINITY;
        auto max16 = [&](int u, const uint32_t* v) {
          if (16 * u + 16 <= keys) {
#pragma unroll
            for (int x = 0; x < 16; x += 2) m = max3f(m, __uint_as_float(v[x]), __uint_as_float(v[x + 1]));
          } else {
#pragma unroll
            for (int x = 0; x < 16; ++x)
              if (16 * u + x < keys) m = fmaxf(m, __uint_as_float(v[x]));
          }
        };
        {
          uint32_t va[16], vb[16];
          tmem_ld_32x32b_x16(srow, va);
          tmem_wait_ld();
          reg_fence16(va);
          for (int u = 0; u < nchunk; u += 2) {
            if (u + 1 < nchunk) tmem_ld_32x32b_x16(srow + 16 * (u + 1), vb);
            max16(u, va);
            tmem_wait_ld();
            reg_fence16(vb);
            if (u + 1 < nchunk) {
              if (u + 2 < nchunk) tmem_ld_32x32b_x16(srow + 16 * (u + 2), va);
              max16(u + 1, vb);
              tmem_wait_ld();
              reg_fence16(va);
            }
          }
        }
        if (g.extra) {   // the keys past 256, scored by the epilogue warps
          ok = mbar_wait(se_full(sl), (uint32_t)(i >> 1) & 1u, err, kDevErrTimeoutFull);
          const float* ser = reinterpret_cast<const float*>(gb + g.se) + (sl * 128 + r) * kB16sExtraMax;
#pragma unroll
          for (int e = 0; e < kB16sExtraMax; ++e) {
            if (e < g.extra) {
              se[e] = ser[e];
              m = fmaxf(m, se[e]);
            }
          }
        }
        // pass 2: P = 2^((s - max) c) -> bf16 pairs over the slot's first 128 columns (chunk u's
        // pairs land in columns 8u..8u+7, scores this thread has already read), row sums in fp32
        const float nmc = -m * c;
        const unsigned long long c2 = f32x2_pack(c, c), nmc2 = f32x2_pack(nmc, nmc);
        unsigned long long lsum2 = f32x2_pack(0.f, 0.f);
        auto exp16 = [&](int u, const uint32_t* v) {
          float p[16];
#pragma unroll
          for (int x = 0; x < 8; ++x) {
            float x0, x1;
            f32x2_unpack(fma_f32x2(f32x2_pack(__uint_as_float(v[2 * x]), __uint_as_float(v[2 * x + 1])), c2, nmc2), &x0,
                         &x1);
            p[2 * x] = ex2_approx(x0);
            p[2 * x + 1] = ex2_approx(x1);
          }
          if (16 * u + 16 > keys) {
#pragma unroll
            for (int x = 0; x < 16; ++x)
              if (16 * u + x >= keys) p[x] = 0.f;
          }
          uint32_t w[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) {
            lsum2 = add_f32x2(lsum2, f32x2_pack(p[2 * x], p[2 * x + 1]));
            __nv_bfloat162 pv = __floats2bfloat162_rn(p[2 * x], p[2 * x + 1]);
            w[x] = *reinterpret_cast<uint32_t*>(&pv);
          }
          tmem_st_32x32b_x8(srow + 8 * u, w);
        };
        {
          uint32_t va[16], vb[16];
          tmem_ld_32x32b_x16(srow, va);
          tmem_wait_ld();
          reg_fence16(va);
          for (int u = 0; u < nchunk; u += 2) {
            if (u + 1 < nchunk) tmem_ld_32x32b_x16(srow + 16 * (u + 1), vb);
            exp16(u, va);
            tmem_wait_ld();
            reg_fence16(vb);
            if (u + 1 < nchunk) {
              if (u + 2 < nchunk) tmem_ld_32x32b_x16(srow + 16 * (u + 2), va);
              exp16(u + 1, vb);
              tmem_wait_ld();
              reg_fence16(va);
            }
          }
        }
        float l0, l1;
        f32x2_unpack(lsum2, &l0, &l1);
        lsum = l0 + l1;
        if (g.extra) {
          // the extra keys' P row (zero past S) as the A operand of one more K = 16 step:
          // K-major core matrices, 8-row groups 256 bytes apart, the two 8-key halves 128 bytes apart
          uint32_t w[8];
#pragma unroll
          for (int x = 0; x < 8; ++x) w[x] = 0u;
#pragma unroll
          for (int e = 0; e < kB16sExtraMax; ++e) {
            if (e < g.extra) {
              const float pe = ex2_approx(fmaf(se[e], c, nmc));
              lsum += pe;
              const uint32_t hbits = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(pe));
              w[e >> 1] |= (e & 1) ? hbits << 16 : hbits;
            }
          }
          uint8_t* prow = gb + g.pe[sl] + (uint32_t)(r >> 3) * 256u + (uint32_t)(r & 7) * 16u;
          *reinterpret_cast<uint4*>(prow) = make_uint4(w[0], w[1], w[2], w[3]);
          *reinterpret_cast<uint4*>(prow + 128) = make_uint4(w[4], w[5], w[6], w[7]);
        }
        tmem_wait_st();
      }
      red_l[r] = lsum;
      fence_async_shared();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full(sl));
    }
  } else if (warp >= kB16sEpiW && warp < kB16sEpiW + 4) {
    // ------------------------------------------------------------ epilogue: O / rowsum -> bf16
    const int qd = warp & 3, r = qd * 32 + lane;
    const uint32_t lane_base = (uint32_t)(qd * 32) << 16;
    // max |out| as bf16 magnitude bits in two 16-bit lanes: unsigned order of non-negative bf16
    // bits is numeric order and a NaN (0x7FC0) sorts above +inf, so a NaN output reaches the amax
    // as torch's amax would give it
    uint32_t out_max2 = 0;
    bool ok = true;
    // the scores of the keys past 256 for the rows of tile i (s_e = q_r . k_(256 + e) in fp32), handed
    // to the softmax warps through shared memory once the tile's Q and the head's K are in; this
    // warp's Q and extra-K reads then count towards releasing those buffers
    auto extra_scores = [&](int i) {
      const int j = i / nt, sl = i & 1, hb = j & 1;
      if (ok) ok = mbar_wait(q_full(sl), (uint32_t)(i >> 1) & 1u, err, kDevErrTimeoutFull) &&
                   mbar_wait(k_full(hb), (uint32_t)(j >> 1) & 1u, err, kDevErrTimeoutFull);
      float* ser = reinterpret_cast<float*>(gb + g.se) + (sl * 128 + r) * kB16sExtraMax;
      if (ok) {
        const uint8_t* qt = gb + g.qb[sl] + r * 128;
#pragma unroll
        for (int e = 0; e < kB16sExtraMax; ++e) {
          if (e < g.extra) {
            const int key = 256 + e;
            const uint8_t* kt = gb + g.kb[hb] + key * 128;
            unsigned long long acc0 = f32x2_pack(0.f, 0.f), acc1 = acc0;
#pragma unroll
            for (int x = 0; x < 8; ++x) {
              const uint4 a = *reinterpret_cast<const uint4*>(qt + ((x ^ (r & 7)) << 4));
              const uint4 w = *reinterpret_cast<const uint4*>(kt + ((x ^ (key & 7)) << 4));
              acc0 = fma_f32x2(bf16x2_to_f32x2(w.x), bf16x2_to_f32x2(a.x), acc0);
              acc1 = fma_f32x2(bf16x2_to_f32x2(w.y), bf16x2_to_f32x2(a.y), acc1);
              acc0 = fma_f32x2(bf16x2_to_f32x2(w.z), bf16x2_to_f32x2(a.z), acc0);
              acc1 = fma_f32x2(bf16x2_to_f32x2(w.w), bf16x2_to_f32x2(a.w), acc1);
            }
            float a0, a1, b0, b1;
            f32x2_unpack(acc0, &a0, &a1);
            f32x2_unpack(acc1, &b0, &b1);
            ser[e] = (a0 + a1) + (b0 + b1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(se_full(sl));
        mbar_arrive(q_free(sl));
        mbar_arrive(k_free(hb));
      }
    };
    if (g.extra) {
      if (T > 0) extra_scores(0);
      if (T > 1) extra_scores(1);
    }
    for (int i = 0; i < T; ++i) {
      const int j = i / nt, t = i - j * nt, sl = i & 1;
      const int head = (int)blockIdx.x + j * (int)gridDim.x;
      const int b = head / g.H, h = head - b * g.H, row = t * 128 + r;
      const bool wact = t * 128 + qd * 32 < S;
      if (ok) ok = mbar_wait(o_full(sl), (uint32_t)(i >> 1) & 1u, err, kDevErrTimeoutTmem) &&
                   mbar_wait(p_full(sl), (uint32_t)(i >> 1) & 1u, err, kDevErrTimeoutTmem);
      tc_fence_after();
      uint32_t ov[64];
      if (ok && wact) {
        const uint32_t ta = tmem + lane_base + 256u * (uint32_t)sl + 128u;
        tmem_ld_32x32b_x32(ta, ov);
        tmem_ld_32x32b_x32(ta + 32, ov + 32);
        tmem_wait_ld();
      }
      const float lsum = reinterpret_cast<const float*>(gb + g.red)[sl * 128 + r];
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free(sl));
      if (ok && wact && row < S) {
        const float f = 1.0f / lsum;
        __nv_bfloat16* orow = g.out + (int64_t)b * g.osb + (int64_t)h * g.osh + (int64_t)row * g.oss;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t w[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            __nv_bfloat162 hv = __floats2bfloat162_rn(__uint_as_float(ov[8 * cc + 2 * x]) * f,
                                                      __uint_as_float(ov[8 * cc + 2 * x + 1]) * f);
            w[x] = *reinterpret_cast<uint32_t*>(&hv);
            out_max2 = umax_u16x2(out_max2, w[x] & 0x7FFF7FFFu);
          }
          *reinterpret_cast<uint4*>(orow + 8 * cc) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
      if (g.extra && i + 2 < T) extra_scores(i + 2);
    }
    if (g.amax) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, max(out_max2 & 0xFFFFu, out_max2 >> 16) << 16);
      if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(g.amax), m);
    }
  } else if (warp >= kB16sTailW && g.extra) {
    // ------------------------------------------------------------ query rows 256 .. S - 1 of every
    // head on the CUDA cores, from the head's K (with those rows) and V in shared memory; each tail
    // warp takes every barrier below, whatever its wait results
    const int et = threadIdx.x - kB16sTailW * 32, ew = et >> 5;
    uint32_t out_max2 = 0;
    bool ok = true;
    for (int j = 0; j < my_heads; ++j) {
      const int head = (int)blockIdx.x + j * (int)gridDim.x;
      const int b = head / g.H, h = head - b * g.H;
      {
        const int hb = j & 1, ne = g.extra;
        float* tp = reinterpret_cast<float*>(gb + g.tw);   // probabilities, rounded to bf16 [2][272]
        float* to = tp + 2 * 272;                          // partial outputs [key group][2][64]
        float* tr = to + 16 * 2 * 64;                      // per-warp [2 rows][max, sum]
        if (ok) ok = mbar_wait(k_full(hb), (uint32_t)(j >> 1) & 1u, err, kDevErrTimeoutFull) &&
                     mbar_wait(v_full(hb), (uint32_t)(j >> 1) & 1u, err, kDevErrTimeoutFull);
        // scores of keys et, et + 128, et + 256 (< S), one row at a time with the row's q in registers
        float sc[3][kB16sExtraMax], mloc[kB16sExtraMax];
#pragma unroll
        for (int e = 0; e < kB16sExtraMax; ++e) {
          mloc[e] = -INFINITY;
#pragma unroll
          for (int x = 0; x < 3; ++x) sc[x][e] = -INFINITY;
          if (ok && e < ne) {
            unsigned long long q2[32];
            const uint8_t* qrow = gb + g.qt[hb] + e * 128;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
              const uint4 a = *reinterpret_cast<const uint4*>(qrow + ((cc ^ e) << 4));
              q2[4 * cc] = bf16x2_to_f32x2(a.x);
              q2[4 * cc + 1] = bf16x2_to_f32x2(a.y);
              q2[4 * cc + 2] = bf16x2_to_f32x2(a.z);
              q2[4 * cc + 3] = bf16x2_to_f32x2(a.w);
            }
#pragma unroll
            for (int x = 0; x < 3; ++x) {
              const int key = et + 128 * x;
              if (key < S) {
                const uint8_t* kr = gb + g.kb[hb] + key * 128;
                unsigned long long a0 = f32x2_pack(0.f, 0.f), a1 = a0;
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                  const uint4 w = *reinterpret_cast<const uint4*>(kr + ((cc ^ (key & 7)) << 4));
                  a0 = fma_f32x2(bf16x2_to_f32x2(w.x), q2[4 * cc], a0);
                  a1 = fma_f32x2(bf16x2_to_f32x2(w.y), q2[4 * cc + 1], a1);
                  a0 = fma_f32x2(bf16x2_to_f32x2(w.z), q2[4 * cc + 2], a0);
                  a1 = fma_f32x2(bf16x2_to_f32x2(w.w), q2[4 * cc + 3], a1);
                }
                float b0, b1, b2, b3;
                f32x2_unpack(a0, &b0, &b1);
                f32x2_unpack(a1, &b2, &b3);
                sc[x][e] = (b0 + b1) + (b2 + b3);
                mloc[e] = fmaxf(mloc[e], sc[x][e]);
              }
            }
          }
        }
#pragma unroll
        for (int e = 0; e < kB16sExtraMax; ++e) {
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) mloc[e] = fmaxf(mloc[e], __shfl_xor_sync(0xffffffffu, mloc[e], o));
          if (lane == 0) tr[(ew * 2 + e) * 2] = mloc[e];
        }
        named_bar_sync(kB16sBarTail, 128);
        const float c = g.scale * 1.4426950408889634f;
        float lloc[kB16sExtraMax];
#pragma unroll
        for (int e = 0; e < kB16sExtraMax; ++e) {
          const float mx = fmaxf(fmaxf(tr[(0 * 2 + e) * 2], tr[(1 * 2 + e) * 2]), fmaxf(tr[(2 * 2 + e) * 2], tr[(3 * 2 + e) * 2]));
          const float nmc = -mx * c;
          lloc[e] = 0.f;
#pragma unroll
          for (int x = 0; x < 3; ++x) {
            const int key = et + 128 * x;
            if (e < ne && key < S) {
              const float pv = ex2_approx(fmaf(sc[x][e], c, nmc));
              tp[e * 272 + key] = bf16_round(pv);   // the weight PV applies; the sum takes the fp32 value
              lloc[e] += pv;
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) lloc[e] += __shfl_xor_sync(0xffffffffu, lloc[e], o);
        }
        named_bar_sync(kB16sBarTail, 128);   // the maxima are read; the sums reuse their neighbours
#pragma unroll
        for (int e = 0; e < kB16sExtraMax; ++e)
          if (lane == 0) tr[(ew * 2 + e) * 2 + 1] = lloc[e];
        {
          // O partials: dims 8 dg .. 8 dg + 7 (one 16-byte piece of each V row) over the keys
          // kg, kg + 16, ..., with P rounded to bf16 as the MMA sees it
          const int dg = et & 7, kg = et >> 3;
          unsigned long long acc[kB16sExtraMax][4];
#pragma unroll
          for (int e = 0; e < kB16sExtraMax; ++e)
#pragma unroll
            for (int x = 0; x < 4; ++x) acc[e][x] = f32x2_pack(0.f, 0.f);
          if (ok) {
#pragma unroll 2
            for (int key = kg; key < S; key += 16) {
              const uint4 vv = *reinterpret_cast<const uint4*>(gb + g.vb[hb] + key * 128 + ((dg ^ (key & 7)) << 4));
              const unsigned long long v0 = bf16x2_to_f32x2(vv.x), v1 = bf16x2_to_f32x2(vv.y),
                                       v2 = bf16x2_to_f32x2(vv.z), v3 = bf16x2_to_f32x2(vv.w);
#pragma unroll
              for (int e = 0; e < kB16sExtraMax; ++e) {
                if (e < ne) {
                  const float pb = tp[e * 272 + key];
                  const unsigned long long p2 = f32x2_pack(pb, pb);
                  acc[e][0] = fma_f32x2(v0, p2, acc[e][0]);
                  acc[e][1] = fma_f32x2(v1, p2, acc[e][1]);
                  acc[e][2] = fma_f32x2(v2, p2, acc[e][2]);
                  acc[e][3] = fma_f32x2(v3, p2, acc[e][3]);
                }
              }
            }
          }
#pragma unroll
          for (int e = 0; e < kB16sExtraMax; ++e) {
            if (e < ne) {
              float4* dst = reinterpret_cast<float4*>(to + (kg * 2 + e) * 64 + 8 * dg);
              float o[8];
#pragma unroll
              for (int x = 0; x < 4; ++x) f32x2_unpack(acc[e][x], &o[2 * x], &o[2 * x + 1]);
              dst[0] = make_float4(o[0], o[1], o[2], o[3]);
              dst[1] = make_float4(o[4], o[5], o[6], o[7]);
            }
          }
        }
        named_bar_sync(kB16sBarTail, 128);
        if (ok && et < ne * 64) {
          const int e = et >> 6, d = et & 63;
          const float l = (tr[(0 * 2 + e) * 2 + 1] + tr[(1 * 2 + e) * 2 + 1]) + (tr[(2 * 2 + e) * 2 + 1] + tr[(3 * 2 + e) * 2 + 1]);
          float o = 0.f;
#pragma unroll
          for (int kg = 0; kg < 16; ++kg) o += to[(kg * 2 + e) * 64 + d];
          const __nv_bfloat16 ob = __float2bfloat16_rn(o * (1.0f / l));
          g.out[(int64_t)b * g.osb + (int64_t)h * g.osh + (int64_t)(256 + e) * g.oss + d] = ob;
          out_max2 = umax_u16x2(out_max2, (uint32_t)(__bfloat16_as_ushort(ob) & 0x7FFFu));
        }
        named_bar_sync(kB16sBarTail, 128);   // the working storage is written again at the next head
        if (lane == 0) {   // this warp is done with the head's K (and its rows past 256) and V
          mbar_arrive(k_free(hb));
          mbar_arrive(v_free(hb));
        }
      }
    }
    if (g.amax) {
      const uint32_t m = __reduce_max_sync(0xffffffffu, out_max2 << 16);
      if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(g.amax), m);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

static int launch_bf16_slots(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                             int64_t sb, int64_t sh, int64_t ss, float scale, void* out, int64_t osb, int64_t osh,
                             int64_t oss, float* amax, cudaStream_t s) {
  B16sGeom g = make_b16s_geom(B, H, S, D, scale);
  g.amax = amax;
  if (amax && cudaMemsetAsync(amax, 0, sizeof(float), s) != cudaSuccess)
    return fail(VF4_ERR_CUDA, "vf4_attn_bf16: amax reset failed");
  g.out = static_cast<__nv_bfloat16*>(out);
  g.osb = osb;
  g.osh = osh;
  g.oss = oss;
  g.kv_hs = sh < ss;
  FusedGeom fg = make_fused_geom(B, H, S, D, scale);   // the head-view maps take D, S, H, B from it
  CUtensorMap tq, tk, tv, tt;
  memset(&tt, 0, sizeof(tt));
  if (int st = make_head_map(&tq, q, fg, sb, sh, ss, 128, g.kv_hs)) return st;
  if (int st = make_head_map(&tk, k, fg, sb, sh, ss, g.box_rows, g.kv_hs)) return st;
  if (int st = make_head_map(&tv, v, fg, sb, sh, ss, g.box_rows, g.kv_hs)) return st;
  if (g.extra) {
    if (int st = make_head_map(&tt, q, fg, sb, sh, ss, 8, g.kv_hs)) return st;
  }
  if (int st = smem_optin(attn_bf16_slots_kernel, (int)g.total)) return st;
  const int grid = g.heads < num_sms() ? g.heads : num_sms();
  attn_bf16_slots_kernel<<<grid, kB16sWarps * 32, g.total, s>>>(tq, tk, tv, tt, g);
  return launch_status("vf4_attn_bf16");
}

static int make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t rowbytes, int box_x, int box_y,
                    CUtensorMapSwizzle swz) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)rowbytes, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)rowbytes};
  cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
  cuuint32_t es[2] = {1u, 1u};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(VF4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return VF4_OK;
}

template <int DP>
static int launch_fwd(const AttnGeom& g, const uint8_t* ws, float scale, void* out, int64_t osb, int64_t osh,
                      int64_t oss, cudaStream_t s) {
  using C = AttnCfg<DP>;
  AttnSmem L = attn_smem_layout<DP>(g.nc, g.S_pad);
  if (L.total > 227 * 1024)
    return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_nvfp4: sequence %d too long for head dim %d", g.S, g.D);
  CUtensorMap tq, tk, tv;
  const CUtensorMapSwizzle qs = DP == 64 ? CU_TENSOR_MAP_SWIZZLE_32B : CU_TENSOR_MAP_SWIZZLE_64B;
  if (int st = make_map(&tq, ws + g.off_q, g.BH * g.S_pad, C::ROWB, C::ROWB, 128, qs)) return st;
  if (int st = make_map(&tk, ws + g.off_k, g.BH * g.S_pad, C::ROWB, C::ROWB, 128, qs)) return st;
  if (int st = make_map(&tv, ws + g.off_v, g.BH * C::DV, g.S_pad / 2, 64, C::DV, CU_TENSOR_MAP_SWIZZLE_64B))
    return st;
  auto kern = attn_fwd_kernel<DP>;
  if (int st = smem_optin(kern, (int)L.total)) return st;
  const int grid = (int)(g.BH < num_sms() ? g.BH : num_sms());   // persistent: whole heads per CTA
  kern<<<grid, C::THREADS, L.total, s>>>(tq, tk, tv, g, ws, L, scale, static_cast<__nv_bfloat16*>(out), osb, osh,
                                         oss);
  return launch_status("vf4_attn_nvfp4 (forward)");
}

// Workspace of one call: [global maxima (256 B)][per-head means][long-sequence path buffers].
// The first two exist only with tensor-wide globals; the last only off the fused path.
struct AttnWs {
  int64_t off_amax, off_stats, off_gen, off_img, total;
};

// packed: the packed fused route's per-head operand images follow (B*H images of img_bytes)
static AttnWs attn_ws_layout(int64_t B, int64_t H, int64_t S, int64_t D, bool tensor, bool packed = false) {
  AttnWs w{};
  const int64_t Dp = D <= 64 ? 64 : 128;
  int64_t o = 0;
  w.off_amax = 0;
  if (tensor) o = 256;
  w.off_stats = o;
  if (tensor) o = align_up(o + B * H * 2 * Dp * 4, 1024);
  w.off_gen = o;
  if (!fused_ok(S, D)) o += make_geom(B, H, S, D).total;
  w.off_img = o;
  if (packed && packed_ok(S, D)) {
    w.off_img = align_up(o, 1024);
    o = w.off_img + B * H * (int64_t)make_fused_geom(1, 1, S, D, 1.f, true).img_bytes;
  }
  w.total = o;
  return w;
}

}  // namespace vf4

using namespace vf4;

extern "C" {

int64_t vf4_attn_workspace_size(int64_t B, int64_t H, int64_t S, int64_t D) {
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0 || D % 16 != 0 || D > 128) return 0;
  return attn_ws_layout(B, H, S, D, true).total;
}

static constexpr int kAttnFlags = VF4_ATTN_HEAD_GLOBALS | VF4_ATTN_PACKED | VF4_ATTN_NO_SMOOTH_K | VF4_ATTN_NO_SMOOTH_V;

int64_t vf4_attn_workspace_size_ex(int64_t B, int64_t H, int64_t S, int64_t D, int flags) {
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0 || D % 16 != 0 || D > 128) return 0;
  if (flags & ~kAttnFlags) return 0;
  return attn_ws_layout(B, H, S, D, !(flags & VF4_ATTN_HEAD_GLOBALS), (flags & VF4_ATTN_PACKED) != 0).total;
}

int vf4_attn_nvfp4_ex(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                      int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, void* out,
                      int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s, int flags, void* workspace,
                      int64_t workspace_bytes, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(VF4_ERR_ARG, "vf4_attn_nvfp4: bad sizes");
  if (D % 16 != 0 || D > 128) return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_nvfp4: head dim must be a multiple of 16, <= 128");
  if (flags & ~kAttnFlags) return fail(VF4_ERR_ARG, "vf4_attn_nvfp4: unknown flags %d", flags);
  const int smooth = ((flags & VF4_ATTN_NO_SMOOTH_K) ? 0 : 1) | ((flags & VF4_ATTN_NO_SMOOTH_V) ? 0 : 2);
  if (smooth != 3 && (flags & VF4_ATTN_HEAD_GLOBALS))
    return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_nvfp4: smooth-K / smooth-V can be switched off only with the "
                                     "tensor-wide global scales (no VF4_ATTN_HEAD_GLOBALS)");
  if (!q || !k || !v || !out) return fail(VF4_ERR_ARG, "vf4_attn_nvfp4: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      stride_b % 8 || stride_h % 8 || stride_s % 8 || out_stride_b % 8 || out_stride_h % 8 || out_stride_s % 8)
    return fail(VF4_ERR_ALIGN, "vf4_attn_nvfp4: 16-byte aligned pointers and strides (multiples of 8) needed");
  if (B * H > INT32_MAX) return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_nvfp4: B*H too large");
  const bool tensor = !(flags & VF4_ATTN_HEAD_GLOBALS);
  const bool fused = fused_ok(S, D);
  // the fused kernel takes the row max of the raw scores, which is the softmax's max only for scale >= 0
  if (fused && !(scale >= 0.f))
    return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_nvfp4: head dim 64 and S <= 320 need a scale >= 0 (got %g)",
                (double)scale);
  if (!fused && B * H > 65535) return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_nvfp4: B*H must be <= 65535 for S=%lld D=%lld",
                                           (long long)S, (long long)D);
  const bool packed = (flags & VF4_ATTN_PACKED) && packed_ok(S, D);
  const AttnWs w = attn_ws_layout(B, H, S, D, tensor, packed);
  if (w.total > 0 && (!workspace || !aligned16(workspace)))
    return fail(VF4_ERR_ARG, "vf4_attn_nvfp4: a 16-byte aligned workspace of %lld bytes is needed", (long long)w.total);
  if (workspace_bytes < w.total)
    return fail(VF4_ERR_ARG, "vf4_attn_nvfp4: workspace %lld < %lld bytes", (long long)workspace_bytes,
                (long long)w.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const auto* Q = static_cast<const __nv_bfloat16*>(q);
  const auto* K = static_cast<const __nv_bfloat16*>(k);
  const auto* V = static_cast<const __nv_bfloat16*>(v);
  float* stats = nullptr;
  float* amax3 = nullptr;
  if (tensor) {
    stats = reinterpret_cast<float*>(ws + w.off_stats);
    amax3 = reinterpret_cast<float*>(ws + w.off_amax);
    if (cudaMemsetAsync(amax3, 0, 16, s) != cudaSuccess) return fail(VF4_ERR_CUDA, "vf4_attn_nvfp4: memset failed");
    if (D == 64) {
      attn_stats64_kernel<<<(unsigned)(B * H), 256, 0, s>>>(Q, K, V, stride_b, stride_h, stride_s, (int)H, (int)S,
                                                            smooth, stats, amax3);
    } else {
      const int D8 = (int)D / 8, rpi = 256 / D8;
      const int smem = 32 % D8 == 0 ? 8 * 6 * (int)D * 4 : 6 * rpi * (int)D * 4;
      if (int st = smem_optin(attn_stats_kernel, smem)) return st;
      attn_stats_kernel<<<(unsigned)(B * H), 256, smem, s>>>(Q, K, V, stride_b, stride_h, stride_s, (int)H, (int)S,
                                                             (int)D, D <= 64 ? 64 : 128, smooth, stats, amax3);
    }
    if (int st = launch_status("vf4_attn_nvfp4 (statistics)")) return st;
  }
  if (fused)
    return launch_fused(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b, out_stride_h,
                        out_stride_s, stats, amax3, s, packed ? ws + w.off_img : nullptr);
  AttnGeom g = make_geom(B, H, S, D);
  uint8_t* gws = ws + w.off_gen;
  attn_prep_kernel<<<(unsigned)g.BH, 256, 0, s>>>(Q, K, V, stride_b, stride_h, stride_s, g, gws, stats, amax3);
  if (int st = launch_status("vf4_attn_nvfp4 (prep)")) return st;
  if (g.Dp == 64) return launch_fwd<64>(g, gws, scale, out, out_stride_b, out_stride_h, out_stride_s, s);
  return launch_fwd<128>(g, gws, scale, out, out_stride_b, out_stride_h, out_stride_s, s);
}

int vf4_attn_fp8(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                 int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, void* out, int64_t out_stride_b,
                 int64_t out_stride_h, int64_t out_stride_s, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(VF4_ERR_ARG, "vf4_attn_fp8: bad sizes");
  if (!fp8_ok(S, D)) return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_fp8: needs head dim 64 and S <= 320 (S=%lld D=%lld)",
                                 (long long)S, (long long)D);
  if (!q || !k || !v || !out) return fail(VF4_ERR_ARG, "vf4_attn_fp8: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      stride_b % 8 || stride_h % 8 || stride_s % 8 || out_stride_b % 8 || out_stride_h % 8 || out_stride_s % 8)
    return fail(VF4_ERR_ALIGN, "vf4_attn_fp8: 16-byte aligned pointers and strides (multiples of 8) needed");
  if (B * H > INT32_MAX) return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_fp8: B*H too large");
  return launch_fp8(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b, out_stride_h,
                    out_stride_s, 3, reinterpret_cast<cudaStream_t>(stream));
}

int vf4_attn_bf16(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                  int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, void* out, int64_t out_stride_b,
                  int64_t out_stride_h, int64_t out_stride_s, float* out_amax, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(VF4_ERR_ARG, "vf4_attn_bf16: bad sizes");
  if (!bf16_attn_ok(S, D))
    return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_bf16: needs head dim 64 and S <= 288 (S=%lld D=%lld)", (long long)S,
                (long long)D);
  if (!(scale >= 0.f))   // the row max of the raw scores is the softmax's max only for scale >= 0
    return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_bf16: needs a scale >= 0 (got %g)", (double)scale);
  if (!q || !k || !v || !out) return fail(VF4_ERR_ARG, "vf4_attn_bf16: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) ||
      stride_b % 8 || stride_h % 8 || stride_s % 8 || out_stride_b % 8 || out_stride_h % 8 || out_stride_s % 8)
    return fail(VF4_ERR_ALIGN, "vf4_attn_bf16: 16-byte aligned pointers and strides (multiples of 8) needed");
  if (B * H > INT32_MAX) return fail(VF4_ERR_UNSUPPORTED, "vf4_attn_bf16: B*H too large");
  if (out_amax && (reinterpret_cast<uintptr_t>(out_amax) & 3u))
    return fail(VF4_ERR_ALIGN, "vf4_attn_bf16: out_amax must be 4-byte aligned");
  // the two-slot kernel up to S = 258, the single-slot one past that; VF4_BF16_ATTN=tiles selects the
  // single-slot kernel for every S
  const char* mode = getenv("VF4_BF16_ATTN");
  if (b16s_ok(S, D) && !(mode && mode[0] == 't'))
    return launch_bf16_slots(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b,
                             out_stride_h, out_stride_s, out_amax, reinterpret_cast<cudaStream_t>(stream));
  return launch_bf16(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b, out_stride_h,
                     out_stride_s, out_amax, reinterpret_cast<cudaStream_t>(stream));
}

int vf4_attn_nvfp4(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                   int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, void* out,
                   int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s, void* workspace,
                   int64_t workspace_bytes, vf4_stream_t stream) {
  return vf4_attn_nvfp4_ex(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b, out_stride_h,
                           out_stride_s, 0, workspace, workspace_bytes, stream);
}

int64_t vf4_attn_workspace_size_modes(int64_t B, int64_t H, int64_t S, int64_t D, int qk_mode, int pv_mode,
                                      int flags) {
  if (qk_mode == VF4_ATTN_MODE_NVFP4 && pv_mode == VF4_ATTN_MODE_NVFP4)
    return vf4_attn_workspace_size_ex(B, H, S, D, flags);
  if (qk_mode == VF4_ATTN_MODE_FP8 && pv_mode == VF4_ATTN_MODE_FP8) {
    if (B <= 0 || H <= 0 || (flags & ~(VF4_ATTN_NO_SMOOTH_K | VF4_ATTN_NO_SMOOTH_V))) return 0;
    if (fp8_ok(S, D) || !f8l_ok(S, D)) return 0;   // the short kernel needs none; unsupported shapes fail
    return make_f8l_geom(B, H, S, D).total;
  }
  return 0;
}

int vf4_attn(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
             int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, int qk_mode, int pv_mode, int flags,
             void* workspace, int64_t workspace_bytes, void* out, int64_t out_stride_b, int64_t out_stride_h,
             int64_t out_stride_s, vf4_stream_t stream) {
  const bool nvfp4 = qk_mode == VF4_ATTN_MODE_NVFP4 && pv_mode == VF4_ATTN_MODE_NVFP4;
  const bool fp8 = qk_mode == VF4_ATTN_MODE_FP8 && pv_mode == VF4_ATTN_MODE_FP8;
  const bool bf16 = qk_mode == VF4_ATTN_MODE_BF16 && pv_mode == VF4_ATTN_MODE_BF16;
  if (nvfp4)
    return vf4_attn_nvfp4_ex(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b,
                             out_stride_h, out_stride_s, flags, workspace, workspace_bytes, stream);
  if (fp8) {
    if (flags & ~(VF4_ATTN_NO_SMOOTH_K | VF4_ATTN_NO_SMOOTH_V))
      return fail(VF4_ERR_ARG, "vf4_attn: flags %d do not apply to the FP8 route", flags);
    if (int st = check_device()) return st;
    if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(VF4_ERR_ARG, "vf4_attn: bad sizes");
    const bool short_route = fp8_ok(S, D);
    if (!short_route && !f8l_ok(S, D))
      return fail(VF4_ERR_UNSUPPORTED, "vf4_attn: FP8 attention needs a head dim that is a multiple of 16 and <= 128, "
                  "and a sequence whose keys fit shared memory (S=%lld D=%lld)", (long long)S, (long long)D);
    if (!q || !k || !v || !out) return fail(VF4_ERR_ARG, "vf4_attn: null pointer");
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || stride_b % 8 || stride_h % 8 ||
        stride_s % 8 || out_stride_b % 8 || out_stride_h % 8 || out_stride_s % 8)
      return fail(VF4_ERR_ALIGN, "vf4_attn: 16-byte aligned pointers and strides (multiples of 8) needed");
    if (B * H > INT32_MAX) return fail(VF4_ERR_UNSUPPORTED, "vf4_attn: B*H too large");
    const int smooth = ((flags & VF4_ATTN_NO_SMOOTH_K) ? 0 : 1) | ((flags & VF4_ATTN_NO_SMOOTH_V) ? 0 : 2);
    if (short_route)
      return launch_fp8(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b, out_stride_h,
                        out_stride_s, smooth, reinterpret_cast<cudaStream_t>(stream));
    const int64_t need = make_f8l_geom(B, H, S, D).total;
    if (!workspace || !aligned16(workspace) || workspace_bytes < need)
      return fail(VF4_ERR_ARG, "vf4_attn: the long-sequence FP8 route needs a 16-byte aligned workspace of %lld bytes "
                  "(got %lld)", (long long)need, (long long)workspace_bytes);
    return launch_fp8_long(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b, out_stride_h,
                           out_stride_s, smooth, static_cast<uint8_t*>(workspace),
                           reinterpret_cast<cudaStream_t>(stream));
  }
  if (bf16) {   // smoothing is exact under the softmax and the PV product: the flags change no result
    if (flags & ~(VF4_ATTN_NO_SMOOTH_K | VF4_ATTN_NO_SMOOTH_V))
      return fail(VF4_ERR_ARG, "vf4_attn: flags %d do not apply to the bf16 route", flags);
    return vf4_attn_bf16(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b, out_stride_h,
                         out_stride_s, nullptr, stream);
  }
  return fail(VF4_ERR_UNSUPPORTED, "vf4_attn: qk_mode %d / pv_mode %d is not a kernel route (the mixed routes run "
              "the reference's emulation on the host side)", qk_mode, pv_mode);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot call cudaMalloc at all: a host runtime that has handed the whole device
// to its own memory pool, or a plugin loaded into an inference server that forbids library
// allocations (and the implicit device synchronisation cudaMalloc/cudaFree can cause) while
// requests run.  vf4_attn_nvfp4_noalloc serves them: it runs the same kernels as
// vf4_attn_nvfp4, but its workspace is this file-scope device array instead of caller memory.
//
// Limits and contract:
//   * at most kNoAllocScratchBytes (16 MiB) of workspace, i.e. vf4_attn_workspace_size(B,H,S,D)
//     must not exceed it (the fused route needs 512 bytes per head, about 2000 ViT-L/14 images;
//     the long-sequence route about 4 ViT-H/14 @448 images); larger calls return
//     VF4_ERR_UNSUPPORTED and launch nothing;
//   * the array lives on every GPU that loads the library until the process exits;
//   * the host name g_attn_scratch is only a host-side stand-in for the symbol, never a device
//     address: the first call in each CUDA context (with its device current) resolves the real
//     address with cudaGetSymbolAddress and caches it keyed by the context's ID, so make that
//     first call before any stream capture; a new context on the device (after a device reset,
//     or a caller's own driver-API context) resolves again, and a failed resolution caches
//     nothing, so a later call retries;
//   * every call shares the one array and it keeps the last call's contents; nothing in it
//     has to start at zero (each call clears the three maxima itself, and the statistics and
//     prep kernels rewrite every other byte the later kernels read);
//   * calls whose kernels overlap on the GPU (different streams, no ordering) race on it.
// ---------------------------------------------------------------------------------------
namespace vf4 {
constexpr int64_t kNoAllocScratchBytes = 16ll << 20;
static __device__ __align__(256) uint8_t g_attn_scratch[kNoAllocScratchBytes];
struct ScratchSlot {
  unsigned long long ctx_id;   // CUDA context the address was resolved in (0: none yet)
  uint8_t* ptr;
};
static ScratchSlot g_scratch[64];
static std::mutex g_scratch_mu;

// The device address of g_attn_scratch in the current context, resolved on first use there.
static int scratch_address(int dev, uint8_t** out) {
  unsigned long long id = 0;
  if (current_context_id(&id) != VF4_OK)
    return fail(VF4_ERR_CUDA, "vf4_attn_nvfp4_noalloc: no current CUDA context");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  if (slot.ptr == nullptr || slot.ctx_id != id) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p)
      return fail(VF4_ERR_CUDA, "vf4_attn_nvfp4_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    slot.ptr = static_cast<uint8_t*>(p);
    slot.ctx_id = id;
  }
  *out = slot.ptr;
  return VF4_OK;
}
}  // namespace vf4

extern "C" int vf4_attn_nvfp4_noalloc(const void* q, const void* k, const void* v, int64_t B, int64_t H,
                                      int64_t S, int64_t D, int64_t stride_b, int64_t stride_h,
                                      int64_t stride_s, float scale, void* out, int64_t out_stride_b,
                                      int64_t out_stride_h, int64_t out_stride_s, vf4_stream_t stream) {
  if (int st = check_device()) return st;
  if (B <= 0 || H <= 0 || S <= 0 || D <= 0) return fail(VF4_ERR_ARG, "vf4_attn_nvfp4_noalloc: bad sizes");
  const int64_t need = vf4_attn_workspace_size(B, H, S, D);
  if (need > kNoAllocScratchBytes)
    return fail(VF4_ERR_UNSUPPORTED,
                "vf4_attn_nvfp4_noalloc: needs %lld bytes of scratch, the fixed device array holds %lld; "
                "split the batch or use vf4_attn_nvfp4 with a caller workspace",
                (long long)need, (long long)kNoAllocScratchBytes);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(VF4_ERR_CUDA, "vf4_attn_nvfp4_noalloc: no current device");
  uint8_t* scratch = nullptr;
  if (int st = scratch_address(dev, &scratch)) return st;
  return vf4_attn_nvfp4(q, k, v, B, H, S, D, stride_b, stride_h, stride_s, scale, out, out_stride_b,
                        out_stride_h, out_stride_s, scratch, kNoAllocScratchBytes, stream);
}
