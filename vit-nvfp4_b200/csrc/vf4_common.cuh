// Shared device helpers for the sm_100a NVFP4 kernels: exact fp32 arithmetic for the
// quantizer, E4M3/E2M1 encoders, mbarrier / TMA / tcgen05 inline PTX with bounded waits.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "vitfp4.h"

#define VF4_DEV __device__ __forceinline__

// A wait that exceeds this many nanoseconds of %globaltimer sets the device error word
// and returns false, so a kernel never spins forever on the shared GPU.
#ifndef VF4_WAIT_TIMEOUT_NS
#define VF4_WAIT_TIMEOUT_NS 4000000000ull
#endif

namespace vf4 {

// ---------------------------------------------------------------------------------------
// Device error word (one per translation unit; read through the TU's *_device_error()).
// ---------------------------------------------------------------------------------------
enum DevErr : int {
  kDevErrNone = 0,
  kDevErrTimeoutFull = 1,     // producer data never arrived
  kDevErrTimeoutEmpty = 2,    // consumer never released a stage
  kDevErrTimeoutTmem = 3,     // accumulator hand-off timed out
  kDevErrTimeoutDrain = 4,    // final drain of async tensor-core work timed out
  kDevErrTimeoutOther = 5,
};

VF4_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------
// Numeric formats
// ---------------------------------------------------------------------------------------
// fp32 -> E4M3 (float8_e4m3fn) bits, round-to-nearest-even with saturation to +-448.
VF4_DEV uint32_t f32_to_e4m3(float x) {
  __nv_fp8_storage_t r = __nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
  return (uint32_t)r;
}

VF4_DEV float e4m3_to_f32(uint32_t b) {
  __half_raw h = __nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)b, __NV_E4M3);
  return __half2float(*reinterpret_cast<__half*>(&h));
}

// E2M1 code of q with the reference's rounding: ties go to the smaller magnitude,
// NaN/+-inf saturate to index 7 (fminf(NaN, 6) == 6).
VF4_DEV uint32_t e2m1_code(float q) {
  uint32_t s = q < 0.f ? 8u : 0u;
  float m = fminf(fabsf(q), 6.f);
  uint32_t i = (uint32_t)(m > 0.25f) + (uint32_t)(m > 0.75f) + (uint32_t)(m > 1.25f) +
               (uint32_t)(m > 1.75f) + (uint32_t)(m > 2.5f) + (uint32_t)(m > 3.5f) +
               (uint32_t)(m > 5.0f);
  return s | i;
}

VF4_DEV float e2m1_value(uint32_t c) {
  // magnitudes {0,.5,1,1.5,2,3,4,6}
  uint32_t i = c & 7u;
  float m = i < 4 ? 0.5f * (float)i : (i == 7 ? 6.f : (float)(i - 2));
  return (c & 8u) ? -m : m;
}

// Exact erf-GELU (0.5*x*(1+erf(x/sqrt2))) using CUDA's erff.
VF4_DEV float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f));
}

VF4_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// ---------------------------------------------------------------------------------------
// Quantize one 16-element block exactly as the reference quantizer (RTN "six" or
// Four-Over-Six "mse").  v: fp32 values; gs: global scale; s_enc = 1/gs.
// Returns the 8 packed bytes (low nibble = even element) and the E4M3 scale byte.
// ---------------------------------------------------------------------------------------
struct BlockQ {
  uint64_t packed;
  uint32_t sf;
};

VF4_DEV void encode_candidate(const float* v, float amax, float divisor, float s_enc, float gs,
                              uint32_t* codes, uint32_t* sf, float* dec_out) {
  float bs_f = fminf(__fmul_rn(__fdiv_rn(amax, divisor), s_enc), 448.f);
  uint32_t b = f32_to_e4m3(bs_f);
  float dec = __fmul_rn(e4m3_to_f32(b), gs);
#pragma unroll
  for (int i = 0; i < 16; ++i) codes[i] = e2m1_code(__fdiv_rn(v[i], dec));
  *sf = b;
  *dec_out = dec;
}

VF4_DEV float block_mse_aten(const float* v, const uint32_t* codes, float dec) {
  float e[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    float d = __fsub_rn(__fmul_rn(e2m1_value(codes[i]), dec), v[i]);
    e[i] = __fmul_rn(d, d);
  }
  float s = __fadd_rn(e[0], e[8]);
#pragma unroll
  for (int i = 1; i < 8; ++i) s = __fadd_rn(s, __fadd_rn(e[i], e[i + 8]));
  return __fdiv_rn(s, 16.f);
}

// ---------------------------------------------------------------------------------------
// Fast exact encoder.
//
// q = RN(x / dec) is obtained from inv = RN(1/dec) with one Markstein correction step
// (P. Markstein, "Computation of elementary functions on the IBM RISC System/6000
// processor", IBM J. Res. Dev. 34(1), 1990): q0 = x*inv, r = x - q0*dec (exact with an FMA),
// q = q0 + r*inv, which is the correctly rounded quotient for normal results.  The E2M1 code is
// then produced by the hardware converter (cvt.rn.satfinite.e2m1x2.f32, nearest-even), and the
// three ties where nearest-even rounds UP to an even code while the reference rounds DOWN
// (|q| = 0.75, 1.75, 3.5) are moved one code down.  -0.0 is mapped to +0.0 first (the reference
// sign is q < 0).  dec == 0 (scale underflow) gives q = +-inf or NaN in the reference: 7 / 15.
// ---------------------------------------------------------------------------------------
VF4_DEV float div_markstein(float x, float d, float inv) {
  float q = __fmul_rn(x, inv);
  float r = __fmaf_rn(-q, d, x);
  return __fmaf_rn(r, inv, q);
}

// Four E2M1 bytes from eight values: byte i = (code(v[2i+1]) << 4) | code(v[2i]).
VF4_DEV uint32_t cvt_e2m1x8(const float* v) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(out)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return out;
}

VF4_DEV uint32_t odd_tie(float q) {
  float a = fabsf(q);
  return (uint32_t)((a == 0.75f) | (a == 1.75f) | (a == 3.5f));
}

// Bit-exact reference encoding of 16 values with decode scale dec (>= 0).
VF4_DEV uint64_t encode16_exact(const float* v, float dec) {
  if (dec == 0.f) {
    uint64_t p = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) p |= (uint64_t)(v[i] < 0.f ? 15u : 7u) << (4 * i);
    return p;
  }
  const float inv = __frcp_rn(dec);
  uint32_t w[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float q[8];
    uint32_t fix = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      q[i] = __fadd_rn(div_markstein(v[8 * h + i], dec, inv), 0.0f);
      fix |= odd_tie(q[i]) << (4 * i);
    }
    w[h] = cvt_e2m1x8(q) - fix;
  }
  return (uint64_t)w[0] | ((uint64_t)w[1] << 32);
}

// Bit-exact reference encoding of 8 values (half a block) with decode scale dec (>= 0).
VF4_DEV uint32_t encode8_exact(const float* v, float dec) {
  if (dec == 0.f) {
    uint32_t p = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) p |= (v[i] < 0.f ? 15u : 7u) << (4 * i);
    return p;
  }
  const float inv = __frcp_rn(dec);
  float q[8];
  uint32_t fix = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    q[i] = __fadd_rn(div_markstein(v[i], dec, inv), 0.0f);
    fix |= odd_tie(q[i]) << (4 * i);
  }
  return cvt_e2m1x8(q) - fix;
}

// Out-of-line entries to the exact encoders, for the rare blocks the bracketing encoders below
// cannot settle.  Kept out of line so the compiler branches around them: inlined, their
// correctly rounded reciprocal, Markstein quotients and tie tests were evaluated under a predicate
// for every block, more than doubling the instructions of the common path.
static __device__ __noinline__ uint64_t encode16_exact_ool(float4 a, float4 b, float4 c, float4 d, float dec) {
  const float v[16] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w, c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
  return encode16_exact(v, dec);
}

static __device__ __noinline__ uint32_t encode8_exact_ool(float4 a, float4 b, float dec) {
  const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  return encode8_exact(v, dec);
}

VF4_DEV uint64_t encode16_exact_call(const float* v, float dec) {
  return encode16_exact_ool(make_float4(v[0], v[1], v[2], v[3]), make_float4(v[4], v[5], v[6], v[7]),
                            make_float4(v[8], v[9], v[10], v[11]), make_float4(v[12], v[13], v[14], v[15]), dec);
}

VF4_DEV uint32_t encode8_exact_call(const float* v, float dec) {
  return encode8_exact_ool(make_float4(v[0], v[1], v[2], v[3]), make_float4(v[4], v[5], v[6], v[7]), dec);
}

// Bracketing encoder, bit-exact with encode16_exact at a fraction of its cost.
//
// The reference code of x is round_half_down(q) with q = RN(x / dec).  Instead of q, two
// brackets a = RN(x * lo) and b = RN(x * hi) are formed with lo, hi = (1 -+ 2^-20) / dec, so
// a < q < b strictly (the approximate reciprocal and the three roundings move them by less
// than 2^-21 relative), and both are converted with the hardware's nearest-even E2M1 rounding.
// The conversion is monotone, so equal codes for a and b mean that no E2M1 rounding boundary
// (midpoint) lies strictly between them; if a is itself an odd-type midpoint (0.75, 1.75, 3.5,
// where nearest-even rounds up), q > a rounds up in the reference too, and if b is a midpoint
// the codes differ unless nearest-even rounds b down, as the reference does for q < b.  So
// equal codes are the reference codes, and unequal codes (an element within ~2^-20 of a
// midpoint, rare for real data) send the block to encode16_exact.  The +0 in the FMA maps
// x = -0 to code 0 (the reference's sign is q < 0).  The fast path needs 2^-120 <= dec <=
// dec_max, where dec_max keeps every non-zero |x| / dec above 2^-150 so that q cannot round to
// -0 (the one case where a negative x has reference code 0): 2^17 for bf16 inputs
// (|x| >= 2^-133), 2 for fp32 inputs (|x| >= 2^-149).  Two packed FMAs per element pair
// (fma.rn.f32x2) and two converts per pair replace the divide, correction and tie tests.
VF4_DEV unsigned long long f32x2_pack(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}

VF4_DEV void f32x2_unpack(unsigned long long r, float* a, float* b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(*a), "=f"(*b) : "l"(r));
}

VF4_DEV unsigned long long fma_f32x2(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

VF4_DEV unsigned long long add_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

VF4_DEV unsigned long long mul_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// bf16 pair (low half = first element) <-> fp32 pair, and RN rounding of an fp32 pair to bf16
VF4_DEV unsigned long long bf16x2_to_f32x2(uint32_t w) {
  return f32x2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

VF4_DEV uint32_t bf16x2_round(unsigned long long p) {
  float a, b;
  f32x2_unpack(p, &a, &b);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(b), "f"(a));   // first operand -> upper half
  return r;
}

// The bracketing multipliers lo < 1/dec < hi of the encoders below.
VF4_DEV void bracket_mults(float dec, float* lo, float* hi) {
  float inv;
  asm("rcp.approx.f32 %0, %1;" : "=f"(inv) : "f"(dec));
  *lo = __fmul_rn(inv, 1.0f - 0x1p-20f);
  *hi = __fmul_rn(inv, 1.0f + 0x1p-20f);
}

// The fast path is computed whatever dec is and then checked once, together with dec's range (one
// branch to the exact path instead of two); out of range its codes are discarded.  q = {dec, lo,
// hi} (bracket_mults of dec): the form whose caller looked them up in a per-scale-byte table.
VF4_DEV uint64_t encode16_bracket_q(const float* v, float4 q, float dec_max) {
  const float dec = q.x, lo = q.y, hi = q.z;
  const unsigned long long lo2 = f32x2_pack(lo, lo), hi2 = f32x2_pack(hi, hi), z2 = f32x2_pack(0.f, 0.f);
  uint32_t wa[2], wb[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float a[8], b[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const unsigned long long x2 = f32x2_pack(v[8 * h + 2 * i], v[8 * h + 2 * i + 1]);
      f32x2_unpack(fma_f32x2(x2, lo2, z2), &a[2 * i], &a[2 * i + 1]);
      f32x2_unpack(fma_f32x2(x2, hi2, z2), &b[2 * i], &b[2 * i + 1]);
    }
    wa[h] = cvt_e2m1x8(a);
    wb[h] = cvt_e2m1x8(b);
  }
  const bool fast = (dec >= 0x1p-120f) & (dec <= dec_max) & (wa[0] == wb[0]) & (wa[1] == wb[1]);
  if (!fast) return encode16_exact_call(v, dec);
  return (uint64_t)wa[0] | ((uint64_t)wa[1] << 32);
}

VF4_DEV uint64_t encode16_bracket(const float* v, float dec, float dec_max) {
  float lo, hi;
  bracket_mults(dec, &lo, &hi);
  return encode16_bracket_q(v, make_float4(dec, lo, hi, 0.f), dec_max);
}

// Half a block (8 values) with the bracketing scheme of encode16_bracket.
VF4_DEV uint32_t encode8_bracket_q(const float* v, float4 q, float dec_max) {
  const float dec = q.x, lo = q.y, hi = q.z;
  const unsigned long long lo2 = f32x2_pack(lo, lo), hi2 = f32x2_pack(hi, hi), z2 = f32x2_pack(0.f, 0.f);
  float a[8], b[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const unsigned long long x2 = f32x2_pack(v[2 * i], v[2 * i + 1]);
    f32x2_unpack(fma_f32x2(x2, lo2, z2), &a[2 * i], &a[2 * i + 1]);
    f32x2_unpack(fma_f32x2(x2, hi2, z2), &b[2 * i], &b[2 * i + 1]);
  }
  const uint32_t wa = cvt_e2m1x8(a), wb = cvt_e2m1x8(b);
  const bool fast = (dec >= 0x1p-120f) & (dec <= dec_max) & (wa == wb);
  return fast ? wa : encode8_exact_call(v, dec);
}

VF4_DEV uint32_t encode8_bracket(const float* v, float dec, float dec_max) {
  float lo, hi;
  bracket_mults(dec, &lo, &hi);
  return encode8_bracket_q(v, make_float4(dec, lo, hi, 0.f), dec_max);
}

// Epilogue encoding: quotient by reciprocal multiply and hardware nearest-even rounding
// (differs from the reference only within one ulp of a rounding boundary or on an exact tie).
VF4_DEV uint64_t encode16_fast(const float* v, float dec) {
  if (dec == 0.f) {
    uint64_t p = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) p |= (uint64_t)(v[i] < 0.f ? 15u : 7u) << (4 * i);
    return p;
  }
  const float inv = __frcp_rn(dec);
  float q[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) q[i] = v[i] * inv;
  return (uint64_t)cvt_e2m1x8(q) | ((uint64_t)cvt_e2m1x8(q + 8) << 32);
}

// encode16_fast with the reciprocal of the decode scale given (inv = __frcp_rn(dec)) and the
// products formed by packed multiplies; zero_scale selects the dec == 0 codes of encode16_fast.
VF4_DEV uint64_t encode16_inv(const float* v, float inv, bool zero_scale) {
  if (zero_scale) {
    uint64_t p = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) p |= (uint64_t)(v[i] < 0.f ? 15u : 7u) << (4 * i);
    return p;
  }
  const unsigned long long inv2 = f32x2_pack(inv, inv);
  float q[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) f32x2_unpack(mul_f32x2(f32x2_pack(v[2 * i], v[2 * i + 1]), inv2), &q[2 * i], &q[2 * i + 1]);
  return (uint64_t)cvt_e2m1x8(q) | ((uint64_t)cvt_e2m1x8(q + 8) << 32);
}

// per-16-bit-lane unsigned max of two pairs (max.u16x2)
VF4_DEV uint32_t umax_u16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("max.u16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// max(a, b, c) in one instruction (three-operand max.f32, sm_100)
VF4_DEV float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// min(a, b, c) in one instruction (three-operand min.f32, sm_100)
VF4_DEV float min3f(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// max |v_i| over 16 values
VF4_DEV float amax16(const float* v) {
  float m = max3f(fabsf(v[0]), fabsf(v[1]), fabsf(v[2]));
#pragma unroll
  for (int i = 3; i < 15; i += 2) m = max3f(m, fabsf(v[i]), fabsf(v[i + 1]));
  return fmaxf(m, fabsf(v[15]));
}

// E4M3 block scale (six rule) and its decode value: bs = e4m3(min((amax/6)*s_enc, 448)).
// RN(a / 6) for normal a by one Markstein correction step (q0 = a*y, r = a - 6*q0 exact by FMA,
// q = q0 + r*y with y = RN(1/6)); checked against IEEE division for every significand in
// [1, 2), which covers all a >= 1e-12 since both sides scale exactly by powers of two.
VF4_DEV float div6_rn(float a) {
  const float y = 0.16666667163372039795f;   // RN(1/6) = 0x3E2AAAAB
  const float q = __fmul_rn(a, y);
  return __fmaf_rn(__fmaf_rn(-q, 6.0f, a), y, q);
}

// The six rule's E4M3 scale byte of a block with maximum |x| amax (0 .. 126).
VF4_DEV uint32_t six_code(float amax, float s_enc) {
  return f32_to_e4m3(fminf(__fmul_rn(div6_rn(fmaxf(amax, 1e-12f)), s_enc), 448.f));
}

// {dec, lo, hi} of scale byte b under the global scale gs: the decode scale six_scale returns and
// its bracketing multipliers, for a per-CTA table indexed by the scale byte.
VF4_DEV float4 scale_entry(uint32_t b, float gs) {
  const float dec = __fmul_rn(e4m3_to_f32(b), gs);
  float lo, hi;
  bracket_mults(dec, &lo, &hi);
  return make_float4(dec, lo, hi, 0.f);
}

VF4_DEV uint32_t six_scale(float amax, float s_enc, float gs, float* dec) {
  float bs_f = fminf(__fmul_rn(div6_rn(fmaxf(amax, 1e-12f)), s_enc), 448.f);
  uint32_t b = f32_to_e4m3(bs_f);
  *dec = __fmul_rn(e4m3_to_f32(b), gs);
  return b;
}

// dec_max: the largest decode scale for which encode16_bracket may take its fast path for the
// inputs at hand (2^17 for bf16 values, 2 for arbitrary fp32 values).
template <bool kMse>
VF4_DEV BlockQ quantize_block(const float* v, float gs, float s_enc, float dec_max = 2.0f) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[i]));
  amax = fmaxf(amax, 1e-12f);
  BlockQ r;
  if constexpr (kMse) {
    uint32_t c6[16], sf6, c4[16], sf4;
    float dec6, dec4;
    encode_candidate(v, amax, 6.f, s_enc, gs, c6, &sf6, &dec6);
    encode_candidate(v, amax, 4.f, s_enc, gs, c4, &sf4, &dec4);
    bool pick4 = block_mse_aten(v, c4, dec4) < block_mse_aten(v, c6, dec6);
    uint64_t p = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) p |= (uint64_t)(pick4 ? c4[i] : c6[i]) << (4 * i);
    r.packed = p;
    r.sf = pick4 ? sf4 : sf6;
  } else {
    float dec;
    r.sf = six_scale(amax, s_enc, gs, &dec);
    r.packed = encode16_bracket(v, dec, dec_max);
  }
  return r;
}

// GELU in its tanh form, 0.5x(1 + tanh(sqrt(2/pi)(x + 0.044715x^3))), with the hardware
// tanh.approx.f32: one special-function op per element (the A&S form above needs two).
VF4_DEV float gelu_tanh(float x) {
  const float v = x * __fmaf_rn(0.0356774081f, x * x, 0.7978845608f);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(v));
  const float hx = 0.5f * x;
  return __fmaf_rn(hx, t, hx);
}

// gelu_tanh on an element pair with the packed fp32 ops (the same roundings, op for op)
VF4_DEV unsigned long long gelu_tanh_x2(unsigned long long x2) {
  const unsigned long long c1 = f32x2_pack(0.0356774081f, 0.0356774081f);
  const unsigned long long c0 = f32x2_pack(0.7978845608f, 0.7978845608f);
  const unsigned long long half2 = f32x2_pack(0.5f, 0.5f);
  float u0, u1, t0, t1;
  f32x2_unpack(mul_f32x2(x2, fma_f32x2(mul_f32x2(x2, x2), c1, c0)), &u0, &u1);
  asm("tanh.approx.f32 %0, %1;" : "=f"(t0) : "f"(u0));
  asm("tanh.approx.f32 %0, %1;" : "=f"(t1) : "f"(u1));
  const unsigned long long hx = mul_f32x2(x2, half2);
  return fma_f32x2(hx, f32x2_pack(t0, t1), hx);
}

// RN(a + b) of two bf16 pairs.  For bf16 operands this equals torch's bf16 add (an fp32 add, then
// one rounding to bf16): the fp32 sum of two bf16 values is exact unless their exponents differ by
// more than 16, and then the sum lies within 2^-16 relative of the larger operand, far from any
// bf16 rounding midpoint, so rounding once or twice gives the same bf16 value.
VF4_DEV uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// RN(a * b) of two bf16 pairs.  The exact product of two bf16 values has at most 16 significant
// bits, so the fp32 product is exact (outside fp32's subnormal range) and torch's bf16 multiply (an
// fp32 multiply, then one rounding to bf16) gives the same bf16 value.
VF4_DEV uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// erf-GELU, 0.5 x (1 + erf(x / sqrt 2)), on an element pair in packed fp32 arithmetic.  Since erf
// is odd, gelu(x) = relu(x) - |x| E with E = 0.5 erfc(|x| / sqrt 2), and E comes from Abramowitz &
// Stegun 7.1.26 (|error of erf| <= 1.5e-7):
//   E = 0.5 (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-x^2 / 2),   t = 1 / (1 + p |x| / sqrt 2),
// with exp(-x^2 / 2) = 2^(-(|x| s)^2), s = sqrt(log2(e) / 2): one reciprocal and one ex2 per element
// and no comparison or select (measured in a throughput probe as the fastest of the erf forms tried,
// 1.25x the single-ex2 polynomial).  For x -> -inf the result goes to 0 as E underflows (also at
// x = -inf, where 0.5 x (1 + erf(x / sqrt 2)) is NaN); +inf gives +inf and NaN propagates.
VF4_DEV unsigned long long gelu_erf_x2(unsigned long long x2) {
  constexpr float kP = 0.3275911f * 0.70710678118654752f;   // p / sqrt 2
  constexpr float kS = 0.84932180028801904272f;              // sqrt(log2(e) / 2)
  // -0.5 a_k: the polynomial comes out negated, -E / exp(-x^2 / 2), exactly (RN is sign-symmetric)
  constexpr float kA1 = -0.5f * 0.254829592f, kA2 = -0.5f * -0.284496736f, kA3 = -0.5f * 1.421413741f,
                  kA4 = -0.5f * -1.453152027f, kA5 = -0.5f * 1.061405429f;
  float x0, x1;
  f32x2_unpack(x2, &x0, &x1);
  // |x| capped below +inf, so that |x| * exp(-x^2 / 2) is 0 rather than inf * 0 for x = +-inf; the
  // NaN-propagating min keeps a NaN input NaN (through m below; the relu term drops it)
  float z0, z1;
  asm("min.NaN.f32 %0, %1, 0f7E800000;" : "=f"(z0) : "f"(fabsf(x0)));
  asm("min.NaN.f32 %0, %1, 0f7E800000;" : "=f"(z1) : "f"(fabsf(x1)));
  const unsigned long long z = f32x2_pack(z0, z1);
  float d0, d1, t0, t1;
  f32x2_unpack(fma_f32x2(z, f32x2_pack(kP, kP), f32x2_pack(1.f, 1.f)), &d0, &d1);
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(d1));
  const unsigned long long t = f32x2_pack(t0, t1);
  unsigned long long poly = fma_f32x2(f32x2_pack(kA5, kA5), t, f32x2_pack(kA4, kA4));
  poly = fma_f32x2(poly, t, f32x2_pack(kA3, kA3));
  poly = fma_f32x2(poly, t, f32x2_pack(kA2, kA2));
  poly = fma_f32x2(poly, t, f32x2_pack(kA1, kA1));
  poly = mul_f32x2(poly, t);
  const unsigned long long w = mul_f32x2(z, f32x2_pack(kS, kS));
  float q0, q1, e0, e1;
  f32x2_unpack(mul_f32x2(w, w), &q0, &q1);
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(-q0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(-q1));
  const unsigned long long m = mul_f32x2(z, f32x2_pack(e0, e1));              // |x| exp(-x^2 / 2)
  const unsigned long long relu = f32x2_pack(fmaxf(x0, 0.f), fmaxf(x1, 0.f));
  return fma_f32x2(m, poly, relu);                                          // relu(x) - |x| E
}

// Offset of scale factor (row r, column c) inside the 128x4-tiled ("to_blocked") layout.
VF4_DEV int64_t sf_swizzle_offset(int64_t r, int64_t c, int64_t n_col_blocks) {
  return ((r >> 7) * n_col_blocks + (c >> 2)) * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (c & 3);
}

// ---------------------------------------------------------------------------------------
// Shared memory, mbarrier and TMA helpers
// ---------------------------------------------------------------------------------------
VF4_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

VF4_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

VF4_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

VF4_DEV void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

VF4_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

VF4_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

VF4_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (after recording `code` in *err) if the phase does not complete
// within limit_ns of %globaltimer (checked every 256 polls) or another role already gave up.
VF4_DEV bool mbar_wait_limit(uint32_t bar, uint32_t parity, int* err, int code, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*(volatile int*)err != 0) return false;  // another role already gave up
      if (globaltimer() - t0 > limit_ns) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

VF4_DEV bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
  return mbar_wait_limit(bar, parity, err, code, VF4_WAIT_TIMEOUT_NS);
}

VF4_DEV bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait with cluster-scope acquire (for barriers that the peer CTA arrives on).
VF4_DEV bool mbar_wait_cluster(uint32_t bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*(volatile int*)err != 0) return false;
      if (globaltimer() - t0 > VF4_WAIT_TIMEOUT_NS) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

VF4_DEV void tma_prefetch(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

VF4_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* m, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 2-D tensor store shared -> global (bulk-group completion); coordinates in elements.
VF4_DEV void tma_store_2d(const CUtensorMap* m, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
VF4_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store has finished READING shared memory.
VF4_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
VF4_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Plain (non-tensor) bulk copy global -> shared; dst/src 16B aligned, bytes % 16 == 0.
VF4_DEV void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core) helpers
// ---------------------------------------------------------------------------------------
VF4_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
VF4_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
VF4_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
VF4_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
VF4_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on an mbarrier once all previously issued tcgen05 async ops of this thread finish.
VF4_DEV void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// Block-scaled FP4 MMA: D[tmem] (+)= A[smem] * B[smem]^T with UE4M3 scales (16-element
// vectors) read from tensor memory.  M=128, N from the instruction descriptor, K=64.
VF4_DEV void mma_mxf4nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                          uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// Copy a 32-row x 16-byte matrix from shared memory into tensor memory, replicated into
// all four 32-lane sub-partitions (the scale-factor staging the MMA expects).
VF4_DEV void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// 128 lanes x 256 bits: lane l takes row l of a K-major no-swizzle shared-memory matrix (two
// 16-byte core-matrix columns, LBO apart; 8-row groups SBO apart) into 8 consecutive columns.
VF4_DEV void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

VF4_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns -> 32 registers per thread.
VF4_DEV void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 8 consecutive 32-bit columns -> 8 registers per thread.
VF4_DEV void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns -> 16 registers per thread.
VF4_DEV void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Named barrier over `count` threads (a multiple of 32) of the CTA.
VF4_DEV void named_bar_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 4-D tensor load / store (coordinates innermost first, in elements).
VF4_DEV void tma_load_4d(uint32_t dst, const CUtensorMap* m, int32_t c0, int32_t c1, int32_t c2, int32_t c3,
                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

VF4_DEV void tma_store_4d(const CUtensorMap* m, uint32_t src, int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// ---- CTA-pair (cluster of 2) helpers for cta_group::2 MMAs
VF4_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
VF4_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory variable in CTA `cta` of the cluster.
VF4_DEV uint32_t mapa_shared(uint32_t addr, uint32_t cta) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(cta));
  return r;
}
VF4_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
VF4_DEV void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
VF4_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
VF4_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive (once the issuing thread's tcgen05 ops complete) on the barrier at this shared offset in
// every CTA of `mask` (bit i = cluster CTA i).
VF4_DEV void tc_commit_pair(uint32_t bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(mask)
      : "memory");
}
// Pair MMA: M = 256 split over the two CTAs (128 rows each, A and D in each CTA's own smem / TMEM),
// B's N rows split in halves across the two CTAs' shared memory at the same offsets.
VF4_DEV void mma_mxf4nvf4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t sfa_tmem,
                               uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X [%0], %1, %2, %3, [%5], "
      "[%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// Scale staging for the pair MMA: each CTA copies the 32x16-byte atom at this smem offset into
// its own TMEM (replicated to the four lane sub-partitions).
VF4_DEV void tmem_cp_32x128b_x4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Shared-memory matrix descriptor (tcgen05 "version 1" format).
//   layout 2 = 128-byte swizzle (K-major operand tiles written by TMA SWIZZLE_128B),
//   layout 0 = no swizzle (scale-factor staging for tcgen05.cp).
VF4_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::mxf4nvf4: A/B E2M1, UE4M3 scales, K-major A and B,
// M=128, N=n (multiple of 16, <= 256), dense, K=64.
__host__ __device__ constexpr uint32_t idesc_mxf4nvf4(uint32_t n, uint32_t m = 128) {
  return (1u << 7)             // A format: E2M1
         | (1u << 10)          // B format: E2M1
         | ((n >> 3) << 17)    // N >> 3
         | (0u << 23)          // scale type UE4M3
         | ((m >> 4) << 24);   // M >> 4
}

}  // namespace vf4
