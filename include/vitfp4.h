/*
 * vitfp4 — C ABI of the B200 (sm_100a) NVFP4 W4A4 ViT hot path (libvitfp4.so).
 *
 * Conventions (every entry point):
 *   - plain pointers and sizes, no framework types; all data pointers are DEVICE pointers
 *     owned by the caller (outputs pre-allocated by the caller);
 *   - the CUDA stream is the last argument; every call is asynchronous on that stream;
 *   - the return value is a vf4_status (0 = ok); vf4_last_error_string() describes the
 *     last failure of the calling thread; nothing throws across the ABI;
 *   - no entry point allocates device memory.
 *
 * Layouts:
 *   packed codes : (rows, K/2) uint8, two E2M1 codes per byte, low nibble = even column
 *   swizzled SF  : the 128x4-tiled E4M3 block-scale layout ("to_blocked"):
 *                  padded to (ceil128(rows), ceil4(K/16)); tile (rb,cb) at (rb*nCB+cb)*512;
 *                  element (r,c) of a tile at (r%32)*16 + (r/32)*4 + c
 *   linear SF    : (rows, K/16) uint8 E4M3 bytes, row-major
 *   global scale : one fp32 in device memory; decode x = e2m1 * e4m3 * gs
 *
 * The reference (Dev-Jahn/vit-nvfp4) is pure Python; each function below replaces the
 * Python/Triton/cuBLASLt call named beside it (file:line in the reference project).
 */
#ifndef VITFP4_H_
#define VITFP4_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define VF4_API __attribute__((visibility("default")))
#else
#define VF4_API
#endif

typedef struct CUstream_st* vf4_stream_t; /* == cudaStream_t */

typedef enum {
  VF4_OK = 0,
  VF4_ERR_ARG = 1,         /* bad size / mode / null pointer */
  VF4_ERR_ALIGN = 2,       /* pointer or leading dimension misaligned for the kernel */
  VF4_ERR_ARCH = 3,        /* device is not sm_100 */
  VF4_ERR_LAUNCH = 4,      /* kernel launch failed */
  VF4_ERR_CUDA = 5,        /* other CUDA runtime/driver error */
  VF4_ERR_UNSUPPORTED = 6, /* shape outside what the kernels implement */
  VF4_ERR_DEVICE = 7       /* a kernel recorded a device-side timeout */
} vf4_status;

typedef enum { VF4_BF16 = 0, VF4_F32 = 1 } vf4_dtype;
typedef enum { VF4_SIX = 0, VF4_MSE = 1 } vf4_block_select;
typedef enum {
  VF4_EPI_NONE = 0,      /* out = gs_a*gs_b*acc                                   */
  VF4_EPI_BIAS = 1,      /* out = gs_a*gs_b*acc + bias                            */
  VF4_EPI_GELU_NVFP4 = 2,    /* h = GELU(gs_a*gs_b*acc + bias) (tanh form), NVFP4-cast h */
  VF4_EPI_GELU_ERF_NVFP4 = 3, /* same with erf-GELU (A&S 7.1.26, |erf error| <= 1.5e-7)    */
  VF4_EPI_BIAS_RESIDUAL = 4   /* out = residual + gamma * (gs_a*gs_b*acc + bias), bf16 only;
                                 only through vf4_gemm_nvfp4_residual                       */
} vf4_epilogue;

/* Library version (major*10000 + minor*100 + patch). */
VF4_API int vf4_version(void);

/* Message for the last non-zero status returned on this thread. */
VF4_API const char* vf4_last_error_string(void);

/* Read (and optionally clear) the device-side error word of every kernel family
 * (0 = none; otherwise a kernel gave up on a bounded wait). Synchronizes the device. */
VF4_API int vf4_device_error(int clear);

/* Self-test of the failure detector: launches one kernel whose bounded mbarrier wait (the wait every
 * kernel here uses, given limit_ns instead of the production 4 s) waits on a barrier nothing arrives
 * on.  The kernel gives up after limit_ns (0 < limit_ns <= 1e9), records VF4 device error 1 (producer
 * data never arrived) for vf4_device_error and returns; the context stays usable.  No reference
 * counterpart (the reference has no device-side waits). */
VF4_API int vf4_selftest_wait_timeout(uint64_t limit_ns, vf4_stream_t stream);

/* max|x| (or max|GELU(x)| when gelu != 0) over n elements, written to *amax_out.
 * Replaces the amax pass inside quant.py:48-49 and fused_mlp.py:25-29. */
VF4_API int vf4_amax(const void* x, int dtype, int64_t n, int gelu, float* amax_out, vf4_stream_t stream);

/* *gs_out = max(*amax, 1e-12) / (6 * (block_select == VF4_MSE ? 256 : 448)).
 * Replaces quant.py:48-53. amax and gs_out may alias. */
VF4_API int vf4_global_scale(const float* amax, int block_select, float* gs_out, vf4_stream_t stream);

/* out[i] = erf-GELU(x[i]) for n fp32 values, computed by the device function of the fc1
 * GELU-NVFP4 epilogue: 0.5 x (1 + erf(x / sqrt 2)) with erf from Abramowitz & Stegun 7.1.26
 * (|error| <= 1.5e-7), one reciprocal and one ex2 per element.
 * The reference's GELU is torch's F.gelu / Triton's tl.erf in triton_cast.py:302-303; this
 * elementwise form exists so the epilogue's function can be checked and reused on its own. */
VF4_API int vf4_gelu_erf_f32(const float* x, int64_t n, float* out, vf4_stream_t stream);

/* NVFP4 activation / weight cast, bit-exact to quantize_to_nvfp4 + pack_e2m1 + to_blocked
 * (quant.py:20-69, pack.py:4-9, pack.py:39-58) and the fused GELU cast of
 * triton_cast.py:138 (cast_nvfp4) with the quant.py arithmetic.
 *   x        : (M, K) rows of stride ld elements, dtype VF4_BF16 or VF4_F32, K % 16 == 0
 *   gs       : device fp32 global scale to use (static), or NULL for dynamic: the amax of
 *              the (GELU'd, biased) input is computed first and the scale written to gs_out
 *   bias     : optional (K,) vector of the same dtype added before GELU / quantization
 *   out_packed (M, K/2); out_sf_swizzled (ceil128(M)*ceil4(K/16) bytes, pads zeroed) and/or
 *   out_sf_linear (M, K/16) — either may be NULL; gs_out (1 fp32) receives the scale used
 *   (may be NULL when gs != NULL).
 * Calls whose flat block index and offsets all fit in 31 bits run a kernel with 32-bit index
 * arithmetic; the environment variable VF4_CAST_INDEX64 keeps the 64-bit kernel (same bytes). */
VF4_API int vf4_cast_nvfp4(const void* x, int dtype, int64_t M, int64_t K, int64_t ld, const float* gs,
                   int block_select, int gelu, const void* bias, uint8_t* out_packed,
                   uint8_t* out_sf_swizzled, uint8_t* out_sf_linear, float* gs_out,
                   vf4_stream_t stream);

/* LayerNorm fused into the NVFP4 activation cast, optionally after a fused residual + LayerScale
 * (replaces the bf16 chain  x = x + ls(y);  h = norm(x);  quantize_to_nvfp4(h)  that a timm-style
 * block runs around qlinear.py:42-47 / fused_mlp.py:47; the reference leaves it to torch):
 *   if y != NULL: x' = bf16(x + bf16(y * gamma)) (gamma NULL -> 1) is written to x_out (may be x)
 *   h = bf16(LayerNorm(x'; ln_w, ln_b, eps)) is cast to NVFP4 (six rule) with the static global gs,
 *   or, when gs == NULL, with the dynamic amax(|h|)/(6*448) written to gs_out (two passes; the
 *   first leaves each row's mean and rstd in the first 8 bytes of its out_packed row, which the
 *   second reads and overwrites with the codes, so out_packed must not alias x or y).
 * x, y, x_out: (M, K) bf16 contiguous; gamma, ln_w, ln_b: (K,) bf16; K % 64 == 0, K <= 1280.
 * out_packed (M, K/2); out_sf swizzled (ceil128(M) x K/16, padding rows zeroed). */
VF4_API int vf4_ln_cast_nvfp4(const void* x, const void* y, const void* gamma, void* x_out, const void* ln_w,
                              const void* ln_b, float eps, int64_t M, int64_t K, const float* gs,
                              uint8_t* out_packed, uint8_t* out_sf, float* gs_out, vf4_stream_t stream);

/* pack_e2m1 (pack.py:4-9): codes (rows, K) -> (rows, K/2). K % 2 == 0. */
VF4_API int vf4_pack_e2m1(const uint8_t* codes, int64_t rows, int64_t K, uint8_t* out, vf4_stream_t stream);

/* unpack_e2m1 (pack.py:12-16): (rows, Kh) -> (rows, 2*Kh). */
VF4_API int vf4_unpack_e2m1(const uint8_t* packed, int64_t rows, int64_t Kh, uint8_t* out,
                    vf4_stream_t stream);

/* to_blocked (pack.py:39-58): (R, C) E4M3 bytes -> ceil128(R)*ceil4(C) swizzled bytes. */
VF4_API int vf4_to_blocked(const uint8_t* sf, int64_t R, int64_t C, uint8_t* out, vf4_stream_t stream);

/* Block-scaled FP4 GEMM on tcgen05 tensor cores (replaces torch._scaled_mm_v2 in
 * backends/torch_scaled_mm.py:14-46 and the emulation of backends/reference.py:6-10):
 *   acc[m,n] = sum_k A[m,k]*B[n,k] (E2M1 x E4M3 block scales), fp32 accumulate;
 *   A packed (M, K/2) + swizzled SF, B packed (N, K/2) + swizzled SF, a_gs/b_gs device fp32.
 * epilogue VF4_EPI_NONE / VF4_EPI_BIAS write `out` (M, N) in out_dtype (bias: (N,) bf16);
 * VF4_EPI_GELU_NVFP4 / VF4_EPI_GELU_ERF_NVFP4 (the fused fc1 epilogue of fused_mlp.py:47-51)
 * write out_packed (M, N/2) and out_sf (swizzled, ceil128(M) x N/16) quantized with the
 * static global scale epi_gs (six rule), and ignore `out`.  The fc1 output stays fp32 (the
 * unfused reference rounds it to bf16 first).  VF4_EPI_GELU_NVFP4 evaluates GELU as
 * 0.5x(1 + tanh(0.79788456x + 0.03567741x^3)) with the hardware tanh (max |deviation from
 * erf-GELU| ~1e-3, below the bf16 rounding the reference applies to this tensor);
 * VF4_EPI_GELU_ERF_NVFP4 evaluates erf-GELU to 1.5e-7 at about 1.5x the epilogue cost.
 * Requirements: K % 32 == 0, N % 16 == 0 (N % 64 == 0 for the GELU epilogues), 16-byte
 * aligned pointers. */
VF4_API int vf4_gemm_nvfp4(const uint8_t* a_packed, const uint8_t* a_sf, const float* a_gs,
                   const uint8_t* b_packed, const uint8_t* b_sf, const float* b_gs, int64_t M,
                   int64_t N, int64_t K, const void* bias, int epilogue, void* out, int out_dtype,
                   const float* epi_gs, uint8_t* out_packed, uint8_t* out_sf, vf4_stream_t stream);

/* GEMM with the transformer block's closing step fused into its epilogue:
 *   out = residual + gamma * (bf16(bf16(gs_a*gs_b*acc) + bias))        (all bf16, (M, N))
 * with the same rounding steps as the unfused block x + ls(fc2(h)) of a timm / DINOv2 block:
 * the GEMM result rounds to bf16, the bias add rounds, the LayerScale product rounds, the
 * residual add rounds (gamma NULL: no LayerScale; bias NULL: no bias).  The reference leaves this
 * to eager torch / torch.compile after its fused MLP (ptq/fused_mlp.py:47-55).  residual, gamma
 * and out are bf16, 16-byte aligned; out may be the residual buffer itself. */
VF4_API int vf4_gemm_nvfp4_residual(const uint8_t* a_packed, const uint8_t* a_sf, const float* a_gs,
                                    const uint8_t* b_packed, const uint8_t* b_sf, const float* b_gs,
                                    int64_t M, int64_t N, int64_t K, const void* bias, const void* residual,
                                    const void* gamma, void* out, vf4_stream_t stream);

/* B scale image: the weight-side copy of b_sf that lets the GEMM load a 256-row tile's scales for a
 * K64 block with one tensor-memory copy instead of two (each atom of the to_blocked layout held four
 * times over: per 256-row tile and K64 block [rows 0-127 atom x4][rows 128-255 atom x4], 4 KB).  No
 * counterpart in the reference (cuBLASLt takes the to_blocked scales as they are); built once per
 * weight, like the reference's packed weight cache.  vf4_b_scale_image_bytes(N, K) is its size;
 * vf4_b_scale_image writes it from b_sf ((N, K) weight, to_blocked scales; 16-byte aligned). */
VF4_API int64_t vf4_b_scale_image_bytes(int64_t N, int64_t K);
VF4_API int vf4_b_scale_image(const uint8_t* b_sf, int64_t N, int64_t K, uint8_t* image, vf4_stream_t stream);

/* vf4_gemm_nvfp4 / vf4_gemm_nvfp4_residual with every option in one call: epilogue any VF4_EPI_*
 * (residual and gamma for VF4_EPI_BIAS_RESIDUAL, else NULL) and b_image (NULL or the B scale image of
 * b_sf): with it the streaming kernel (K > 1024, N >= 256) copies each K64 block's B scales with one
 * tensor-memory copy (fc2 of ViT-L/14, K = 4096: about 10% faster); results are bit-identical. */
VF4_API int vf4_gemm_nvfp4_ex(const uint8_t* a_packed, const uint8_t* a_sf, const float* a_gs,
                              const uint8_t* b_packed, const uint8_t* b_sf, const uint8_t* b_image,
                              const float* b_gs, int64_t M, int64_t N, int64_t K, const void* bias, int epilogue,
                              void* out, int out_dtype, const float* epi_gs, uint8_t* out_packed, uint8_t* out_sf,
                              const void* residual, const void* gamma, vf4_stream_t stream);

/* Bytes of workspace vf4_attn_nvfp4 needs for (B, H, S, D) (0 for invalid sizes). */
VF4_API int64_t vf4_attn_workspace_size(int64_t B, int64_t H, int64_t S, int64_t D);

/* NVFP4 attention (replaces the emulated quant_sdpa(qk='nvfp4', pv='nvfp4'),
 * nvfp4/attention.py:53-86, reached through ptq/qattention.py:20-30):
 *   q, k, v : bf16, element (b, h, s, d) at ptr + b*stride_b + h*stride_h + s*stride_s + d
 *             (the packed qkv projection output and (B, H, S, D) tensors both fit)
 *   out     : bf16, element (b, h, s, d) at out + b*out_stride_b + h*out_stride_h + s*out_stride_s + d
 *   smooth-K / smooth-V always on; global scales of Q, K~, V~ over the whole tensors, as the
 *   reference (a statistics kernel runs first); P quantized along keys with the fixed global
 *   1/(6*448) instead of the amax of the whole P tensor; no mask, not causal.
 *   D % 16 == 0, D <= 128; S <= 1152 for D > 64.  Every route quantizes P = exp(S - rowmax) (in
 *   [0, 1], exactly 1 at the row max) and divides the output by the row sum.  Head dim 64 with
 *   S <= 320 (ViT-S/B/L) runs as one fused kernel and needs scale >= 0 (VF4_ERR_UNSUPPORTED
 *   otherwise); other shapes run prep + forward kernels and take any scale.
 *   workspace: at least vf4_attn_workspace_size(B, H, S, D) bytes, 16-byte aligned. */
VF4_API int vf4_attn_nvfp4(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S,
                           int64_t D, int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale,
                           void* out, int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s,
                           void* workspace, int64_t workspace_bytes, vf4_stream_t stream);

/* FP8 attention, the reference's default route quant_sdpa(qk='fp8', pv='fp8') (attention.py:53-86,
 * fp8.py:6-17, reached through ptq/qattention.py:20-30 with enable_quant_attention's defaults):
 * smooth-K / smooth-V, then Q and K~ quantized to E4M3 per token (scale amax/448 of the row), P per
 * query row and V~ per head-dim column along tokens; E4M3 MMAs with fp32 accumulation and the
 * scales applied to scores and output.  Same operand / output layout and strides as
 * vf4_attn_nvfp4; head dim 64 and S <= 320 (VF4_ERR_UNSUPPORTED otherwise); no workspace. */
VF4_API int vf4_attn_fp8(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                         int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, void* out,
                         int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s, vf4_stream_t stream);

/* bf16 attention: softmax(q k^T * scale) v with bf16 operands, fp32 accumulation and an exact
 * softmax -- the route the reference leaves to torch's scaled_dot_product_attention for blocks
 * kept in bf16 (ptq/qattention.py:20-30 falls through to the model's own attention when quant
 * attention is off; timm's Attention.forward calls F.scaled_dot_product_attention).  No
 * counterpart kernel in the reference.  Same operand / output layout and strides as
 * vf4_attn_nvfp4; head dim 64, S <= 288 and scale >= 0 (VF4_ERR_UNSUPPORTED otherwise); no workspace.
 * Up to S = 258 a two-slot kernel runs (the softmax of one 128-query tile overlapping the MMAs of
 * the next; the environment variable VF4_BF16_ATTN=tiles selects the single-slot kernel instead),
 * past that the single-slot kernel; both give the same arithmetic to fp32 rounding order.
 * out_amax (may be NULL): receives max |out| over the whole bf16 output -- the amax the next
 * QuantLinear's dynamic activation cast would compute (quant.py:48-54), so the caller can cast
 * with vf4_global_scale(out_amax) and skip that pass. */
VF4_API int vf4_attn_bf16(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                          int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, void* out,
                          int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s, float* out_amax,
                          vf4_stream_t stream);

/* vf4_attn_nvfp4 with options.  flags: VF4_ATTN_HEAD_GLOBALS takes the Q / K~ / V~ global scales per
 * (image, head) instead of over the whole tensors as the reference does: no statistics pass and,
 * for head dim 64 and S <= 320, no workspace at all (workspace may then be NULL), at the cost of
 * differing from the reference's quantization by independent FP4 noise (cos ~0.98 instead of
 * ~0.9999 against quant_sdpa).  0 = vf4_attn_nvfp4. */
#define VF4_ATTN_HEAD_GLOBALS 1
/* flags: VF4_ATTN_PACKED (head dim 64, S <= 320; ignored otherwise) quantizes the operands of every
 * head in a separate high-occupancy pass into per-head operand images in the workspace, which the
 * fused kernel then bulk-copies: same results as the default route (identical bits with tensor-wide
 * globals), faster, but the workspace grows by ~38 KB per (image, head) -- size it with
 * vf4_attn_workspace_size_ex(B, H, S, D, flags). */
#define VF4_ATTN_PACKED 2
/* flags: VF4_ATTN_NO_SMOOTH_K / VF4_ATTN_NO_SMOOTH_V switch off the reference's smooth-K (k minus its
 * token mean) / smooth-V (v minus its token mean, added back to the output), i.e. quant_sdpa(...,
 * smooth_k=False / smooth_v=False) of attention.py:53-54.  Only with the tensor-wide globals (not
 * with VF4_ATTN_HEAD_GLOBALS, which returns VF4_ERR_UNSUPPORTED). */
#define VF4_ATTN_NO_SMOOTH_K 4
#define VF4_ATTN_NO_SMOOTH_V 8

/* Operand precision of a route of vf4_attn (the reference's 'bf16' | 'fp8' | 'nvfp4'). */
#define VF4_ATTN_MODE_BF16 0
#define VF4_ATTN_MODE_FP8 1
#define VF4_ATTN_MODE_NVFP4 2
VF4_API int64_t vf4_attn_workspace_size_ex(int64_t B, int64_t H, int64_t S, int64_t D, int flags);
VF4_API int vf4_attn_nvfp4_ex(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S,
                              int64_t D, int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale,
                              void* out, int64_t out_stride_b, int64_t out_stride_h, int64_t out_stride_s,
                              int flags, void* workspace, int64_t workspace_bytes, vf4_stream_t stream);

/* quant_sdpa(q, k, v, scale=scale, qk=qk_mode, pv=pv_mode, smooth_k, smooth_v) of attention.py:53-86
 * (reached through _quant_attention, qattention.py:20-30) as one entry point: qk_mode / pv_mode are
 * VF4_ATTN_MODE_*, flags VF4_ATTN_NO_SMOOTH_K / _V switch smooth-K / smooth-V off (and, for the NVFP4
 * route, VF4_ATTN_HEAD_GLOBALS / VF4_ATTN_PACKED as vf4_attn_nvfp4_ex).  Kernel routes: nvfp4/nvfp4
 * (vf4_attn_nvfp4_ex), fp8/fp8 (E4M3 kernels: one fused kernel for head dim 64 and S <= 320, else a
 * prep kernel and a long-sequence kernel for head dims that are multiples of 16 up to 128 -- S up to
 * 1408 at head dim 80, 2304 at 64, 896 at 128), bf16/bf16 (vf4_attn_bf16, where smoothing changes no
 * result).  Mixed modes return VF4_ERR_UNSUPPORTED.  The NVFP4 route and the long-sequence FP8 route
 * need a workspace: size it with vf4_attn_workspace_size_modes (0 = none needed). */
VF4_API int vf4_attn(const void* q, const void* k, const void* v, int64_t B, int64_t H, int64_t S, int64_t D,
                     int64_t stride_b, int64_t stride_h, int64_t stride_s, float scale, int qk_mode, int pv_mode,
                     int flags, void* workspace, int64_t workspace_bytes, void* out, int64_t out_stride_b,
                     int64_t out_stride_h, int64_t out_stride_s, vf4_stream_t stream);
VF4_API int64_t vf4_attn_workspace_size_modes(int64_t B, int64_t H, int64_t S, int64_t D, int qk_mode, int pv_mode,
                                              int flags);

/* vf4_attn_nvfp4 without a caller workspace, for callers that cannot allocate device memory
 * (a runtime that owns all device memory through its own pool, or a plugin that may not
 * allocate or synchronize the device while it serves requests).  No counterpart in the
 * reference: the reference is Python and allocates freely.  The scratch is one fixed 16 MiB
 * device array inside the library (held on every GPU that loads it until exit): calls needing
 * more than vf4_attn_workspace_size(B,H,S,D) <= 16 MiB return VF4_ERR_UNSUPPORTED.  Its first
 * call on a device resolves the array's device address, so make that call before any stream
 * capture; all calls share the array, so calls that overlap on the GPU race.  Allocates nothing. */
VF4_API int vf4_attn_nvfp4_noalloc(const void* q, const void* k, const void* v, int64_t B, int64_t H,
                                   int64_t S, int64_t D, int64_t stride_b, int64_t stride_h,
                                   int64_t stride_s, float scale, void* out, int64_t out_stride_b,
                                   int64_t out_stride_h, int64_t out_stride_s, vf4_stream_t stream);

/* vf4_cast_nvfp4 (six rule, bf16) of an operand whose rows arrive in two parts per image: x_main
 * (n_img, rows_main, K) and x_tail (n_img, rows_tail, K), both contiguous; output row
 * i * (rows_main + rows_tail) + t takes main row t, then the tail rows follow.  gs NULL: dynamic
 * global over both parts into gs_out (the amax of the assembled tensor); otherwise gs is used.  Codes
 * and scales equal vf4_cast_nvfp4 of the assembled (n_img * (rows_main + rows_tail), K) tensor.  The
 * attention output of a query range split at a multiple of 128 (the bf16 route runs cuDNN on
 * queries [0, 128 k) and on the few remaining ones separately) goes to the proj GEMM this way
 * without being copied into one tensor.  No counterpart in the reference (its proj QuantLinear
 * casts the one SDPA output: nvfp4/gemm.py:32-38). */
VF4_API int vf4_cast_nvfp4_split(const void* x_main, int64_t rows_main, const void* x_tail, int64_t rows_tail,
                                 int64_t n_img, int64_t K, const float* gs, float* gs_out, uint8_t* out_packed,
                                 uint8_t* out_sf_swizzled, vf4_stream_t stream);

/* Token embedding of the ViT forward around the (bf16) patch-projection GEMM.  No kernel counterpart
 * in the reference: timm's PatchEmbed runs a strided Conv2d, then the model does
 * torch.cat([cls, patches]) + pos_embed (vit.py / timm VisionTransformer._pos_embed).
 * vf4_patchify: images (B, C, H, W) bf16 contiguous (W % 8 == 0, H and W multiples of p) ->
 *   out (B * (H/p) * (W/p), k_pad) bf16, row = one patch with its C*p*p values in (c, i, j) order
 *   (the Conv2d weight's flattening) and zeros up to k_pad (>= C*p*p, a multiple of 8).
 * vf4_embed_tokens: y (B, T-1, D) patch projections, cls (D,), pos (T, D) -> x (B, T, D) with
 *   x[:, 0] = cls + pos[0] and x[:, 1:] = y + pos[1:], each sum rounded once to bf16 (as cat + add). */
VF4_API int vf4_patchify(const void* images, int64_t B, int64_t C, int64_t H, int64_t W, int64_t p, int64_t k_pad,
                         void* out, vf4_stream_t stream);
VF4_API int vf4_embed_tokens(const void* y, const void* cls, const void* pos, int64_t B, int64_t T, int64_t D, void* x,
                             vf4_stream_t stream);

/* GPTQ column loop of one block of input columns (replaces the inner loop of gptq_quantize_weight,
 * src/vit_nvfp4/ptq/gptq.py:101-122; the caller keeps the Hessian preparation, gptq.py:79-94, and the
 * cross-block update W[:, i2:] -= Err @ Hinv[i1:i2, i2:], gptq.py:124-126).  For each row n < N of
 * the fp32 weight block w (columns col0 .. col0 + count of W, row stride ldw; read only) and the
 * block's upper inverse-Cholesky factor hinv (count x count, row stride ldh), columns i = 0..count-1
 * in order: code = E2M1 code of w_i / s, q = value(code) * s, err_i = (w_i - q) / hinv[i][i], and
 * w_c -= err_i * hinv[i][c] for c > i, with s = e4m3(block_scale[n][(col0 + i) / 16]) * global_scale
 * (block_scale: the frozen per-16 E4M3 bytes of the original weight, row stride ldb; global_scale one
 * fp32 on the device).  Writes codes[n][col0 + i] (uint8 E2M1 code of q / s, the reference's final
 * re-encoding; row stride ldc) and err[n][i] (fp32, row stride lde).  Divisions correctly rounded,
 * products rounded before the subtraction, as the reference's torch ops.  16 <= count <= 128 and
 * col0 multiples of 16. */
VF4_API int vf4_gptq_block(const float* w, int64_t ldw, const float* hinv, int64_t ldh, const uint8_t* block_scale,
                           int64_t ldb, const float* global_scale, int64_t N, int64_t col0, int64_t count,
                           uint8_t* codes, int64_t ldc, float* err, int64_t lde, vf4_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* VITFP4_H_ */
