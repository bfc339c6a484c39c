"""CPU oracle for the NVFP4 W4A4 ViT hot path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the ``vitfp4`` package,
its CUDA library or its C ABI) imports, links or executes this file.  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` leg use it, and only as the checker or the timed CPU
baseline.

It restates, in plain numpy float32 arithmetic, the algorithm of the
reference package (Dev-Jahn/vit-nvfp4, a pure-Python torch toolkit):

* E2M1 rounding / decoding ....... ``src/vit_nvfp4/nvfp4/format.py:17-33``
* two-level NVFP4 quantizer ...... ``src/vit_nvfp4/nvfp4/quant.py:6-76``
  (RTN "six" and Four-Over-Six "mse" block selection)
* nibble packing, SF swizzle ..... ``src/vit_nvfp4/nvfp4/pack.py:4-58``
* fp32-emulated GEMM ............. ``src/vit_nvfp4/nvfp4/backends/reference.py:6-10``
* FP8 per-row qdq ................ ``src/vit_nvfp4/nvfp4/fp8.py:6-17``
* emulated low-precision SDPA .... ``src/vit_nvfp4/nvfp4/attention.py:28-86``

Parity is PINNED: ``tests/golden/make_golden.py`` runs the reference itself
(imported from its source tree, in the build container) and stores its outputs
as fixtures; ``tests/test_oracle_golden.py`` checks this file against them
bit-for-bit (codes, scale bytes, global scales) and to fp32 tolerance (GEMM,
attention).

Arithmetic contract reproduced here (all fp32, IEEE, no fused multiply-add):
  gs      = max(amax|x|, 1e-12) / (6*448)   (six)   or / (6*256)  (mse)
  s_enc   = 1 / gs
  bs_f    = min((amax_b / D) * s_enc, 448)  D = 6 (and 4 for the FoS candidate)
  bs      = e4m3_rne(bs_f)
  dec     = float(bs) * gs
  code    = sign(q<0)<<3 | #{mid in (.25,.75,1.25,1.75,2.5,3.5,5) : mid < min(|q|,6)},
            q = x / dec, NaN -> index 7 (torch.bucketize puts NaN last)
  FoS     : pick 4 iff mean16((deq4-x)^2) < mean16((deq6-x)^2), the 16-term mean
            summed as p_i = e_i + e_{i+8} (i<8), then ((p0+p1)+p2)...+p7, / 16
            (the order ATen's vectorised CPU mean uses for a 16-wide row).
"""
from __future__ import annotations

import math

import numpy as np

E2M1_MAX = np.float32(6.0)
E4M3_MAX = np.float32(448.0)
FOS_SCALE_MAX = np.float32(256.0)
MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
MID = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
F32 = np.float32


# --------------------------------------------------------------------------
# E2M1 (format.py:17-33)
# --------------------------------------------------------------------------
def round_to_e2m1_code(q: np.ndarray) -> np.ndarray:
    """format.py:17-25 — ties go to the SMALLER magnitude, NaN -> index 7."""
    q = np.asarray(q, dtype=np.float32)
    sign = (q < 0).astype(np.uint8)
    m = np.minimum(np.abs(q), E2M1_MAX)          # NaN propagates like torch.clamp
    idx = np.zeros(q.shape, dtype=np.uint8)
    for t in MID:
        idx += (m > t).astype(np.uint8)           # bucketize(right=False): count mids < m
    idx = np.where(np.isnan(m), np.uint8(7), idx).astype(np.uint8)
    return ((sign << 3) | idx).astype(np.uint8)


def code_to_value(code: np.ndarray) -> np.ndarray:
    """format.py:28-33."""
    code = np.asarray(code).astype(np.int64)
    sign = F32(1.0) - F32(2.0) * ((code >> 3) & 1).astype(np.float32)
    return (sign * MAG[code & 7]).astype(np.float32)


# --------------------------------------------------------------------------
# FP8 E4M3 (float8_e4m3fn) round-to-nearest-even encode / decode
# --------------------------------------------------------------------------
def _e4m3_decode_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 7
        if e == 0xF and m == 7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * m * 2.0 ** -9
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_DECODE = _e4m3_decode_table()


def e4m3_decode(bits: np.ndarray) -> np.ndarray:
    return E4M3_DECODE[np.asarray(bits, dtype=np.uint8)]


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """fp32 -> float8_e4m3fn bits, round-to-nearest-even (torch ``.to(float8_e4m3fn)``).

    Finite magnitudes at or above 464 (the midpoint past 448) become NaN (0x7F/0xFF),
    as in torch; callers clamp to 448 first, as quant.py:12 does.
    """
    x = np.asarray(x, dtype=np.float32)
    xd = x.astype(np.float64)
    sign = np.where(np.signbit(x), 0x80, 0).astype(np.int64)
    a = np.abs(xd)
    out = np.zeros(x.shape, dtype=np.int64)
    sub = a < 2.0 ** -6
    # subnormals: multiples of 2^-9, RNE (np.rint is half-to-even); may round up to 2^-6
    ms = np.rint(a * 512.0).astype(np.int64)
    out = np.where(sub, ms, out)                 # ms == 8 is exactly code 0x08 (2^-6)
    # normals
    with np.errstate(divide="ignore", invalid="ignore"):
        _, ex = np.frexp(np.where(sub, 1.0, a))  # a = f*2^ex, f in [0.5,1)
    e = ex - 1
    sig = np.where(sub, 1.0, a) / np.ldexp(1.0, e)          # in [1,2), exact
    mn = np.rint((sig - 1.0) * 8.0).astype(np.int64)
    carry = mn == 8
    e = np.where(carry, e + 1, e)
    mn = np.where(carry, 0, mn)
    code_n = ((e + 7) << 3) | mn
    code_n = np.where(e + 7 > 15, 0x7F, code_n)
    code_n = np.where(code_n > 0x7E, 0x7F, code_n)          # >448 after rounding -> NaN
    out = np.where(sub, out, code_n)
    out = np.where(np.isnan(xd) | np.isinf(xd), 0x7F, out)
    return (out | sign).astype(np.uint8)


# --------------------------------------------------------------------------
# Two-level NVFP4 quantizer (quant.py:6-76)
# --------------------------------------------------------------------------
def global_scale_of(x: np.ndarray, block_select: str = "six") -> np.float32:
    """quant.py:48-53."""
    xf = np.asarray(x, dtype=np.float32)
    amax = F32(np.max(np.abs(xf))) if xf.size else F32(0.0)
    amax = max(amax, F32(1e-12))
    denom = FOS_SCALE_MAX if block_select == "mse" else E4M3_MAX
    return F32(amax / F32(E2M1_MAX * denom))


def _encode_block(xb, amax_b, divisor, s_enc, gs):
    """quant.py:6-17."""
    bs_f = np.minimum((amax_b / F32(divisor)) * s_enc, E4M3_MAX)
    bse = e4m3_encode(bs_f)
    dec = e4m3_decode(bse) * gs
    with np.errstate(divide="ignore", invalid="ignore"):
        codes = round_to_e2m1_code(xb / dec)
    deq = code_to_value(codes) * dec
    return codes, bse, deq


def mean16_aten(e: np.ndarray) -> np.ndarray:
    """16-term mean along the last axis in ATen's vectorised CPU order."""
    assert e.shape[-1] == 16
    p = (e[..., :8] + e[..., 8:]).astype(np.float32)
    s = p[..., 0]
    for i in range(1, 8):
        s = (s + p[..., i]).astype(np.float32)
    return (s / F32(16.0)).astype(np.float32)


def quantize_to_nvfp4(x, block: int = 16, global_scale=None, block_select: str = "six"):
    """quant.py:20-69.  Returns (codes uint8 (...,K), bs e4m3 BITS uint8 (...,K/16), gs float32)."""
    x = np.asarray(x)
    assert x.shape[-1] % block == 0 and block == 16
    assert block_select in ("six", "mse")
    xf = x.astype(np.float32)
    gs = global_scale_of(xf, block_select) if global_scale is None else F32(global_scale)
    s_enc = F32(F32(1.0) / gs)
    xb = xf.reshape(*xf.shape[:-1], xf.shape[-1] // block, block)
    amax_b = np.maximum(np.abs(xb).max(axis=-1, keepdims=True), F32(1e-12)).astype(np.float32)
    c6, b6, d6 = _encode_block(xb, amax_b, 6.0, s_enc, gs)
    if block_select == "six":
        codes, bse = c6, b6
    else:
        c4, b4, d4 = _encode_block(xb, amax_b, 4.0, s_enc, gs)
        e4 = ((d4 - xb) ** 2).astype(np.float32)
        e6 = ((d6 - xb) ** 2).astype(np.float32)
        pick4 = (mean16_aten(e4) < mean16_aten(e6))[..., None]
        codes = np.where(pick4, c4, c6)
        bse = np.where(pick4, b4, b6)
    return codes.reshape(x.shape).astype(np.uint8), bse[..., 0].astype(np.uint8), gs


def dequantize_nvfp4(codes, bs_bits, gs):
    """quant.py:72-76 (block scale given as e4m3 bits)."""
    codes = np.asarray(codes)
    nb = bs_bits.shape[-1]
    blk = codes.shape[-1] // nb
    vals = code_to_value(codes).reshape(*codes.shape[:-1], nb, blk)
    scale = (e4m3_decode(bs_bits) * F32(gs))[..., None]
    return (vals * scale).reshape(codes.shape).astype(np.float32)


# --------------------------------------------------------------------------
# Packing and the 128x4 scale-factor swizzle (pack.py:4-58)
# --------------------------------------------------------------------------
def pack_e2m1(codes):
    """pack.py:4-9 — low nibble = even index, high nibble = odd index."""
    codes = np.asarray(codes, dtype=np.uint8)
    return ((codes[..., 1::2] << 4) | codes[..., 0::2]).astype(np.uint8)


def unpack_e2m1(packed):
    """pack.py:12-16."""
    packed = np.asarray(packed, dtype=np.uint8)
    out = np.stack([packed & 0xF, (packed >> 4) & 0xF], axis=-1)
    return out.reshape(*packed.shape[:-1], packed.shape[-1] * 2).astype(np.uint8)


def to_blocked(sf):
    """pack.py:39-58: pad to (ceil128(R), ceil4(C)); tile (rb,cb) at (rb*nCB+cb)*512;
    inside a tile element (r,c) at (r%32)*16 + (r//32)*4 + c."""
    sf = np.asarray(sf)
    R, C = sf.shape
    nrb, ncb = -(-R // 128), -(-C // 4)
    pad = np.zeros((nrb * 128, ncb * 4), dtype=sf.dtype)
    pad[:R, :C] = sf
    blocks = pad.reshape(nrb, 128, ncb, 4).transpose(0, 2, 1, 3)           # (rb, cb, 128, 4)
    out = blocks.reshape(-1, 4, 32, 4).transpose(0, 2, 1, 3).reshape(-1)   # (tile, r%32, r//32, c)
    return np.ascontiguousarray(out)


def from_blocked(flat, R, C):
    """Inverse of :func:`to_blocked` (drops the padding)."""
    nrb, ncb = -(-R // 128), -(-C // 4)
    t = np.asarray(flat).reshape(nrb, ncb, 32, 4, 4).transpose(0, 1, 3, 2, 4)  # (rb,cb,r//32,r%32,c)
    t = t.reshape(nrb, ncb, 128, 4).transpose(0, 2, 1, 3).reshape(nrb * 128, ncb * 4)
    return np.ascontiguousarray(t[:R, :C])


# --------------------------------------------------------------------------
# GEMM oracle (backends/reference.py:6-10)
# --------------------------------------------------------------------------
def gemm_reference(a_codes, a_bs, a_gs, b_codes, b_bs, b_gs):
    """fp32 emulated NVFP4 GEMM: dequant(A) @ dequant(B).T, A:(M,K), B:(N,K)."""
    a = dequantize_nvfp4(a_codes, a_bs, a_gs)
    b = dequantize_nvfp4(b_codes, b_bs, b_gs)
    return (a @ b.T).astype(np.float32)


# --------------------------------------------------------------------------
# The Triton cast (nvfp4/triton_cast.py:138-370): the reference's fused-MLP casts
# --------------------------------------------------------------------------
E4M3_EPS = F32(1.5258789e-05)      # triton_cast.py:247, the lower clamp of a block scale


def e2m1_code_rne(q: np.ndarray) -> np.ndarray:
    """E2M1 code of q with nearest-even rounding (the hardware fp32 -> fp4 conversion the Triton
    cast uses, triton_cast.py:343): ties at 0.75, 1.75 and 3.5 go UP to the even code, the other
    ties (0.25, 1.25, 2.5, 5.0) down; the sign bit is q's (so -0.0 -> code 8)."""
    q = np.asarray(q, dtype=np.float32)
    m = np.minimum(np.abs(q), E2M1_MAX)
    idx = np.zeros(q.shape, dtype=np.uint8)
    for mid in MID:
        idx += (m > mid).astype(np.uint8)
    idx += np.isin(m, np.array([0.75, 1.75, 3.5], np.float32)).astype(np.uint8)
    return (np.signbit(q).astype(np.uint8) << 3) | idx


def triton_cast_nvfp4(x, per_tensor_scale, apply_gelu: bool = False):
    """cast_nvfp4 (triton_cast.py:138-233, kernel :235-370; E4M3 scales, precise math):
    g = 1 / per_tensor_scale (:163); optional fp32 erf-GELU first (:302-303); per 16-block
    scale = e4m3(clamp(RN(amax / 6) * g, 2^-16, 448)) (:318-322); q = x * RN(g / scale) (:327-331);
    nearest-even E2M1.  Returns (codes (M, K) uint8, scale bytes (M, K/16) uint8)."""
    xf = np.asarray(x, dtype=np.float32)
    if apply_gelu:
        xf = gelu(xf)
    g = F32(1.0) / F32(per_tensor_scale)
    blocks = xf.reshape(*xf.shape[:-1], xf.shape[-1] // 16, 16)
    amax = np.abs(blocks).max(axis=-1)
    sc = np.clip((amax / F32(6.0)).astype(np.float32) * g, E4M3_EPS, E4M3_MAX).astype(np.float32)
    s8 = e4m3_encode(sc)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        total = (g / e4m3_decode(s8)).astype(np.float32)
        q = (blocks * total[..., None]).astype(np.float32)
    return e2m1_code_rne(q).reshape(xf.shape), s8


# --------------------------------------------------------------------------
# bf16 rounding, GELU, FP8 qdq, emulated SDPA
# --------------------------------------------------------------------------
def to_bf16(x) -> np.ndarray:
    """fp32 -> bf16 (round-to-nearest-even), returned widened back to fp32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u >> 16) & 1) + 0x7FFF
    v = ((u + r) & 0xFFFF0000).astype(np.uint32)
    v = np.where(np.isnan(x), np.uint32(0x7FC00000), v)
    return v.view(np.float32)


def bf16_bits(x) -> np.ndarray:
    return (to_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint32) << 16).view(np.float32)


def _erf(x):
    try:
        from scipy.special import erf
        return erf(x.astype(np.float64)).astype(np.float32)
    except ImportError:  # pragma: no cover - scipy ships with the image
        return np.vectorize(math.erf)(x.astype(np.float64)).astype(np.float32)


def gelu(x):
    """Exact erf GELU: 0.5*x*(1+erf(x/sqrt 2))."""
    x = np.asarray(x, dtype=np.float32)
    return (F32(0.5) * x * (F32(1.0) + _erf(x * F32(0.7071067811865476)))).astype(np.float32)


def fp8_e4m3_quant_dequant(x):
    """fp8.py:6-17 — per-row amax/448 scale, RNE to e4m3, back to fp32."""
    xf = np.asarray(x, dtype=np.float32)
    amax = np.maximum(np.abs(xf).max(axis=-1, keepdims=True), F32(1e-12))
    scale = (amax / E4M3_MAX).astype(np.float32)
    q = np.clip(xf / scale, -E4M3_MAX, E4M3_MAX).astype(np.float32)
    return (e4m3_decode(e4m3_encode(q)) * scale).astype(np.float32)


def nvfp4_qdq(x, block: int = 16):
    """attention.py:28-36 — NVFP4 round trip along the last dim, zero-padded to 16."""
    x = np.asarray(x, dtype=np.float32)
    k = x.shape[-1]
    pad = (-k) % block
    if pad:
        x = np.concatenate([x, np.zeros((*x.shape[:-1], pad), np.float32)], axis=-1)
    c, b, g = quantize_to_nvfp4(x, block)
    d = dequantize_nvfp4(c, b, g)
    return d[..., :k] if pad else d


def _qdq(x, mode, axis=-1):
    """attention.py:39-50."""
    if mode == "bf16":
        return to_bf16(x)
    if axis not in (-1, x.ndim - 1):
        return np.swapaxes(_qdq(np.ascontiguousarray(np.swapaxes(x, axis, -1)), mode, -1), axis, -1)
    if mode == "fp8":
        return fp8_e4m3_quant_dequant(x)
    if mode == "nvfp4":
        return nvfp4_qdq(x)
    raise ValueError(mode)


def softmax(s):
    s = np.asarray(s, dtype=np.float32)
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m).astype(np.float32)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def quant_sdpa(q, k, v, scale=None, qk="nvfp4", pv="nvfp4", smooth_k=True, smooth_v=True,
               is_causal=False):
    """attention.py:53-86 (no mask / dropout; optional causal)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    D = q.shape[-1]
    scale = F32(1.0 / math.sqrt(D)) if scale is None else F32(scale)
    if smooth_k:
        k = (k - k.mean(axis=-2, keepdims=True)).astype(np.float32)
    s = (_qdq(q, qk) @ np.swapaxes(_qdq(k, qk), -1, -2)).astype(np.float32) * scale
    if is_causal:
        Sq, Sk = s.shape[-2], s.shape[-1]
        mask = np.tril(np.ones((Sq, Sk), bool), Sk - Sq)
        s = np.where(mask, s, -np.inf).astype(np.float32)
    p = softmax(s)
    mu = None
    if smooth_v:
        mu = v.mean(axis=-2, keepdims=True).astype(np.float32)
        v = (v - mu).astype(np.float32)
    out = (_qdq(p, pv, -1) @ _qdq(v, pv, -2)).astype(np.float32)
    if mu is not None:
        out = (out + mu).astype(np.float32)
    return out
