"""W4A4 NVFP4 GEMM / linear entry points (reference: src/vit_nvfp4/nvfp4/gemm.py:12-38 and
backends/torch_scaled_mm.py:14-46, triton_cast.py:138).

There is one implementation: the tcgen05 block-scaled FP4 GEMM of libvitfp4.so.  The
reference's backend ladder is kept as an API (``backend=`` is accepted, ``register_backend``
records callables) but ``nvfp4_gemm`` always runs the CUDA kernel unless a caller explicitly
names a backend it registered itself.
"""
from __future__ import annotations

import torch

from . import ops
from .quant import quantize_to_nvfp4

_BACKENDS: dict = {}
_NATIVE = "vitfp4_sm100a"


def register_backend(name, fn):
    _BACKENDS[name] = fn


def available_backends():
    return [_NATIVE, *_BACKENDS]


def _default_backend():
    return _NATIVE


def _packed_operand(codes: torch.Tensor, bs: torch.Tensor):
    """Unpacked codes (R, K) + row-major E4M3 scales (R, K/16) -> (packed, swizzled scales)."""
    c2 = codes.reshape(-1, codes.shape[-1])
    b2 = bs.reshape(-1, bs.shape[-1])
    return ops.pack_e2m1(c2), ops.to_blocked(b2)


def nvfp4_gemm(a_codes, a_bs, a_gs, b_codes, b_bs, b_gs, *, out_dtype=torch.bfloat16, backend=None):
    """A:(M,K) codes x B:(N,K) codes -> (M,N). Packs + swizzles both operands, then one GEMM."""
    if backend not in (None, _NATIVE):
        return _BACKENDS[backend](a_codes, a_bs, a_gs, b_codes, b_bs, b_gs, out_dtype=out_dtype)
    ap, asf = _packed_operand(a_codes, a_bs)
    bp, bsf = _packed_operand(b_codes, b_bs)
    return ops.gemm(ap, asf, a_gs, bp, bsf, b_gs, out_dtype=out_dtype)


def gemm_packed(a_fp4, a_sf, a_g, w_fp4, w_sf, w_g, out_dtype=torch.bfloat16):
    """W4A4 GEMM on operands already packed (M,K/2)/(N,K/2) with swizzled E4M3 scales."""
    return ops.gemm(a_fp4, a_sf, a_g, w_fp4, w_sf, w_g, out_dtype=out_dtype)


@torch.library.custom_op("vitfp4::cast_nvfp4", mutates_args=())
def cast_nvfp4_op(x: torch.Tensor, gs: torch.Tensor, apply_gelu: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(M, K) -> packed codes (M, K/2) uint8 and the 128x4-tiled scales (ceil128(M), ceil4(K/16)) uint8."""
    K = x.shape[-1]
    packed, sf, _, _ = ops.cast(x, gs, "six", gelu=apply_gelu)
    return packed, sf.view(-1, ((K // 16) + 3) // 4 * 4)


@cast_nvfp4_op.register_fake
def _(x, gs, apply_gelu):
    K = x.shape[-1]
    M = x.numel() // K
    return (x.new_empty((M, K // 2), dtype=torch.uint8),
            x.new_empty(((M + 127) // 128 * 128, ((K // 16) + 3) // 4 * 4), dtype=torch.uint8))


def cast_nvfp4(x: torch.Tensor, per_tensor_scale: torch.Tensor | None, apply_gelu: bool = False,
               use_e8m0_scale: bool = False, use_precise_math: bool = True):
    """Fused single-pass NVFP4 cast (optionally GELU first) -> (qdata float4_e2m1fn_x2, swizzled scale).

    Same contract as the reference's Triton cast_nvfp4 (triton_cast.py:138-233): ``per_tensor_scale`` is
    the decode global (``amax/(6*448)``), None means 1.0; the scale comes back 2-D (ceil128(M),
    ceil4(K/16)).  The block arithmetic is the reference quantizer's (quant.py), not the Triton
    kernel's.  A ``torch.library`` custom op (``vitfp4::cast_nvfp4``), so torch.compile traces around it.
    """
    if use_e8m0_scale:
        raise NotImplementedError("E8M0 scales are not part of the NVFP4 path")
    K = x.shape[-1]
    gs = per_tensor_scale if per_tensor_scale is not None else torch.ones((), device=x.device)
    packed, sf = cast_nvfp4_op(x.reshape(-1, K), gs.reshape(()).float(), bool(apply_gelu))
    return (packed.view(*x.shape[:-1], K // 2).view(torch.float4_e2m1fn_x2), sf.view(torch.float8_e4m3fn))


def nvfp4_linear(x, w_codes, w_bs, w_gs, *, x_global_scale=None, bias=None, backend=None):
    """W4A4 linear: online NVFP4 cast of x (six rule), FP4 GEMM, + bias; output in x.dtype."""
    if backend not in (None, _NATIVE):
        xc, xb, xg = quantize_to_nvfp4(x, 16, global_scale=x_global_scale)
        y = _BACKENDS[backend](xc, xb, xg, w_codes, w_bs, w_gs, out_dtype=x.dtype)
        return y if bias is None else y + bias.to(y.dtype)
    wp, wsf = _packed_operand(w_codes, w_bs)
    return linear_packed(x, wp, wsf, w_gs, x_global_scale=x_global_scale, bias=bias)


def linear_packed(x, w_packed, w_sf, w_gs, *, x_global_scale=None, bias=None):
    """nvfp4_linear with the weight already packed + swizzled (the QuantLinear fast path)."""
    K = x.shape[-1]
    ap, asf, _, ag = ops.cast(x, x_global_scale, "six")
    out_dtype = x.dtype if x.dtype in (torch.float32, torch.bfloat16) else torch.float32
    y = ops.gemm(ap, asf, ag, w_packed, w_sf, w_gs, bias=bias, out_dtype=out_dtype)
    y = y.reshape(*x.shape[:-1], w_packed.shape[0])
    return y if y.dtype == x.dtype else y.to(x.dtype)
