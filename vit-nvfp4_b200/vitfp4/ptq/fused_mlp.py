"""Fused NVFP4 W4A4 transformer MLP ``fc1 -> GELU -> fc2`` (reference:
src/vit_nvfp4/ptq/fused_mlp.py:25-167).

The fc1 GEMM's epilogue applies ``+b1 -> GELU -> NVFP4 cast`` straight from the TMEM
accumulator, so the (M, 4d) intermediate never round-trips HBM in bf16; fc2 consumes the packed
FP4 codes + swizzled scales directly and adds ``b2`` in its epilogue.  Three kernels per MLP:
activation cast, fc1 GEMM (fused epilogue), fc2 GEMM (bias epilogue).  The epilogue's GELU is the tanh form evaluated with the hardware tanh by default (its
deviation from erf-GELU, ~1e-3 at most, is below the bf16 rounding the reference applies to the fc1
output before its GELU); ``exact_gelu=True`` selects an erf-GELU epilogue accurate to 1.5e-7.

Buffers and calibration follow the reference: weights are quantized once with the RTN "six"
rule and stored packed (``float4_e2m1fn_x2``) with swizzled E4M3 scales; the activation globals
``gx`` / ``gh`` (amax/(6*448)) are frozen on the first forward.
"""
from __future__ import annotations

import warnings

import torch
import torch.nn as nn

from ..nvfp4 import ops


def _global_scale(t: torch.Tensor, gelu: bool = False) -> torch.Tensor:
    """amax / (6*448) of t (of GELU(t) when ``gelu``); 1.0 for an empty tensor."""
    if t.numel() == 0:
        return torch.ones((), device=t.device, dtype=torch.float32)
    return ops.global_scale(ops.amax(t, gelu=gelu), "six")


def _quant_weight(linear: nn.Linear):
    w = linear.weight.data
    g = _global_scale(w)
    packed, sf, _, _ = ops.cast(w.to(torch.bfloat16), g, "six")
    sf2 = sf.view(-1, ((w.shape[1] // 16) + 3) // 4 * 4)
    return packed.view(torch.float4_e2m1fn_x2), sf2.view(torch.float8_e4m3fn), g


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


@torch.library.custom_op("vitfp4::fused_mlp", mutates_args=())
def fused_mlp_op(x: torch.Tensor, w1q: torch.Tensor, w1sf: torch.Tensor, w1g: torch.Tensor,
                 b1: torch.Tensor | None, w2q: torch.Tensor, w2sf: torch.Tensor, w2g: torch.Tensor,
                 b2: torch.Tensor | None, gx: torch.Tensor, gh: torch.Tensor, k1: int, n2: int,
                 exact_gelu: bool = False) -> torch.Tensor:
    M = x.numel() // k1
    x2 = x.reshape(M, k1)
    ap, asf, _, _ = ops.cast(x2, gx, "six")
    hp, hsf = ops.gemm_gelu_nvfp4(ap, asf, gx, _u8(w1q), _u8(w1sf), w1g, b1, gh, exact=exact_gelu)
    y = ops.gemm(hp, hsf, gh, _u8(w2q), _u8(w2sf), w2g, bias=b2, out_dtype=torch.bfloat16)
    return y.reshape(*x.shape[:-1], n2)


@fused_mlp_op.register_fake
def _(x, w1q, w1sf, w1g, b1, w2q, w2sf, w2g, b2, gx, gh, k1, n2, exact_gelu=False):
    return x.new_empty(*x.shape[:-1], n2, dtype=torch.bfloat16)


class FusedNVFP4MLP(nn.Module):
    """Drop-in replacement for a ``fc1 -> GELU -> fc2`` MLP with NVFP4 W4A4 and GELU fusion."""

    def __init__(self, fc1: nn.Linear, fc2: nn.Linear, exact_gelu: bool = False):
        super().__init__()
        self.exact_gelu = exact_gelu
        assert fc1.out_features == fc2.in_features, "not an fc1->fc2 MLP pair"
        assert fc1.in_features > 0 and fc1.in_features % 16 == 0 and fc2.in_features % 16 == 0, \
            "NVFP4 needs K > 0 and K % 16 == 0"
        assert fc1.weight.is_cuda, "FusedNVFP4MLP requires CUDA weights (sm_100a kernels)"
        w1q, w1sf, w1g = _quant_weight(fc1)
        w2q, w2sf, w2g = _quant_weight(fc2)
        self.register_buffer("w1q", w1q)
        self.register_buffer("w1sf", w1sf)
        self.register_buffer("w1g", w1g)
        self.register_buffer("w2q", w2q)
        self.register_buffer("w2sf", w2sf)
        self.register_buffer("w2g", w2g)
        self.register_buffer("b1", None if fc1.bias is None else fc1.bias.detach().to(torch.bfloat16))
        self.register_buffer("b2", None if fc2.bias is None else fc2.bias.detach().to(torch.bfloat16))
        self.k1 = fc1.in_features
        self.n2 = fc2.out_features
        self.register_buffer("gx", None)
        self.register_buffer("gh", None)

    @torch.no_grad()
    def _calibrate(self, x: torch.Tensor) -> None:
        x2 = x.reshape(-1, self.k1).to(torch.bfloat16)
        gx = _global_scale(x2)
        ap, asf, _, _ = ops.cast(x2, gx, "six")
        y1 = ops.gemm(ap, asf, gx, _u8(self.w1q), _u8(self.w1sf), self.w1g, bias=self.b1)
        self.gx = gx
        self.gh = _global_scale(y1, gelu=True)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.gx is None:
            self._calibrate(x)
        return fused_mlp_op(x.to(torch.bfloat16) if x.dtype != torch.bfloat16 else x,
                            self.w1q, self.w1sf, self.w1g, self.b1, self.w2q, self.w2sf, self.w2g,
                            self.b2, self.gx, self.gh, self.k1, self.n2, self.exact_gelu)

    def extra_repr(self) -> str:
        return f"in={self.k1}, hidden={self.w1q.shape[0]}, out={self.n2}, nvfp4=W4A4+gelu_fused"


# activation class names: exact erf-GELU (fusable) vs approximations (never fused)
_EXACT_GELU = {"GELUActivation"}
_APPROX_GELU = {"PytorchGELUTanh", "NewGELUActivation", "QuickGELUActivation", "FastGELUActivation",
                "GELUTanh", "ClippedGELUActivation"}


def _is_exact_gelu(module: nn.Module):
    """True: exact GELU child; False: known approximation; None: no activation found."""
    for child in module.children():
        cname = type(child).__name__
        if cname in _EXACT_GELU:
            return True
        if cname in _APPROX_GELU:
            return False
        if isinstance(child, nn.GELU):
            return child.approximate == "none"
    return None


def _mlp_pair(module: nn.Module):
    """(fc1, fc2) of a plain fc1->act->fc2 MLP, else None (gated MLPs are never pairs)."""
    if getattr(module, "gate_proj", None) is not None:
        return None
    for up, down in (("fc1", "fc2"), ("up_proj", "down_proj")):
        f1, f2 = getattr(module, up, None), getattr(module, down, None)
        if isinstance(f1, nn.Linear) and isinstance(f2, nn.Linear) and f1.out_features == f2.in_features \
                and f1.in_features % 16 == 0:
            return f1, f2
    return None


def fuse_mlps(model: nn.Module, skip_ends: int = 2, require_gelu: bool = True) -> int:
    """Swap each block's GELU MLP for FusedNVFP4MLP in place; returns the number fused.

    ``skip_ends`` leaves the first/last N fusible MLPs in bf16; ``require_gelu`` fuses only
    MLPs whose activation is confirmed exact erf-GELU (others stay bf16 with a warning)."""
    cands = [(n, m, p) for n, m in model.named_modules() if (p := _mlp_pair(m)) is not None]
    if require_gelu:
        unsure = [n for n, m, _ in cands if _is_exact_gelu(m) is not True]
        if unsure:
            warnings.warn(f"fuse_mlps: leaving {len(unsure)} MLP(s) in BF16 — activation not confirmed "
                          f"exact GELU (e.g. {unsure[:3]}). Pass require_gelu=False to force.")
        cands = [(n, m, p) for n, m, p in cands if _is_exact_gelu(m) is True]
    if skip_ends and 2 * skip_ends >= len(cands):
        raise ValueError(f"skip_ends={skip_ends} too large for {len(cands)} fusible MLP block(s)")
    keep = cands[skip_ends:len(cands) - skip_ends] if skip_ends else cands
    for name, _m, pair in keep:
        parent_name, _, attr = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, attr, FusedNVFP4MLP(*pair))
    return len(keep)
