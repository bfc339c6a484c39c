"""Fused NVFP4 W4A4 transformer MLP ``fc1 -> GELU -> fc2`` (reference:
src/vit_nvfp4/ptq/fused_mlp.py:25-167).

The fc1 GEMM's epilogue applies ``+b1 -> GELU -> NVFP4 cast`` straight from the TMEM
accumulator, so the (M, 4d) intermediate never round-trips HBM in bf16; fc2 consumes the packed
FP4 codes + swizzled scales directly and adds ``b2`` in its epilogue.  Three kernels per MLP:
activation cast, fc1 GEMM (fused epilogue), fc2 GEMM (bias epilogue).

The epilogue computes what the reference's unfused steps compute: the fc1 result rounded to bf16,
``+ b1`` in bf16, then erf-GELU in fp32 on that bf16 value and the NVFP4 cast of the fp32 GELU
(the reference's Triton cast with ``apply_gelu``).  ``exact_gelu=False`` selects the cheaper
tanh-form GELU on the unrounded accumulator instead (within ~1e-3 of erf-GELU).

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
                 exact_gelu: bool = True, w2img: torch.Tensor | None = None) -> torch.Tensor:
    M = x.numel() // k1
    x2 = x.reshape(M, k1)
    ap, asf, _, _ = ops.cast(x2, gx, "six")
    hp, hsf = ops.gemm_gelu_nvfp4(ap, asf, gx, _u8(w1q), _u8(w1sf), w1g, b1, gh, exact=exact_gelu)
    y = ops.gemm(hp, hsf, gh, _u8(w2q), _u8(w2sf), w2g, bias=b2, out_dtype=torch.bfloat16, b_image=w2img)
    return y.reshape(*x.shape[:-1], n2)


@fused_mlp_op.register_fake
def _(x, w1q, w1sf, w1g, b1, w2q, w2sf, w2g, b2, gx, gh, k1, n2, exact_gelu=True, w2img=None):
    return x.new_empty(*x.shape[:-1], n2, dtype=torch.bfloat16)


class FusedNVFP4MLP(nn.Module):
    """Drop-in replacement for a ``fc1 -> GELU -> fc2`` MLP with NVFP4 W4A4 and GELU fusion."""

    def __init__(self, fc1: nn.Linear, fc2: nn.Linear, exact_gelu: bool = True):
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
        self._w2img = None       # (w2sf version stamp, B scale image of w2sf): derived, not saved

    def w2_image(self) -> torch.Tensor:
        """fc2's B scale image (``ops.b_scale_image`` of w2sf), rebuilt when w2sf moves, is written in
        place (tracked by its version counter; inference tensors have none) or is loaded from a
        state_dict."""
        try:
            version = self.w2sf._version
        except RuntimeError:
            version = None
        stamp = (self.w2sf.data_ptr(), version, self.w2sf.device)
        if self._w2img is None or self._w2img[0] != stamp:
            self._w2img = (stamp, ops.b_scale_image(self.w2sf, self.n2, self.w2q.shape[1] * 2))
        return self._w2img[1]

    def _load_from_state_dict(self, *args, **kwargs):
        self._w2img = None
        super()._load_from_state_dict(*args, **kwargs)

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
                            self.b2, self.gx, self.gh, self.k1, self.n2, self.exact_gelu, self.w2_image())

    def extra_repr(self) -> str:
        return f"in={self.k1}, hidden={self.w1q.shape[0]}, out={self.n2}, nvfp4=W4A4+gelu_fused"


# Activation modules by what they compute.  The fused epilogue applies erf-GELU, so only an MLP
# whose activation is known to be erf-GELU computes the same function after fusion.
_ERF_GELU_CLASSES = frozenset({"GELUActivation"})
_APPROXIMATE_GELU_CLASSES = frozenset({"PytorchGELUTanh", "NewGELUActivation", "QuickGELUActivation",
                                       "FastGELUActivation", "GELUTanh", "ClippedGELUActivation"})


def _activation_kind(mlp: nn.Module) -> str:
    """"erf", "approximate" or "unknown": the first direct child that is a recognised activation
    decides (torch's nn.GELU by its ``approximate`` flag, HF activations by class name)."""
    for child in mlp.children():
        if isinstance(child, nn.GELU):
            return "erf" if child.approximate == "none" else "approximate"
        tname = type(child).__name__
        if tname in _ERF_GELU_CLASSES:
            return "erf"
        if tname in _APPROXIMATE_GELU_CLASSES:
            return "approximate"
    return "unknown"


def _fc_pair(mlp: nn.Module):
    """(fc1, fc2) of an ungated two-Linear MLP whose shapes chain and whose input width is a
    multiple of 16 (timm ``fc1/fc2`` or HF ``up_proj/down_proj`` names), else None."""
    if getattr(mlp, "gate_proj", None) is not None:     # gated (SwiGLU-style) MLPs have no fc1->act->fc2 form
        return None
    for up_name, down_name in (("fc1", "fc2"), ("up_proj", "down_proj")):
        up, down = getattr(mlp, up_name, None), getattr(mlp, down_name, None)
        if not (isinstance(up, nn.Linear) and isinstance(down, nn.Linear)):
            continue
        if up.out_features == down.in_features and up.in_features % 16 == 0:
            return up, down
    return None


def plan_mlp_fusion(model: nn.Module, skip_ends: int = 2, require_gelu: bool = True) -> list:
    """The MLPs ``fuse_mlps`` would replace, as (dotted name, fc1, fc2) in module order.

    Pure module-tree inspection (no CUDA): every ungated fc1->act->fc2 MLP is a candidate; with
    ``require_gelu`` only those whose activation is known erf-GELU stay candidates (a warning names
    the others); then ``skip_ends`` candidates are dropped from each end of the list."""
    found = []
    for name, mod in model.named_modules():
        pair = _fc_pair(mod)
        if pair is not None:
            found.append((name, mod, pair))
    if require_gelu:
        left_out = [name for name, mod, _ in found if _activation_kind(mod) != "erf"]
        if left_out:
            warnings.warn(f"fuse_mlps: {len(left_out)} MLP(s) stay in bf16 because their activation is not "
                          f"known to be erf-GELU (first: {left_out[:3]}); require_gelu=False fuses them anyway")
        found = [entry for entry in found if _activation_kind(entry[1]) == "erf"]
    if skip_ends:
        if 2 * skip_ends >= len(found):
            raise ValueError(f"fuse_mlps: skip_ends={skip_ends} leaves nothing of {len(found)} fusible MLP(s)")
        found = found[skip_ends:-skip_ends]
    return [(name, pair[0], pair[1]) for name, _, pair in found]


def fuse_mlps(model: nn.Module, skip_ends: int = 2, require_gelu: bool = True, exact_gelu: bool = True) -> int:
    """Replace the MLPs chosen by ``plan_mlp_fusion`` with ``FusedNVFP4MLP`` in place; returns how
    many were replaced (reference: src/vit_nvfp4/ptq/fused_mlp.py:143-167)."""
    plan = plan_mlp_fusion(model, skip_ends, require_gelu)
    for name, fc1, fc2 in plan:
        model.set_submodule(name, FusedNVFP4MLP(fc1, fc2, exact_gelu=exact_gelu))
    return len(plan)
