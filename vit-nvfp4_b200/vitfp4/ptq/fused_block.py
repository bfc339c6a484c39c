"""Fused timm / DINOv2-style transformer block for the W4A4 path.

A converted block (``norm1 -> attn{qkv: QuantLinear, proj: QuantLinear} -> ls1 -> +x -> norm2 ->
mlp: FusedNVFP4MLP -> ls2 -> +x``) spends most of its non-GEMM time in bf16 LayerNorm,
LayerScale, residual adds and the activation casts that follow them.  ``FusedNVFP4Block`` runs the
same computation with those steps fused:

  norm1 + dynamic NVFP4 cast ............ one kernel pair (amax pass, quantize pass)
  qkv GEMM (+bias) -> attention -> proj QuantLinear (cast + GEMM + bias)
  x + ls1(proj) + norm2 + static cast .... one kernel (residual written once, normalised rows
                                           quantized with the MLP's calibrated gx)
  fc1 GEMM (+b1 -> GELU -> NVFP4 epilogue) -> fc2 GEMM (+b2 -> *ls2 -> +x epilogue)

Numerics follow the unfused modules (bf16 rounding after LayerScale, after the residual add and
after LayerNorm); only the kernels change.  ``fuse_norms`` converts every eligible block in place.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..nvfp4 import ops
from .fused_mlp import FusedNVFP4MLP, _u8
from .qlinear import QuantLinear


def _gamma(ls: nn.Module):
    return getattr(ls, "gamma", None) if not isinstance(ls, nn.Identity) else None


class FusedNVFP4Block(nn.Module):
    def __init__(self, block: nn.Module):
        super().__init__()
        self.norm1, self.attn, self.ls1 = block.norm1, block.attn, block.ls1
        self.norm2, self.mlp, self.ls2 = block.norm2, block.mlp, block.ls2

    @staticmethod
    def eligible(block: nn.Module) -> bool:
        attn = getattr(block, "attn", None)
        return (not isinstance(block, FusedNVFP4Block) and isinstance(getattr(block, "norm1", None), nn.LayerNorm) and isinstance(getattr(block, "norm2", None), nn.LayerNorm)
                and attn is not None and isinstance(getattr(attn, "qkv", None), QuantLinear)
                and isinstance(getattr(attn, "proj", None), QuantLinear) and isinstance(getattr(block, "mlp", None), FusedNVFP4MLP)
                and block.norm1.weight is not None and block.norm1.bias is not None
                and block.norm1.normalized_shape[0] % 64 == 0 and block.norm1.normalized_shape[0] <= 1280)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        a, mlp = self.attn, self.mlp
        qkv_l: QuantLinear = a.qkv
        proj_l: QuantLinear = a.proj
        if mlp.gx is None:   # first call: calibrate the MLP's static globals eagerly, as the module does
            self._calibrate(x)
        qk, pv = (a._nvfp4_qk, a._nvfp4_pv) if getattr(a, "_nvfp4_attn", False) else ("none", "none")
        wp, wsf = qkv_l._packed_weight()
        wp2, wsf2 = proj_l._packed_weight()
        return fused_block_op(
            x, self.norm1.weight, self.norm1.bias, float(self.norm1.eps),
            wp, wsf, qkv_l.w_global_scale, qkv_l.bias, qkv_l.x_global_scale,
            wp2, wsf2, proj_l.w_global_scale, proj_l.bias, proj_l.x_global_scale, _gamma(self.ls1),
            self.norm2.weight, self.norm2.bias, float(self.norm2.eps),
            _u8(mlp.w1q), _u8(mlp.w1sf), mlp.w1g, mlp.b1, _u8(mlp.w2q), _u8(mlp.w2sf), mlp.w2g, mlp.b2, mlp.gx, mlp.gh,
            _gamma(self.ls2), int(a.num_heads), float(a.scaling), qk, pv, bool(mlp.exact_gelu), mlp.w2_image())

    @torch.no_grad()
    def _calibrate(self, x: torch.Tensor) -> None:
        """The MLP's static globals from this input, through the same attention half as the block."""
        B, S, C = x.shape
        x2 = x.reshape(B * S, C).to(torch.bfloat16).contiguous()
        a = self.attn
        qk, pv = (a._nvfp4_qk, a._nvfp4_pv) if getattr(a, "_nvfp4_attn", False) else ("none", "none")
        qkv_l, proj_l = a.qkv, a.proj
        wp, wsf = qkv_l._packed_weight()
        wp2, wsf2 = proj_l._packed_weight()
        y = _attention_half(x2, B, S, C, self.norm1.weight, self.norm1.bias, float(self.norm1.eps), wp, wsf,
                            qkv_l.w_global_scale, qkv_l.bias, qkv_l.x_global_scale, wp2, wsf2, proj_l.w_global_scale,
                            proj_l.bias, proj_l.x_global_scale, int(a.num_heads), float(a.scaling), qk, pv)
        x_mid = x2 + self.ls1(y.reshape(B, S, C)).reshape(B * S, C)
        self.mlp._calibrate(F.layer_norm(x_mid, (C,), self.norm2.weight, self.norm2.bias, self.norm2.eps))


def _attention_route(qkv: torch.Tensor, H: int, scaling: float, qk: str, pv: str):
    """Attention of the packed (B, S, 3*H*D) projection: a (B, S, H*D) tensor, ("amax", out, max |out|) from
    the bf16 kernel, or ("split", out[:, :128k], out[:, 128k:]) from two cuDNN calls.  qk = pv = "none" is the
    unflagged (bf16) route."""
    B, S, C3 = qkv.shape
    D = C3 // (3 * H)
    if qk == "nvfp4" and pv == "nvfp4":
        return ops.attention_packed_qkv(qkv, H, scaling)
    if qk == "none" and qkv.dtype == torch.bfloat16 and ops.bf16_kernel_ok(S, D, scaling):
        # the reference's bf16 route (torch SDPA) on the tcgen05 kernel: exact softmax, fp32 accumulation,
        # output (B, S, H*D) read by the proj cast as it is; the kernel also returns max |out|, the amax of
        # the proj's dynamic activation cast
        am = torch.empty((), dtype=torch.float32, device=qkv.device)
        return "amax", ops.attention_bf16_packed_qkv(qkv, H, scaling, out_amax=am), am
    q, k, v = qkv.reshape(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
    if qk != "none":   # the fp8 and mixed routes
        from ..nvfp4.attention import quant_sdpa
        o = quant_sdpa(q, k, v, scale=scaling, qk=qk, pv=pv)
        return o.transpose(1, 2).reshape(B, S, H * D)
    s_main = S // 128 * 128
    if s_main >= 128 and 0 < S - s_main <= 16:
        # cuDNN's SDPA pays for whole 128-query tiles (S = 257 costs 2.6x S = 256): run queries [0, s_main)
        # and the few remaining ones as two calls over all keys -- each row's softmax is complete in
        # either -- and hand both parts to the proj cast as they are
        o1 = F.scaled_dot_product_attention(q[:, :, :s_main], k, v, scale=scaling)
        o2 = F.scaled_dot_product_attention(q[:, :, s_main:], k, v, scale=scaling)
        return "split", o1.transpose(1, 2).reshape(B, s_main, H * D), o2.transpose(1, 2).reshape(B, S - s_main, H * D)
    return F.scaled_dot_product_attention(q, k, v, scale=scaling).transpose(1, 2).reshape(B, S, H * D)


def _attention_half(x2, B, S, C, n1w, n1b, eps1, qkv_wp, qkv_wsf, qkv_wg, qkv_b, qkv_xg, proj_wp, proj_wsf,
                    proj_wg, proj_b, proj_xg, H, scaling, qk, pv):
    """norm1 -> NVFP4 -> qkv GEMM -> attention -> NVFP4 -> proj GEMM: the (B*S, C) bf16 proj output."""
    # norm1 -> NVFP4 (QuantLinear's activation global: static if calibrated, else dynamic)
    ap, asf, ag, _ = ops.ln_cast(x2, n1w, n1b, eps1, gs=qkv_xg)
    qkv = ops.gemm(ap, asf, ag, qkv_wp, qkv_wsf, qkv_wg, bias=qkv_b).reshape(B, S, -1)
    o = _attention_route(qkv, H, scaling, qk, pv)
    if isinstance(o, tuple) and o[0] == "split":   # one NVFP4 operand from both parts, no concatenation
        op, osf, og = ops.cast_split(o[1], o[2], gs=proj_xg)
    elif isinstance(o, tuple):                      # the attention kernel measured the amax: cast with its global
        gs = proj_xg if proj_xg is not None else ops.global_scale(o[2])
        op, osf, _, og = ops.cast(o[1].reshape(B * S, C), gs, "six")
    else:
        op, osf, _, og = ops.cast(o.reshape(B * S, C), proj_xg, "six")
    return ops.gemm(op, osf, og, proj_wp, proj_wsf, proj_wg, bias=proj_b)


@torch.library.custom_op("vitfp4::fused_block", mutates_args=())
def fused_block_op(x: torch.Tensor, n1w: torch.Tensor, n1b: torch.Tensor, eps1: float, qkv_wp: torch.Tensor,
                   qkv_wsf: torch.Tensor, qkv_wg: torch.Tensor, qkv_b: torch.Tensor | None,
                   qkv_xg: torch.Tensor | None, proj_wp: torch.Tensor, proj_wsf: torch.Tensor,
                   proj_wg: torch.Tensor, proj_b: torch.Tensor | None, proj_xg: torch.Tensor | None,
                   ls1: torch.Tensor | None, n2w: torch.Tensor, n2b: torch.Tensor, eps2: float, w1q: torch.Tensor,
                   w1sf: torch.Tensor, w1g: torch.Tensor, b1: torch.Tensor | None, w2q: torch.Tensor,
                   w2sf: torch.Tensor, w2g: torch.Tensor, b2: torch.Tensor | None, gx: torch.Tensor,
                   gh: torch.Tensor, ls2: torch.Tensor | None, num_heads: int, scaling: float, qk: str, pv: str,
                   exact_gelu: bool, w2img: torch.Tensor | None = None) -> torch.Tensor:
    """One converted transformer block on the fused kernels (FusedNVFP4Block.forward after calibration):
    (B, S, C) -> (B, S, C) bf16."""
    B, S, C = x.shape
    x2 = x.reshape(B * S, C)
    if x2.dtype != torch.bfloat16 or not x2.is_contiguous():
        x2 = x2.to(torch.bfloat16).contiguous()
    y = _attention_half(x2, B, S, C, n1w, n1b, eps1, qkv_wp, qkv_wsf, qkv_wg, qkv_b, qkv_xg, proj_wp, proj_wsf,
                        proj_wg, proj_b, proj_xg, num_heads, scaling, qk, pv)
    # x + ls1(y) -> norm2 -> NVFP4 with the MLP's static gx; the new residual x_mid is written once
    hp, hsf, gxx, x_mid = ops.ln_cast(x2, n2w, n2b, eps2, gs=gx, y=y, gamma=ls1)
    gp, gsf = ops.gemm_gelu_nvfp4(hp, hsf, gxx, w1q, w1sf, w1g, b1, gh, exact=exact_gelu)
    out = ops.gemm_residual(gp, gsf, gh, w2q, w2sf, w2g, b2, x_mid, gamma=ls2, out=x_mid, b_image=w2img)
    return out.reshape(B, S, C)


@fused_block_op.register_fake
def _(x, n1w, n1b, eps1, qkv_wp, qkv_wsf, qkv_wg, qkv_b, qkv_xg, proj_wp, proj_wsf, proj_wg, proj_b, proj_xg, ls1,
      n2w, n2b, eps2, w1q, w1sf, w1g, b1, w2q, w2sf, w2g, b2, gx, gh, ls2, num_heads, scaling, qk, pv, exact_gelu,
      w2img=None):
    return x.new_empty(x.shape, dtype=torch.bfloat16)


def fuse_norms(model: nn.Module) -> int:
    """Replace every eligible converted block (see FusedNVFP4Block.eligible) in place; returns the count."""
    n = 0
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if FusedNVFP4Block.eligible(child):
                setattr(mod, cname, FusedNVFP4Block(child))
                n += 1
    return n
