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

    def _attention(self, qkv: torch.Tensor):
        """Attention of the packed (B, S, 3*H*D) projection: a (B, S, H*D) tensor, ("amax", out,
        max |out|) from the bf16 kernel, or ("split", out[:, :128k], out[:, 128k:]) from two cuDNN calls."""
        a = self.attn
        B, S, _ = qkv.shape
        H, D = a.num_heads, a.head_dim
        if getattr(a, "_nvfp4_attn", False) and a._nvfp4_qk == "nvfp4" and a._nvfp4_pv == "nvfp4":
            return ops.attention_packed_qkv(qkv, H, a.scaling)
        if not getattr(a, "_nvfp4_attn", False) and qkv.dtype == torch.bfloat16 and ops.bf16_kernel_ok(S, D):
            # the reference's bf16 route (torch SDPA) on the tcgen05 kernel: exact softmax, fp32
            # accumulation, output (B, S, H*D) read by the proj cast as it is; the kernel also
            # returns max |out|, the amax of the proj's dynamic activation cast
            am = torch.empty((), dtype=torch.float32, device=qkv.device)
            return "amax", ops.attention_bf16_packed_qkv(qkv, H, a.scaling, out_amax=am), am
        q, k, v = qkv.reshape(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
        if getattr(a, "_nvfp4_attn", False):   # the fp8 and mixed routes (GPU emulation)
            from ..nvfp4.attention import quant_sdpa
            o = quant_sdpa(q, k, v, scale=a.scaling, qk=a._nvfp4_qk, pv=a._nvfp4_pv)
            return o.transpose(1, 2).reshape(B, S, H * D)
        s_main = S // 128 * 128
        if s_main >= 128 and 0 < S - s_main <= 16:
            # cuDNN's SDPA pays for whole 128-query tiles (S = 257 costs 2.6x S = 256): run queries
            # [0, s_main) and the few remaining ones as two calls over all keys -- each row's softmax
            # is complete in either -- and hand both parts to the proj cast as they are
            o1 = F.scaled_dot_product_attention(q[:, :, :s_main], k, v, scale=a.scaling)
            o2 = F.scaled_dot_product_attention(q[:, :, s_main:], k, v, scale=a.scaling)
            return "split", o1.transpose(1, 2).reshape(B, s_main, H * D), o2.transpose(1, 2).reshape(B, S - s_main, H * D)
        return F.scaled_dot_product_attention(q, k, v, scale=a.scaling).transpose(1, 2).reshape(B, S, H * D)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, S, C = x.shape
        x2 = x.reshape(B * S, C)
        if x2.dtype != torch.bfloat16 or not x2.is_contiguous():
            x2 = x2.to(torch.bfloat16).contiguous()
        qkv_l: QuantLinear = self.attn.qkv
        proj_l: QuantLinear = self.attn.proj
        # norm1 -> NVFP4 (QuantLinear's activation global: static if calibrated, else dynamic)
        ap, asf, ag, _ = ops.ln_cast(x2, self.norm1.weight, self.norm1.bias, self.norm1.eps, gs=qkv_l.x_global_scale)
        wp, wsf = qkv_l._packed_weight()
        qkv = ops.gemm(ap, asf, ag, wp, wsf, qkv_l.w_global_scale, bias=qkv_l.bias).reshape(B, S, -1)
        o = self._attention(qkv)
        if isinstance(o, tuple) and o[0] == "split":   # one NVFP4 operand from both parts, no concatenation
            op, osf, og = ops.cast_split(o[1], o[2], gs=proj_l.x_global_scale)
            wp2, wsf2 = proj_l._packed_weight()
            y = ops.gemm(op, osf, og, wp2, wsf2, proj_l.w_global_scale, bias=proj_l.bias)
        elif isinstance(o, tuple):   # the attention kernel measured the amax: cast with its global
            gs = proj_l.x_global_scale if proj_l.x_global_scale is not None else ops.global_scale(o[2])
            op, osf, _, og = ops.cast(o[1].reshape(B * S, C), gs, "six")
            wp2, wsf2 = proj_l._packed_weight()
            y = ops.gemm(op, osf, og, wp2, wsf2, proj_l.w_global_scale, bias=proj_l.bias)
        else:
            y = proj_l(o).reshape(B * S, C)
        mlp: FusedNVFP4MLP = self.mlp
        if mlp.gx is None:   # first call: calibrate the MLP's static globals exactly as the module does
            x_mid = (x2 + self.ls1(y.reshape(B, S, C)).reshape(B * S, C))
            mlp._calibrate(F.layer_norm(x_mid, (C,), self.norm2.weight, self.norm2.bias, self.norm2.eps))
        # x + ls1(y) -> norm2 -> NVFP4 with the MLP's static gx; the new residual x_mid is written once
        hp, hsf, gx, x_mid = ops.ln_cast(x2, self.norm2.weight, self.norm2.bias, self.norm2.eps, gs=mlp.gx, y=y,
                                         gamma=_gamma(self.ls1))
        gp, gsf = ops.gemm_gelu_nvfp4(hp, hsf, gx, _u8(mlp.w1q), _u8(mlp.w1sf), mlp.w1g, mlp.b1, mlp.gh,
                                      exact=mlp.exact_gelu)
        out = ops.gemm_residual(gp, gsf, mlp.gh, _u8(mlp.w2q), _u8(mlp.w2sf), mlp.w2g, mlp.b2, x_mid,
                                gamma=_gamma(self.ls2), out=x_mid)
        return out.reshape(B, S, C)


def fuse_norms(model: nn.Module) -> int:
    """Replace every eligible converted block (see FusedNVFP4Block.eligible) in place; returns the count."""
    n = 0
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if FusedNVFP4Block.eligible(child):
                setattr(mod, cname, FusedNVFP4Block(child))
                n += 1
    return n
