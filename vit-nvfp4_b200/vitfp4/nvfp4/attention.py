"""Low-precision scaled-dot-product attention (reference: src/vit_nvfp4/nvfp4/attention.py:53-86).

``quant_sdpa`` keeps the reference's signature.  Routes:
  qk = pv = 'nvfp4' -> the sm_100a FP4 attention kernels of libvitfp4.so (QK^T and PV as
                       block-scaled tcgen05 MMAs, exact two-pass softmax, P re-quantised to NVFP4
                       in shared memory, smooth-K / smooth-V);
  qk = pv = 'bf16'  -> exact bf16 attention (torch SDPA), the route the reference keeps for
                       unquantised blocks;
  any other mix     -> NotImplementedError (the FP8 route is not built).
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

_MODES = ("bf16", "fp8", "nvfp4")


def _bf16_sdpa(q, k, v, attn_mask, is_causal, scale, smooth_k, smooth_v):
    if smooth_k:
        k = k - k.mean(dim=-2, keepdim=True)
    mu = None
    if smooth_v:
        mu = v.mean(dim=-2, keepdim=True)
        v = v - mu
    out = F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, is_causal=is_causal, scale=scale)
    return out if mu is None else out + mu


def quant_sdpa(query, key, value, attn_mask=None, is_causal=False, scale=None, qk="fp8", pv="fp8",
               smooth_k=True, smooth_v=True):
    """Drop-in low-precision attention: (..., S, D) operands -> (..., S, D) in query.dtype."""
    assert qk in _MODES and pv in _MODES
    D = query.shape[-1]
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if qk == "bf16" and pv == "bf16":
        return _bf16_sdpa(query, key, value, attn_mask, is_causal, scale, smooth_k, smooth_v).to(query.dtype)
    if qk == "nvfp4" and pv == "nvfp4":
        if attn_mask is not None or is_causal:
            raise NotImplementedError("the FP4 attention kernel is for ViT (no mask, not causal)")
        if not (smooth_k and smooth_v):
            raise NotImplementedError("the FP4 attention kernel always applies smooth-K / smooth-V")
        from . import ops
        return ops.attention_bhsd(query, key, value, scale).to(query.dtype)
    raise NotImplementedError(f"attention route qk={qk!r}, pv={pv!r} is not built (nvfp4/nvfp4 and bf16/bf16 are)")
