"""Low-precision scaled-dot-product attention (reference: src/vit_nvfp4/nvfp4/attention.py:53-86).

``quant_sdpa`` keeps the reference's signature.  Routes:
  qk = pv = 'nvfp4' -> the sm_100a FP4 attention kernels of libvitfp4.so (QK^T and PV as
                       block-scaled tcgen05 MMAs, exact two-pass softmax, P re-quantised to NVFP4
                       in shared memory, smooth-K / smooth-V each on or off as asked);
  qk = pv = 'bf16'  -> exact bf16 attention (torch SDPA), the route the reference keeps for
                       unquantised blocks;
  qk = pv = 'fp8'   -> the sm_100a FP8 attention kernels (E4M3 MMAs, per-row scales, no mask): one
                       fused kernel for head dim 64 and S <= 320, a prep kernel plus a long-sequence
                       kernel for other head dims (multiples of 16 up to 128) and longer sequences
                       (ViT-H/14: head dim 80, S = 257 or 1025); shapes beyond those take the
                       emulation below;
  any other mix     -> the reference's own emulation (quantize-dequantize of the operands, fp32
                       matmuls and softmax) run on the GPU with torch ops, in chunks of heads; NVFP4
                       operands are quantized by the CUDA cast kernel (whole-tensor globals, the P
                       global from a first pass over all chunks), FP8 ones per row as fp8.py.  No
                       dedicated kernel is built for the mixed routes.
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


def _nvfp4_qdq_gpu(x: torch.Tensor, global_scale: torch.Tensor | None = None) -> torch.Tensor:
    """NVFP4 round trip along the last dim (zero-padded to 16) on the GPU (attention.py:28-36)."""
    from .quant import dequantize_nvfp4, quantize_to_nvfp4
    k = x.shape[-1]
    pad = (-k) % 16
    xp = F.pad(x, (0, pad)) if pad else x
    codes, bs, gs = quantize_to_nvfp4(xp.contiguous(), 16, global_scale=global_scale)
    d = dequantize_nvfp4(codes, bs, gs)
    return d[..., :k] if pad else d


def _qdq_gpu(x: torch.Tensor, mode: str, axis: int = -1, global_scale: torch.Tensor | None = None):
    """attention.py:39-50 on the GPU."""
    from .fp8 import fp8_e4m3_quant_dequant
    if mode == "bf16":
        return x.to(torch.bfloat16).to(torch.float32)
    if axis not in (-1, x.ndim - 1):
        return _qdq_gpu(x.transpose(axis, -1).contiguous(), mode, -1, global_scale).transpose(axis, -1)
    if mode == "fp8":
        return fp8_e4m3_quant_dequant(x)
    return _nvfp4_qdq_gpu(x, global_scale)


def _emulated_sdpa(q, k, v, attn_mask, is_causal, scale, qk, pv, smooth_k, smooth_v,
                   chunk_bytes: int = 1 << 30):
    """The reference's quant_sdpa arithmetic (attention.py:53-86) with torch GPU ops; the (..., S, S)
    score tensors are formed for chunks of the leading (batch x head) rows at a time."""
    lead = q.shape[:-2]
    S, D = q.shape[-2], q.shape[-1]
    Sk = k.shape[-2]
    qf, kf, vf = (t.float().reshape(-1, t.shape[-2], t.shape[-1]) for t in (q, k, v))
    if smooth_k:
        kf = kf - kf.mean(dim=-2, keepdim=True)
    mu = None
    if smooth_v:
        mu = vf.mean(dim=-2, keepdim=True)
        vf = vf - mu
    qd, kd = _qdq_gpu(qf, qk), _qdq_gpu(kf, qk)     # globals over the whole tensors
    vd = _qdq_gpu(vf, pv, axis=-2)
    mask = None
    if attn_mask is not None:
        mask = attn_mask.expand(*lead, S, Sk).reshape(-1, S, Sk)
    n = qf.shape[0]
    step = max(1, chunk_bytes // (S * Sk * 4))

    def probs(i0: int, i1: int) -> torch.Tensor:
        s = torch.matmul(qd[i0:i1], kd[i0:i1].transpose(-1, -2)) * scale
        if is_causal:
            causal = torch.ones(S, Sk, dtype=torch.bool, device=s.device).tril(Sk - S)
            s = s.masked_fill(~causal, float("-inf"))
        if mask is not None:
            s = s.masked_fill(~mask[i0:i1], float("-inf")) if mask.dtype == torch.bool else s + mask[i0:i1]
        return torch.softmax(s, dim=-1)

    p_gs = None
    if pv == "nvfp4":   # the reference's P global is the amax of the whole P tensor
        amax = torch.zeros((), device=q.device)
        for i0 in range(0, n, step):
            amax = torch.maximum(amax, probs(i0, min(n, i0 + step)).abs().amax())
        p_gs = torch.clamp(amax, min=1e-12) / (6.0 * 448.0)
    out = torch.empty(n, S, D, dtype=torch.float32, device=q.device)
    for i0 in range(0, n, step):
        i1 = min(n, i0 + step)
        out[i0:i1] = torch.matmul(_qdq_gpu(probs(i0, i1), pv, -1, p_gs), vd[i0:i1])
    if mu is not None:
        out = out + mu
    return out.reshape(*lead, S, D)


@torch.library.custom_op("vitfp4::attention_lowp", mutates_args=())
def attention_lowp_op(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, qk: str, pv: str,
                      smooth_k: bool, smooth_v: bool) -> torch.Tensor:
    """The kernel routes of quant_sdpa (nvfp4/nvfp4, and fp8/fp8 where ops.fp8_kernel_ok) on (B, H, S, D)
    operands -> (B, H, S, D) bf16, laid out as a (B, S, H, D) tensor (the kernels' output layout)."""
    from . import ops
    if qk == "nvfp4":
        return ops.attention_bhsd(q, k, v, scale, smooth_k=smooth_k, smooth_v=smooth_v)
    return ops.attention_fp8_bhsd(q, k, v, scale, smooth_k=smooth_k, smooth_v=smooth_v)


@attention_lowp_op.register_fake
def _(q, k, v, scale, qk, pv, smooth_k, smooth_v):
    B, H, S, D = q.shape
    return q.new_empty((B, S, H, D), dtype=torch.bfloat16).transpose(1, 2)


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
        if query.dim() == 4:
            return attention_lowp_op(query, key, value, float(scale), qk, pv, smooth_k, smooth_v).to(query.dtype)
        from . import ops
        return ops.attention_bhsd(query, key, value, scale, smooth_k=smooth_k, smooth_v=smooth_v).to(query.dtype)
    if not query.is_cuda:
        raise RuntimeError("quant_sdpa runs on the GPU (CUDA tensors required)")
    if qk == "fp8" and pv == "fp8" and attn_mask is None and not is_causal and query.dim() == 4:
        from . import ops
        if ops.fp8_kernel_ok(query.shape[-2], D):
            return attention_lowp_op(query, key, value, float(scale), qk, pv, smooth_k, smooth_v).to(query.dtype)
    return _emulated_sdpa(query, key, value, attn_mask, is_causal, scale, qk, pv, smooth_k, smooth_v).to(query.dtype)
