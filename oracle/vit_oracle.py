"""CPU restatement of a W4A4 ViT forward with the reference's torch-backend semantics.

TEST INFRASTRUCTURE ONLY (the CPU baseline / ``bench.py --impl reference`` arm).  It never
runs in the product path.

Semantics restated (Dev-Jahn/vit-nvfp4):
  * QuantLinear.forward (src/vit_nvfp4/ptq/qlinear.py:42-47) -> nvfp4_linear (nvfp4/gemm.py:32-38):
    dynamic NVFP4 activation cast (six), fp32-emulated GEMM (backends/reference.py:6-10), output
    rounded to the activation dtype (bf16), + bias in bf16; weights quantized once with
    Four-Over-Six ('mse', qlinear.py:34-39).
  * FusedNVFP4MLP (ptq/fused_mlp.py:38-55): x cast with the static gx, GEMM, + b1, GELU fused into
    the cast with the static gh, GEMM, + b2; gx / gh frozen on the first forward
    (fused_mlp.py:89-98); weights quantized with the "six" rule.
  * attention: exact softmax attention in fp32 on bf16 operands (the unflagged route,
    ptq/qattention.py:27-29), or the emulated NVFP4 quant_sdpa (nvfp4/attention.py:53-86).
Weights are random N(0, 0.02) (numpy generator), biases 0, LayerNorm (1, 0), LayerScale 1e-5.
"""
from __future__ import annotations

import numpy as np

from nvfp4_oracle import (dequantize_nvfp4, gelu, global_scale_of, quant_sdpa, quantize_to_nvfp4,
                          to_bf16)

F32 = np.float32


def make_weights(embed_dim=1024, depth=24, num_heads=16, mlp_ratio=4, patch=14, img=224, num_classes=1000,
                 init_values=1e-5, seed=0):
    rng = np.random.default_rng(seed)
    d, h = embed_dim, int(embed_dim * mlp_ratio)
    n = lambda *s: to_bf16((rng.standard_normal(s) * 0.02).astype(F32))
    W = {"cfg": dict(d=d, depth=depth, heads=num_heads, patch=patch, img=img, hidden=h, ls=init_values),
         "patch_w": n(d, 3 * patch * patch), "cls": n(1, d), "pos": n((img // patch) ** 2 + 1, d),
         "head_w": n(num_classes, d), "blocks": []}
    for _ in range(depth):
        blk = {}
        for name, (o, i) in {"qkv": (3 * d, d), "proj": (d, d)}.items():
            c, b, g = quantize_to_nvfp4(n(o, i), 16, block_select="mse")
            blk[name] = dequantize_nvfp4(c, b, g)
        for name, (o, i) in {"fc1": (h, d), "fc2": (d, h)}.items():
            c, b, g = quantize_to_nvfp4(n(o, i), 16, block_select="six")
            blk[name] = dequantize_nvfp4(c, b, g)
        blk["gx"] = blk["gh"] = None
        W["blocks"].append(blk)
    return W


def _layernorm(x, eps=1e-6):
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return to_bf16((x - m) / np.sqrt(v + F32(eps)))


def _w4a4(x2, w_deq, gs=None):
    c, b, g = quantize_to_nvfp4(x2, 16, global_scale=gs)
    return dequantize_nvfp4(c, b, g) @ w_deq.T


def forward(W, images: np.ndarray, attn: str = "bf16") -> np.ndarray:
    """images (B, 3, img, img) fp32 -> logits (B, classes) fp32."""
    cfg = W["cfg"]
    B, p, d, H = images.shape[0], cfg["patch"], cfg["d"], cfg["heads"]
    g = cfg["img"] // p
    patches = images.reshape(B, 3, g, p, g, p).transpose(0, 2, 4, 1, 3, 5).reshape(B, g * g, 3 * p * p)
    x = to_bf16(to_bf16(patches) @ W["patch_w"].T)
    x = np.concatenate([np.broadcast_to(W["cls"], (B, 1, d)), x], axis=1) + W["pos"]
    x = to_bf16(x)
    S, Dh = x.shape[1], d // H
    for blk in W["blocks"]:
        h = _layernorm(x).reshape(B * S, d)
        qkv = to_bf16(_w4a4(h, blk["qkv"])).reshape(B, S, 3, H, Dh).transpose(2, 0, 3, 1, 4)
        if attn == "nvfp4":
            o = quant_sdpa(qkv[0], qkv[1], qkv[2], qk="nvfp4", pv="nvfp4")
        else:
            s = (qkv[0] @ np.swapaxes(qkv[1], -1, -2)) * F32(Dh ** -0.5)
            s = np.exp(s - s.max(-1, keepdims=True))
            o = (s / s.sum(-1, keepdims=True)) @ qkv[2]
        o = to_bf16(o).transpose(0, 2, 1, 3).reshape(B * S, d)
        y = to_bf16(_w4a4(o, blk["proj"]))
        x = to_bf16(x + F32(cfg["ls"]) * y.reshape(B, S, d))
        h2 = _layernorm(x).reshape(B * S, d)
        if blk["gx"] is None:                                  # first forward freezes the MLP globals
            blk["gx"] = global_scale_of(h2)
            blk["gh"] = global_scale_of(gelu(to_bf16(_w4a4(h2, blk["fc1"], blk["gx"]))))
        y1 = to_bf16(_w4a4(h2, blk["fc1"], blk["gx"]))
        y2 = to_bf16(_w4a4(gelu(y1), blk["fc2"], blk["gh"]))
        x = to_bf16(x + F32(cfg["ls"]) * y2.reshape(B, S, d))
    x = _layernorm(x)
    return (x[:, 0] @ W["head_w"].T).astype(F32)
