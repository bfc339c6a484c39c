"""CPU restatement of a W4A4 ViT forward with the reference's torch-backend semantics.

TEST INFRASTRUCTURE ONLY (the checker of the end-to-end tests and the CPU baseline /
``bench.py --impl reference`` arm).  It never runs in the product path.

Semantics restated (Dev-Jahn/vit-nvfp4):
  * QuantLinear.forward (src/vit_nvfp4/ptq/qlinear.py:42-47) -> nvfp4_linear (nvfp4/gemm.py:32-38):
    dynamic NVFP4 activation cast (six), fp32-emulated GEMM (backends/reference.py:6-10), output
    rounded to the activation dtype, + bias in that dtype.
  * FusedNVFP4MLP (ptq/fused_mlp.py:38-55): x cast (the Triton cast's arithmetic,
    nvfp4_oracle.triton_cast_nvfp4) with the static gx, GEMM rounded to bf16, + b1 in bf16, erf-GELU
    in fp32 fused into the Triton cast with the static gh, GEMM, + b2; gx / gh frozen on the first
    forward from amax(x) and amax(F.gelu(y1)) of the bf16 tensors (fused_mlp.py:89-98).
  * attention: softmax attention in fp32 on the operands (the unflagged route, torch SDPA,
    ptq/qattention.py:27-29; with bf16 operands exp(s - max) is rounded to bf16 before the PV
    product and the row sum divides afterwards, as torch's flash-form SDPA does), the output
    rounded to the activation dtype; or the emulated NVFP4 quant_sdpa (nvfp4/attention.py:53-86).
  * LayerNorm, LayerScale and residual adds in the activation dtype (bf16: each op's result rounds
    to bf16, as torch's bf16 ops do).

``precision`` "bf16" rounds every activation the way a bf16 torch model does; "f32" is the fp32
model of BASELINE configuration 1.  ``mlp`` "fused" is FusedNVFP4MLP, "qlinear" is two QuantLinears
around torch's GELU.
"""
from __future__ import annotations

import numpy as np

from nvfp4_oracle import (dequantize_nvfp4, gelu, global_scale_of, quant_sdpa, quantize_to_nvfp4,
                          to_bf16, triton_cast_nvfp4)

F32 = np.float32


def make_weights(embed_dim=1024, depth=24, num_heads=16, mlp_ratio=4, patch=14, img=224, num_classes=1000,
                 init_values=1e-5, seed=0):
    """Random N(0, 0.02) bf16-representable weights (numpy generator), zero biases, LayerNorm (1, 0):
    qkv/proj quantized with Four-Over-Six, fc1/fc2 with the six rule (the fused MLP's)."""
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


def weights_from_model(model, block_select="six", fc_block_select=None):
    """Oracle weights from a vitfp4.vit.VisionTransformer (torch, any device): linear weights quantized
    by the oracle (``block_select`` for qkv/proj, ``fc_block_select`` -- default the same -- for
    fc1/fc2), everything else copied in fp32."""
    def a(t):
        return None if t is None else t.detach().float().cpu().numpy()

    fc_sel = fc_block_select or block_select
    cfg = model.config
    d = cfg.embed_dim
    W = {"cfg": dict(d=d, depth=len(model.blocks), heads=cfg.num_heads, patch=cfg.patch_size, img=cfg.img_size,
                     hidden=int(d * cfg.mlp_ratio), ls=None, eps=cfg.layer_norm_eps),
         "patch_w": a(model.patch_embed.proj.weight).reshape(d, -1), "patch_b": a(model.patch_embed.proj.bias),
         "cls": a(model.cls_token).reshape(1, d), "pos": a(model.pos_embed).reshape(-1, d),
         "norm": (a(model.norm.weight), a(model.norm.bias)),
         "head_w": a(model.head.weight), "head_b": a(model.head.bias), "blocks": []}
    for blk in model.blocks:
        d_ = {"norm1": (a(blk.norm1.weight), a(blk.norm1.bias)), "norm2": (a(blk.norm2.weight), a(blk.norm2.bias)),
              "ls1": a(getattr(blk.ls1, "gamma", None)), "ls2": a(getattr(blk.ls2, "gamma", None))}
        for name, lin, sel in (("qkv", blk.attn.qkv, block_select), ("proj", blk.attn.proj, block_select),
                               ("fc1", blk.mlp.fc1, fc_sel), ("fc2", blk.mlp.fc2, fc_sel)):
            d_[name] = dequantize_nvfp4(*quantize_to_nvfp4(a(lin.weight), 16, block_select=sel))
            d_[name + "_b"] = a(lin.bias)
        d_["gx"] = d_["gh"] = None
        W["blocks"].append(d_)
    return W


def _round_fn(precision):
    return to_bf16 if precision == "bf16" else (lambda x: np.asarray(x, F32))


def _layernorm(x, params, eps, rnd):
    """torch.nn.functional.layer_norm: fp32 statistics, affine, one rounding to the dtype."""
    x = np.asarray(x, F32)
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    y = (x - m) / np.sqrt(v + F32(eps))
    if params is not None and params[0] is not None:
        y = y * params[0] + params[1]
    return rnd(y.astype(F32))


def _w4a4(x2, w_deq, gs=None):
    c, b, g = quantize_to_nvfp4(x2, 16, global_scale=gs)
    return dequantize_nvfp4(c, b, g) @ w_deq.T


def _w4a4_triton(x2, w_deq, gs, apply_gelu=False):
    """The fused MLP's GEMM input: the Triton cast with the static global gs (fused_mlp.py:47, :50)."""
    c, b = triton_cast_nvfp4(x2, gs, apply_gelu=apply_gelu)
    return dequantize_nvfp4(c, b, gs) @ w_deq.T


def _linear_out(y, bias, rnd):
    """nvfp4_linear's output: the GEMM rounded to the dtype, then + bias in the dtype."""
    y = rnd(y)
    return y if bias is None else rnd(y + bias)


def block_forward(blk, cfg, x, attn: str = "bf16", precision: str = "bf16", mlp: str = "fused") -> np.ndarray:
    """One transformer block (timm / DINOv2 layout) on x (B, S, d); ``blk`` from make_weights or
    weights_from_model.  With mlp="fused" the first call freezes blk["gx"] / blk["gh"]."""
    rnd = _round_fn(precision)
    eps = cfg.get("eps", 1e-6)
    x = np.asarray(x, F32)
    B, S, d = x.shape
    H = cfg["heads"]
    Dh = d // H
    ls1 = blk.get("ls1", None if cfg["ls"] is None else np.full(d, cfg["ls"], F32))
    ls2 = blk.get("ls2", None if cfg["ls"] is None else np.full(d, cfg["ls"], F32))
    h = _layernorm(x, blk.get("norm1"), eps, rnd).reshape(B * S, d)
    qkv = _linear_out(_w4a4(h, blk["qkv"]), blk.get("qkv_b"), rnd)
    qkv = qkv.reshape(B, S, 3, H, Dh).transpose(2, 0, 3, 1, 4)
    if attn == "nvfp4":
        o = quant_sdpa(qkv[0], qkv[1], qkv[2], qk="nvfp4", pv="nvfp4")
    else:
        # softmax(q k^T * scale) v in fp32; for bf16 operands torch's SDPA (flash form) multiplies
        # the bf16-rounded exp(s - max) with v and divides by the fp32 row sum afterwards
        s = (qkv[0] @ np.swapaxes(qkv[1], -1, -2)) * F32(Dh ** -0.5)
        e = np.exp(s - s.max(-1, keepdims=True)).astype(F32)
        o = (rnd(e) @ qkv[2]) / e.sum(-1, keepdims=True)
    o = rnd(o).transpose(0, 2, 1, 3).reshape(B * S, d)
    y = _linear_out(_w4a4(o, blk["proj"]), blk.get("proj_b"), rnd).reshape(B, S, d)
    x = rnd(x + (y if ls1 is None else rnd(y * rnd(ls1))))
    h2 = _layernorm(x, blk.get("norm2"), eps, rnd).reshape(B * S, d)
    b1, b2 = blk.get("fc1_b"), blk.get("fc2_b")
    if mlp == "fused":
        if blk["gx"] is None:              # the first forward freezes the MLP globals
            blk["gx"] = global_scale_of(h2)
            y1c = _linear_out(_w4a4_triton(h2, blk["fc1"], blk["gx"]), b1, to_bf16)
            blk["gh"] = global_scale_of(to_bf16(gelu(y1c)))
        y1 = _linear_out(_w4a4_triton(h2, blk["fc1"], blk["gx"]), b1, to_bf16)
        y2 = _linear_out(_w4a4_triton(y1, blk["fc2"], blk["gh"], apply_gelu=True), b2, to_bf16)
    else:
        y1 = _linear_out(_w4a4(h2, blk["fc1"]), b1, rnd)
        y2 = _linear_out(_w4a4(rnd(gelu(y1)), blk["fc2"]), b2, rnd)
    y2 = y2.reshape(B, S, d)
    return rnd(x + (y2 if ls2 is None else rnd(y2 * rnd(ls2))))


def embed(W, images: np.ndarray, precision: str = "bf16") -> np.ndarray:
    """Patch embedding, class token and position embedding: images -> (B, T, d) tokens."""
    rnd = _round_fn(precision)
    cfg = W["cfg"]
    B, p, d = images.shape[0], cfg["patch"], cfg["d"]
    g = cfg["img"] // p
    patches = rnd(images).reshape(B, 3, g, p, g, p).transpose(0, 2, 4, 1, 3, 5).reshape(B, g * g, 3 * p * p)
    x = rnd(patches @ W["patch_w"].T)
    if W.get("patch_b") is not None:
        x = rnd(x + W["patch_b"])
    return rnd(np.concatenate([np.broadcast_to(rnd(W["cls"]), (B, 1, d)), x], axis=1) + rnd(W["pos"]))


def head(W, x: np.ndarray, precision: str = "bf16") -> np.ndarray:
    """Final LayerNorm and the classifier on the class token: (B, T, d) -> (B, classes) fp32."""
    rnd = _round_fn(precision)
    x = _layernorm(x, W.get("norm"), W["cfg"].get("eps", 1e-6), rnd)
    logits = x[:, 0] @ W["head_w"].T
    if W.get("head_b") is not None:
        logits = logits + W["head_b"]
    return rnd(logits).astype(F32)


def forward(W, images: np.ndarray, attn: str = "bf16", precision: str = "bf16", mlp: str = "fused") -> np.ndarray:
    """images (B, 3, img, img) fp32 -> logits (B, classes) fp32."""
    x = embed(W, images, precision)
    for blk in W["blocks"]:
        x = block_forward(blk, W["cfg"], x, attn=attn, precision=precision, mlp=mlp)
    return head(W, x, precision)
