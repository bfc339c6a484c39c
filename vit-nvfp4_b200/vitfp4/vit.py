"""A timm / DINOv2-style Vision Transformer used as the workload of the benchmark and tests.

Module names follow timm (``blocks.N.{norm1, attn.{qkv, proj}, ls1, norm2, mlp.{fc1, act, fc2},
ls2}``) so the reference's conversion policies (``vit_block_policy``, ``fuse_mlps``,
``vit_attn_policy``) select the same layers they select on a timm / DINOv2 model.  The
attention module exposes ``scaling`` and ``config._attn_implementation`` and dispatches through
the attention-function registry the way HF transformers' attention modules do, so
``enable_quant_attention`` routes it unchanged.

Weights are random-initialised (N(0, 0.02), zero biases, LayerNorm gamma=1 beta=0, LayerScale
init value), matching the BASELINE configurations; no checkpoint is loaded.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

# Registry of attention implementations keyed by ``config._attn_implementation`` (mirrors
# transformers' ALL_ATTENTION_FUNCTIONS; vitfp4.ptq.qattention registers into both).
ATTENTION_FUNCTIONS: dict = {}


def sdpa_attention(module, query, key, value, attention_mask=None, dropout=0.0, scaling=None,
                   is_causal=None, **kwargs):
    out = F.scaled_dot_product_attention(query, key, value, attn_mask=attention_mask, dropout_p=dropout,
                                         scale=scaling, is_causal=bool(is_causal))
    return out.transpose(1, 2), None


ATTENTION_FUNCTIONS["sdpa"] = sdpa_attention


def _lookup_attention(name: str):
    fn = ATTENTION_FUNCTIONS.get(name)
    if fn is None:
        try:
            from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS
            fn = ALL_ATTENTION_FUNCTIONS[name]
        except Exception as e:  # pragma: no cover
            raise KeyError(f"unknown attention implementation {name!r}") from e
    return fn


@dataclass
class ViTConfig:
    img_size: int = 224
    patch_size: int = 14
    in_chans: int = 3
    num_classes: int = 1000
    embed_dim: int = 1024
    depth: int = 24
    num_heads: int = 16
    mlp_ratio: float = 4.0
    init_values: float | None = 1e-5     # LayerScale gamma init (None -> no LayerScale)
    layer_norm_eps: float = 1e-6
    _attn_implementation: str = "sdpa"

    @property
    def num_tokens(self) -> int:
        return (self.img_size // self.patch_size) ** 2 + 1


# BASELINE.json configurations
VIT_S16 = dict(img_size=224, patch_size=16, embed_dim=384, depth=12, num_heads=6, init_values=None)
VIT_B16 = dict(img_size=224, patch_size=16, embed_dim=768, depth=12, num_heads=12, init_values=None)
VIT_L14 = dict(img_size=224, patch_size=14, embed_dim=1024, depth=24, num_heads=16, init_values=1e-5)
VIT_H14_448 = dict(img_size=448, patch_size=14, embed_dim=1280, depth=32, num_heads=16, init_values=None)


class LayerScale(nn.Module):
    def __init__(self, dim: int, init_values: float):
        super().__init__()
        self.gamma = nn.Parameter(init_values * torch.ones(dim))

    def forward(self, x):
        return x * self.gamma


class Attention(nn.Module):
    def __init__(self, config: ViTConfig):
        super().__init__()
        self.config = config
        self.num_heads = config.num_heads
        self.head_dim = config.embed_dim // config.num_heads
        self.scaling = self.head_dim ** -0.5
        self.qkv = nn.Linear(config.embed_dim, 3 * config.embed_dim)
        self.proj = nn.Linear(config.embed_dim, config.embed_dim)

    def forward(self, x):
        B, S, C = x.shape
        qkv = self.qkv(x)
        fn = _lookup_attention(self.config._attn_implementation)
        if getattr(fn, "_vitfp4_packed_qkv", False):
            out = fn(self, qkv, num_heads=self.num_heads, scaling=self.scaling)
        else:
            q, k, v = qkv.reshape(B, S, 3, self.num_heads, self.head_dim).permute(2, 0, 3, 1, 4).unbind(0)
            out, _ = fn(self, q, k, v, None, dropout=0.0, scaling=self.scaling, is_causal=False)
        return self.proj(out.reshape(B, S, C))


class Mlp(nn.Module):
    def __init__(self, dim: int, hidden: int):
        super().__init__()
        self.fc1 = nn.Linear(dim, hidden)
        self.act = nn.GELU()
        self.fc2 = nn.Linear(hidden, dim)

    def forward(self, x):
        return self.fc2(self.act(self.fc1(x)))


class Block(nn.Module):
    def __init__(self, config: ViTConfig):
        super().__init__()
        d = config.embed_dim
        self.norm1 = nn.LayerNorm(d, eps=config.layer_norm_eps)
        self.attn = Attention(config)
        self.ls1 = LayerScale(d, config.init_values) if config.init_values else nn.Identity()
        self.norm2 = nn.LayerNorm(d, eps=config.layer_norm_eps)
        self.mlp = Mlp(d, int(d * config.mlp_ratio))
        self.ls2 = LayerScale(d, config.init_values) if config.init_values else nn.Identity()

    def forward(self, x):
        x = x + self.ls1(self.attn(self.norm1(x)))
        x = x + self.ls2(self.mlp(self.norm2(x)))
        return x


class PatchEmbed(nn.Module):
    """Non-overlapping patch projection.  Same parameters as timm's Conv2d(k=stride=patch),
    evaluated as one (B*P, C*p*p) x (C*p*p, d) GEMM on the unfolded patches (the strided conv
    is exactly this matmul, and cuDNN's conv path is several times slower on B200)."""

    def __init__(self, config: ViTConfig):
        super().__init__()
        self.patch = config.patch_size
        self.proj = nn.Conv2d(config.in_chans, config.embed_dim, config.patch_size, config.patch_size)

    def forward(self, x):
        B, C, Hh, Ww = x.shape
        p = self.patch
        g_h, g_w = Hh // p, Ww // p
        K = C * p * p
        if x.is_cuda and x.dtype == torch.bfloat16 and Ww % 8 == 0:
            # CUDA unfold into rows padded to a multiple of 8 values (16-byte rows keep cuBLAS on its
            # sm_100 kernels; the zero columns meet zero weight columns)
            from .nvfp4 import ops
            kp = (K + 7) // 8 * 8
            patches = ops.patchify_op(x, p, kp)
            return F.linear(patches, self._weight_padded(kp), self.proj.bias).reshape(B, g_h * g_w, -1)
        patches = x.reshape(B, C, g_h, p, g_w, p).permute(0, 2, 4, 1, 3, 5).reshape(B, g_h * g_w, K)
        w = self.proj.weight.reshape(self.proj.out_channels, -1)
        return F.linear(patches, w, self.proj.bias)

    def _weight_padded(self, kp: int) -> torch.Tensor:
        w = self.proj.weight
        key = (w.data_ptr(), 0 if w.is_inference() else w._version, w.dtype, kp)
        if getattr(self, "_wp_key", None) != key:
            self._wp = F.pad(w.detach().reshape(w.shape[0], -1), (0, kp - w[0].numel())).contiguous()
            self._wp_key = key
        return self._wp


class VisionTransformer(nn.Module):
    def __init__(self, config: ViTConfig):
        super().__init__()
        self.config = config
        d = config.embed_dim
        self.patch_embed = PatchEmbed(config)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, d))
        self.pos_embed = nn.Parameter(torch.zeros(1, config.num_tokens, d))
        self.blocks = nn.ModuleList(Block(config) for _ in range(config.depth))
        self.norm = nn.LayerNorm(d, eps=config.layer_norm_eps)
        self.head = nn.Linear(d, config.num_classes)

    def forward_features(self, x):
        x = self.patch_embed(x)
        if x.is_cuda and x.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0:
            from .nvfp4 import ops
            x = ops.embed_tokens_op(x, self.cls_token, self.pos_embed)   # cat + add, one pass
        else:
            x = torch.cat([self.cls_token.expand(x.shape[0], -1, -1).to(x.dtype), x], dim=1)
            x = x + self.pos_embed.to(x.dtype)
        for blk in self.blocks:
            x = blk(x)
        return self.norm(x)

    def forward(self, x):
        return self.head(self.forward_features(x)[:, 0])


def init_weights(model: nn.Module, seed: int = 0, std: float = 0.02) -> nn.Module:
    """N(0, std) weights, zero biases, LayerNorm (1, 0); LayerScale keeps its init value.  The random
    stream is a generator on the model's device seeded with ``seed`` (the CPU generator for a CPU
    model, so CPU-built models are the same on every machine)."""
    dev = next(model.parameters()).device
    g = torch.Generator(device=dev).manual_seed(seed)
    for name, p in model.named_parameters():
        with torch.no_grad():
            if name.endswith("gamma"):
                continue
            if p.ndim == 1 and ("norm" in name):
                p.fill_(1.0 if name.endswith("weight") else 0.0)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.copy_(torch.randn(p.shape, generator=g, device=dev, dtype=p.dtype) * std)
    return model


def build_vit(seed: int = 0, device=None, **overrides) -> VisionTransformer:
    """A randomly initialised ViT (``init_weights``); ``device`` builds and initialises it there."""
    cfg = ViTConfig(**overrides)
    if device is None:
        return init_weights(VisionTransformer(cfg), seed=seed)
    with torch.device(device):
        model = VisionTransformer(cfg)
    return init_weights(model, seed=seed)
