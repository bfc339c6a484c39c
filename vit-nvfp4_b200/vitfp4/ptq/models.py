"""Model-aware conversion config (reference: src/vit_nvfp4/ptq/models.py:16-79).

Finds the transformer block stack generically (the longest ModuleList whose first element
contains an nn.Linear), records a few structural quirks, and drives ``quantize_model``."""
from dataclasses import dataclass, field

import torch.nn as nn

from .convert import quantize_model
from .policy import vit_block_policy


@dataclass
class ModelSpec:
    arch: str
    block_container: str
    num_layers: int
    feature: str
    quirks: dict = field(default_factory=dict)


def _linear_stacks(model: nn.Module):
    out = []
    for name, mod in model.named_modules():
        if isinstance(mod, nn.ModuleList) and len(mod) and any(isinstance(s, nn.Linear) for s in mod[0].modules()):
            out.append((name, len(mod)))
    return out


def find_block_container(model: nn.Module) -> str:
    stacks = _linear_stacks(model)
    if not stacks:
        raise ValueError(f"no transformer block ModuleList found in {type(model).__name__}")
    return max(stacks, key=lambda s: s[1])[0]


def _quirks(block: nn.Module) -> dict:
    linear_names = [n for n, s in block.named_modules() if isinstance(s, nn.Linear)]
    type_names = [type(s).__name__ for _, s in block.named_modules()]
    leaf = [n.rsplit(".", 1)[-1] for n in linear_names]
    return {
        "fused_qkv": any("qkv" in n for n in linear_names),
        "swiglu": any("gate" in n for n in linear_names),
        "layerscale": any("LayerScale" in t for t in type_names),
        "rope": any(("Rope" in t or "RoPE" in t) for t in type_names),
        "out_proj": next((x for x in leaf if x in ("out_proj", "proj", "dense", "o_proj")), None),
    }


def model_spec(model: nn.Module) -> ModelSpec:
    container = find_block_container(model)
    blocks = model.get_submodule(container)
    arch = type(model).__name__
    has_cls = any(k in arch.lower() for k in ("dinov2", "dinov3"))  # CLS-token families
    return ModelSpec(arch=arch, block_container=container, num_layers=len(blocks),
                     feature="cls" if has_cls else "mean", quirks=_quirks(blocks[0]))


def quantize_vit(model: nn.Module, skip_first: int = 2, skip_last: int = 2, w_block_select: str = "mse"):
    """Quantize the middle blocks of a ViT to W4A4. Returns (n_swapped, spec)."""
    spec = model_spec(model)
    policy = vit_block_policy(spec.num_layers, skip_first, skip_last, container=spec.block_container)
    return quantize_model(model, policy, w_block_select=w_block_select), spec
