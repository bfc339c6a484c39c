"""Model-aware conversion config: which ``nn.ModuleList`` is the transformer block stack of a ViT,
how deep it is, and which structural features its blocks have (the behaviour of the reference's
src/vit_nvfp4/ptq/models.py:16-79; ``quantize_vit`` keeps its signature and return value).

The stack is found by one walk over the module tree: every ``ModuleList`` whose first element holds
an ``nn.Linear`` is a candidate, and the deepest one wins (the first of equal depth), which picks the
encoder over auxiliary stacks such as a predictor or a merger list.  Features are read from the first
block in the same spirit: a single pass that classifies each submodule by its name and type.
"""
from dataclasses import dataclass, field

import torch.nn as nn

from .convert import quantize_model
from .policy import vit_block_policy

# leaf names that an attention output projection goes by in timm, HF and DINO-style blocks
_OUT_PROJ_NAMES = ("out_proj", "proj", "dense", "o_proj")
# architectures that prepend a class token (their retrieval feature is that token; others pool)
_CLS_TOKEN_ARCHS = ("dinov2", "dinov3")


@dataclass
class ModelSpec:
    arch: str
    block_container: str          # dotted path of the block stack
    num_layers: int
    feature: str                  # "cls" or "mean": how a retrieval feature pools the last hidden state
    quirks: dict = field(default_factory=dict)


def _holds_linear(module: nn.Module) -> bool:
    return any(isinstance(m, nn.Linear) for m in module.modules())


def find_block_container(model: nn.Module) -> str:
    """Dotted path of the deepest ``ModuleList`` whose first block contains an ``nn.Linear``."""
    best_name, best_len = None, 0
    for name, mod in model.named_modules():
        if isinstance(mod, nn.ModuleList) and len(mod) > best_len and _holds_linear(mod[0]):
            best_name, best_len = name, len(mod)
    if best_name is None:
        raise ValueError(f"no transformer block ModuleList found in {type(model).__name__}")
    return best_name


def _block_features(block: nn.Module) -> dict:
    """Structural features of one block, from a single pass over its submodules."""
    feats = {"fused_qkv": False, "swiglu": False, "layerscale": False, "rope": False, "out_proj": None}
    for name, mod in block.named_modules():
        tname = type(mod).__name__
        if "LayerScale" in tname:
            feats["layerscale"] = True
        if "Rope" in tname or "RoPE" in tname:
            feats["rope"] = True
        if not isinstance(mod, nn.Linear):
            continue
        feats["fused_qkv"] |= "qkv" in name
        feats["swiglu"] |= "gate" in name
        leaf = name.rpartition(".")[2]
        if feats["out_proj"] is None and leaf in _OUT_PROJ_NAMES:
            feats["out_proj"] = leaf
    return feats


def model_spec(model: nn.Module) -> ModelSpec:
    """Conversion config of ``model`` (the module later passed to ``quantize_model``)."""
    path = find_block_container(model)
    stack = model.get_submodule(path)
    arch = type(model).__name__
    feature = "cls" if any(tag in arch.lower() for tag in _CLS_TOKEN_ARCHS) else "mean"
    return ModelSpec(arch=arch, block_container=path, num_layers=len(stack), feature=feature,
                     quirks=_block_features(stack[0]))


def quantize_vit(model: nn.Module, skip_first: int = 2, skip_last: int = 2, w_block_select: str = "mse"):
    """Convert the middle blocks of a ViT to W4A4 ``QuantLinear``s; returns (n_swapped, spec)."""
    spec = model_spec(model)
    policy = vit_block_policy(spec.num_layers, skip_first, skip_last, container=spec.block_container)
    return quantize_model(model, policy, w_block_select=w_block_select), spec
