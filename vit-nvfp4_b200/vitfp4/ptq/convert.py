"""In-place Linear -> QuantLinear conversion (reference: src/vit_nvfp4/ptq/convert.py:6-18)."""
import torch.nn as nn

from .qlinear import QuantLinear


def _replace(model: nn.Module, name: str, new: nn.Module) -> None:
    parent_name, _, attr = name.rpartition(".")
    parent = model.get_submodule(parent_name) if parent_name else model
    setattr(parent, attr, new)


def quantize_model(model: nn.Module, should_quantize, w_block_select: str = "mse") -> int:
    """Swap every module selected by ``should_quantize(name, module)`` for a QuantLinear.

    Weights are quantized once on the GPU (``w_block_select`` 'six' or Four-Over-Six 'mse').
    Returns the number of layers swapped."""
    picked = [(n, m) for n, m in model.named_modules() if should_quantize(n, m)]
    for name, module in picked:
        _replace(model, name, QuantLinear.from_linear(module, w_block_select=w_block_select))
    return len(picked)
