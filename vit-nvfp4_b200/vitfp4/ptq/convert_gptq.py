"""Model conversion with GPTQ weights (reference: src/vit_nvfp4/ptq/convert_gptq.py:15-53).

``quantize_model_gptq(model, should_quantize, batches, percdamp=0.01, blocksize=128)`` runs the
calibration ``batches`` through the unconverted model once, collecting each selected Linear's input
Hessian with a forward pre-hook, then replaces every selected Linear by a ``QuantLinear`` whose codes
come from ``gptq_quantize_weight`` (on the GPU).  Returns the number of layers replaced.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .convert import _replace
from .gptq import HessianObserver, gptq_quantize_weight
from .qlinear import QuantLinear


@torch.no_grad()
def quantize_model_gptq(model: nn.Module, should_quantize, batches, percdamp: float = 0.01,
                        blocksize: int = 128) -> int:
    chosen = [(n, m) for n, m in model.named_modules() if should_quantize(n, m)]
    observers = {n: HessianObserver(m.in_features) for n, m in chosen}
    hooks = [m.register_forward_pre_hook(lambda mod, args, obs=observers[n]: obs.observe(args[0]))
             for n, m in chosen]
    try:
        for batch in batches:
            model(**batch) if isinstance(batch, dict) else model(batch)
    finally:
        for h in hooks:
            h.remove()
    for name, module in chosen:
        codes, bscale, gscale = gptq_quantize_weight(module.weight.data, observers[name].H, block=16,
                                                     percdamp=percdamp, blocksize=blocksize)
        _replace(model, name, QuantLinear(codes, bscale, gscale, module.bias, module.in_features,
                                          module.out_features))
    return len(chosen)
