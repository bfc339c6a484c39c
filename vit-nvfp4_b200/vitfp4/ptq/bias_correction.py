"""Bias correction for QuantLinear (reference: src/vit_nvfp4/ptq/bias_correction.py:24-87).

``correct_bias(ref_model, quant_model, batches)`` measures, for every ``QuantLinear`` of
``quant_model``, the mean over calibration tokens of (float layer output - quantized layer output)
on the input the quantized layer actually receives, and adds that per-output-feature shift to the
layer's bias (creating a bias when the layer has none), so the corrected layer's mean output matches
the float layer's (arXiv:2006.10518).  The float output is recomputed in fp32 from the matching
``nn.Linear`` of ``ref_model`` (same module name).  Run it after weight quantization and activation
calibration, on the per-module model (before ``fuse_norms``: the fused blocks do not call the
QuantLinear forward that the hooks observe).  Returns the number of layers corrected.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .qlinear import QuantLinear


@torch.no_grad()
def correct_bias(ref_model, quant_model, batches) -> int:
    floats = dict(ref_model.named_modules())
    layers = {name: m for name, m in quant_model.named_modules() if isinstance(m, QuantLinear)}
    sums: dict[str, torch.Tensor] = {}
    counts = dict.fromkeys(layers, 0)
    dtypes: dict[str, torch.dtype] = {}

    def hook_for(name):
        lin = floats[name]
        w = lin.weight.detach().float()
        b = None if lin.bias is None else lin.bias.detach().float()

        def hook(mod, args, out):
            shift = (F.linear(args[0].float(), w, b) - out.float()).reshape(-1, mod.out_features)
            s = shift.sum(0)
            sums[name] = s if name not in sums else sums[name] + s
            counts[name] += shift.shape[0]
            dtypes[name] = out.dtype
        return hook

    hooks = [m.register_forward_hook(hook_for(name)) for name, m in layers.items()]
    try:
        for batch in batches:
            quant_model(**batch) if isinstance(batch, dict) else quant_model(batch)
    finally:
        for h in hooks:
            h.remove()
    n = 0
    for name, m in layers.items():
        if not counts[name]:
            continue
        shift = sums[name] / counts[name]
        if m.bias is None:
            del m.bias                                  # a plain None attribute until now
            m.register_buffer("bias", shift.to(dtypes[name]))
        else:
            m.bias.add_(shift.to(m.bias.dtype))
        n += 1
    return n
