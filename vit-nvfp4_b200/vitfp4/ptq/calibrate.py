"""Static activation scales for QuantLinear (reference: src/vit_nvfp4/ptq/calibrate.py:11-68).

``calibrate_activations(model, batches, method='max', pct=0.999)`` runs the calibration ``batches``
through ``model`` with a forward pre-hook on every ``QuantLinear``, and then pins each layer's
static activation global scale (``set_activation_scale``) to ``amax / (6 * 448)``:

* ``method='max'``: amax is the largest |x| the layer saw over all batches (the CUDA amax kernel,
  one pass over each input);
* ``method='percentile'``: amax is the mean over batches of each batch's ``pct`` quantile of |x|
  (``torch.quantile`` on at most ~1M elements, every (numel // 1M)-th one), the reference's
  experimental mode.

With a static scale the layer's activation cast needs no amax pass per call.  Run it on the
per-module model (before ``fuse_norms``): the fused blocks read each QuantLinear's scale but do not
call its forward, so its hooks would not fire.  Returns the number of layers calibrated.
"""
from __future__ import annotations

import torch

from ..nvfp4 import ops
from .qlinear import QuantLinear

_SUBSAMPLE = 1_000_000


class _Observer:
    def __init__(self, method: str, pct: float):
        self.method, self.pct = method, pct
        self.values: list[torch.Tensor] = []

    def observe(self, x: torch.Tensor) -> None:
        if self.method == "max":
            self.values.append(ops.amax(x.detach()))
            return
        a = x.detach().abs().float().reshape(-1)
        if a.numel() > _SUBSAMPLE:
            a = a[:: a.numel() // _SUBSAMPLE]
        self.values.append(torch.quantile(a, self.pct))

    def amax(self) -> torch.Tensor:
        s = torch.stack(self.values)
        return s.amax() if self.method == "max" else s.mean()


@torch.no_grad()
def calibrate_activations(model, batches, method: str = "max", pct: float = 0.999) -> int:
    if method not in ("max", "percentile"):
        raise ValueError("method must be 'max' or 'percentile'")
    observed = [(m, _Observer(method, pct)) for m in model.modules() if isinstance(m, QuantLinear)]
    hooks = [m.register_forward_pre_hook(lambda mod, args, o=o: o.observe(args[0])) for m, o in observed]
    try:
        for batch in batches:
            model(**batch) if isinstance(batch, dict) else model(batch)
    finally:
        for h in hooks:
            h.remove()
    n = 0
    for m, o in observed:
        if o.values:
            m.set_activation_scale((o.amax() / 2688.0).float())
            n += 1
    return n
