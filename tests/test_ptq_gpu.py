"""Host-side conversion steps on the GPU: static activation calibration (reference
src/vit_nvfp4/ptq/calibrate.py:35-68) and bias correction (src/vit_nvfp4/ptq/bias_correction.py:24-87)."""
import copy

import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu


def _mlp():
    torch.manual_seed(3)
    return nn.Sequential(nn.Linear(128, 256), nn.GELU(), nn.Linear(256, 64, bias=False)).cuda()


def test_calibrate_max_pins_amax_over_batches():
    from vitfp4.ptq import QuantLinear, calibrate_activations, quantize_model
    model = _mlp()
    quantize_model(model, lambda n, m: isinstance(m, nn.Linear), w_block_select="six")
    batches = [torch.randn(16, 128, device="cuda") * s for s in (1.0, 3.0, 0.5)]
    seen = []
    h = model[2].register_forward_pre_hook(lambda m, a: seen.append(a[0].abs().amax()))
    with torch.no_grad():
        ref0 = max(b.abs().amax() for b in batches)
        assert calibrate_activations(model, batches) == 2
    h.remove()
    assert torch.equal(model[0].x_global_scale, (ref0 / 2688.0).float())
    assert torch.equal(model[2].x_global_scale, (torch.stack(seen).amax() / 2688.0).float())
    assert isinstance(model[0], QuantLinear)
    with torch.no_grad():
        y = model(batches[0])             # static-global path runs
    assert torch.isfinite(y).all()


def test_calibrate_percentile_mode():
    from vitfp4.ptq import calibrate_activations, quantize_model
    model = _mlp()
    quantize_model(model, lambda n, m: isinstance(m, nn.Linear), w_block_select="six")
    batches = [torch.randn(64, 128, device="cuda") for _ in range(2)]
    calibrate_activations(model, batches, method="percentile", pct=0.99)
    ref = torch.stack([torch.quantile(b.abs().reshape(-1), 0.99) for b in batches]).mean() / 2688.0
    assert torch.allclose(model[0].x_global_scale, ref.float())


def test_correct_bias_folds_the_mean_shift():
    from vitfp4.ptq import correct_bias, quantize_model
    ref = _mlp()
    q = copy.deepcopy(ref)
    quantize_model(q, lambda n, m: isinstance(m, nn.Linear), w_block_select="six")
    batches = [torch.randn(512, 128, device="cuda") for _ in range(4)]
    x = torch.cat(batches)

    def mean_shift():
        with torch.no_grad():
            return (ref(x) - q(x)).mean(0).abs().mean().item()
    before = mean_shift()
    assert q[2].bias is None
    assert correct_bias(ref, q, batches) == 2
    assert q[2].bias is not None and q[2].bias.shape == (64,)
    after = mean_shift()
    print(f"mean output shift {before:.4e} -> {after:.4e}")
    assert after < 0.5 * before
