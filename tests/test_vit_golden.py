"""CPU checks of the whole-model oracle against the reference's own outputs (
``tests/golden/golden_vit.npz`` made by ``tests/golden/make_golden_vit.py`` from the reference), and of
the host-side model inspection (block-stack discovery, MLP fusion plan) that needs no GPU.

What the fixture shows, and how the bars follow from it:
  * On identical block inputs the oracle's block equals the reference's: the contribution of a block
    (output - input) agrees to cos >= 0.99999 in fp32 and >= 0.995 in bf16 (where torch's and
    numpy's bf16 roundings differ in the last bit of some elements).
  * End to end, the W4A4 model is chaotic: moving every input element one ulp changes the
    reference's OWN logits to cos ~0.97 (fp32) / ~0.95 (bf16), because FP4 rounding is
    discontinuous and the flipped codes compound over 12 blocks without LayerScale.  Logits of two
    implementations that differ in fp32 summation order therefore cannot agree better than that;
    the end-to-end bar is set from this measured spread, and the tight bar sits at block level.
"""
import os
import sys
import warnings

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import ROOT

sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

import vit_oracle  # noqa: E402
from make_golden_vit import BLOCKS, block_input, config1_images, config1_model  # noqa: E402


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden_vit.npz")))


DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16}
BLOCK_DELTA_BAR = {"f32": 0.99999, "bf16": 0.995}
BLOCK_OUT_BAR = {"f32": 0.999999, "bf16": 0.9999}


@pytest.mark.parametrize("prec", ["f32", "bf16"])
def test_oracle_blocks_match_reference(prec):
    g = _golden()
    W = vit_oracle.weights_from_model(config1_model(DTYPES[prec]), "six")
    x = block_input(DTYPES[prec]).float().numpy()
    for i in BLOCKS:
        out = vit_oracle.block_forward(W["blocks"][i], W["cfg"], x, precision=prec, mlp="qlinear")
        ref = g[f"c1_{prec}_blk{i}_out"]
        assert _cos(out, ref) >= BLOCK_OUT_BAR[prec], (i, _cos(out, ref))
        assert _cos(out - x, ref - x) >= BLOCK_DELTA_BAR[prec], (i, _cos(out - x, ref - x))


@pytest.mark.parametrize("prec", ["f32", "bf16"])
def test_reference_logits_move_under_one_ulp_input_change(prec):
    """The recorded fact the end-to-end bars rest on (no tolerance is chosen here)."""
    g = _golden()
    self_cos = _cos(g[f"c1_{prec}_logits"], g[f"c1_{prec}_pert_logits"])
    assert self_cos < 0.99, self_cos
    # quantization itself moves the logits further from the unquantized model than that
    assert _cos(g[f"c1_{prec}_logits"], g[f"c1_{prec}_exact_logits"]) < 0.97


def test_oracle_logits_vs_reference_f32():
    """End to end the oracle is one more draw from the reference's own spread."""
    g = _golden()
    W = vit_oracle.weights_from_model(config1_model(torch.float32), "six")
    out = vit_oracle.forward(W, config1_images(torch.float32).numpy(), precision="f32", mlp="qlinear")
    ref = g["c1_f32_logits"]
    spread = _cos(ref, g["c1_f32_pert_logits"])
    assert _cos(out, ref) >= spread - 0.03, (_cos(out, ref), spread)
    # same accuracy against the unquantized model as the reference's, within the spread
    exact = g["c1_f32_exact_logits"]
    assert abs(_cos(out, exact) - _cos(ref, exact)) <= 0.02


# ----------------------------------------------------------------------------- host-side inspection
def test_model_spec_of_the_vit():
    from vitfp4 import vit
    from vitfp4.ptq import model_spec
    m = vit.build_vit(seed=0, img_size=32, patch_size=16, embed_dim=64, depth=3, num_heads=2, init_values=1e-5)
    spec = model_spec(m)
    assert spec.block_container == "blocks" and spec.num_layers == 3
    assert spec.feature == "mean"
    assert spec.quirks == {"fused_qkv": True, "swiglu": False, "layerscale": True, "rope": False,
                           "out_proj": "proj"}


def test_find_block_container_prefers_the_deepest_stack():
    from vitfp4.ptq import find_block_container

    class Blk(nn.Module):
        def __init__(self):
            super().__init__()
            self.o_proj = nn.Linear(16, 16)

    class Dinov2Like(nn.Module):
        def __init__(self):
            super().__init__()
            self.predictor = nn.ModuleList(Blk() for _ in range(2))
            self.encoder = nn.Module()
            self.encoder.layer = nn.ModuleList(Blk() for _ in range(4))
            self.norms = nn.ModuleList(nn.LayerNorm(16) for _ in range(9))   # no Linear: never a stack

    from vitfp4.ptq import model_spec
    m = Dinov2Like()
    assert find_block_container(m) == "encoder.layer"
    spec = model_spec(m)
    assert spec.feature == "cls" and spec.quirks["out_proj"] == "o_proj" and not spec.quirks["fused_qkv"]
    with pytest.raises(ValueError):
        find_block_container(nn.Sequential(nn.Linear(4, 4)))


class _Mlp(nn.Module):
    def __init__(self, act, up="fc1", down="fc2", gated=False, k=32):
        super().__init__()
        setattr(self, up, nn.Linear(k, 64))
        self.act = act
        setattr(self, down, nn.Linear(64, k))
        if gated:
            self.gate_proj = nn.Linear(k, 64)


class _GELUActivation(nn.Module):      # stands in for HF's class of that name (matched by name)
    pass


_GELUActivation.__name__ = "GELUActivation"


def _model(acts):
    m = nn.Module()
    m.blocks = nn.ModuleList()
    for a in acts:
        b = nn.Module()
        b.mlp = a if isinstance(a, nn.Module) and hasattr(a, "act") else _Mlp(a)
        m.blocks.append(b)
    return m


def test_mlp_fusion_plan_selects_erf_gelu_mlps_only():
    from vitfp4.ptq.fused_mlp import plan_mlp_fusion
    m = _model([nn.GELU(), nn.GELU("tanh"), _GELUActivation(), nn.ReLU(), _Mlp(nn.GELU(), gated=True),
                _Mlp(nn.GELU(), "up_proj", "down_proj"), _Mlp(nn.GELU(), k=24)])
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        plan = plan_mlp_fusion(m, skip_ends=0)
    # gated MLPs and K % 16 != 0 are never candidates; tanh-GELU and ReLU are left out with a warning
    assert [n for n, _, _ in plan] == ["blocks.0.mlp", "blocks.2.mlp", "blocks.5.mlp"]
    assert len(w) == 1 and "2 MLP(s)" in str(w[0].message)
    forced = plan_mlp_fusion(m, skip_ends=0, require_gelu=False)
    assert [n for n, _, _ in forced] == ["blocks.0.mlp", "blocks.1.mlp", "blocks.2.mlp", "blocks.3.mlp",
                                         "blocks.5.mlp"]
    assert all(isinstance(f1, nn.Linear) and f1.out_features == f2.in_features for _, f1, f2 in plan)


def test_mlp_fusion_plan_skip_ends():
    from vitfp4.ptq.fused_mlp import plan_mlp_fusion
    m = _model([nn.GELU() for _ in range(6)])
    assert [n for n, _, _ in plan_mlp_fusion(m, skip_ends=2)] == ["blocks.2.mlp", "blocks.3.mlp"]
    with pytest.raises(ValueError):
        plan_mlp_fusion(m, skip_ends=3)
