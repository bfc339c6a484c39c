"""Whole-model parity on the GPU.

1. BASELINE configuration 1 (ViT-S/16, 12 blocks, RTN weights, every block Linear a QuantLinear) against
   the reference's own outputs (``tests/golden/golden_vit.npz``, made from the reference on CPU):
   * blocks 0 and 11 on one synthetic block input: the block's contribution (output - input) to
     cos >= 0.99999 (fp32) / 0.995 (bf16) -- the same bars the oracle meets against the reference;
   * logits of the 8 images: within the reference's own spread under a one-ulp input change (W4A4
     is chaotic over 12 blocks without LayerScale, see tests/test_vit_golden.py), and the same
     accuracy against the unquantized model as the reference's.
2. The headline composition (fused MLPs with the erf-GELU epilogue, fused blocks, bf16 attention
   kernel) teacher-forced against the oracle: every block of the configuration-1 model fed the
   GPU's own block input, contribution cos >= 0.995.
3. BASELINE configuration 4 (the benchmark's DINOv2-style ViT-L/14, 24 blocks, LayerScale 1e-5), two
   images end to end against the oracle: logits cos >= 0.999 and the same top-1 class.
The oracle reads the quantized weights from the converted model itself (the weight cast is held
bit-exact to the oracle in tests/test_cast_gpu.py), so these compare activations, GEMMs and glue.
"""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import ROOT, oracle

sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

import vit_oracle  # noqa: E402
from make_golden_vit import BLOCKS, block_input, config1_images, config1_model  # noqa: E402

pytestmark = pytest.mark.gpu

DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16}
BLOCK_DELTA_BAR = {"f32": 0.99999, "bf16": 0.995}
BLOCK_OUT_BAR = {"f32": 0.999999, "bf16": 0.9999}


def _cos(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


def _np(t):
    return None if t is None else t.detach().float().cpu().numpy()


def _golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden_vit.npz")))


# ----------------------------------------------------------------------------- oracle weights
def _deq_qlinear(q):
    return oracle.dequantize_nvfp4(q.w_codes.cpu().numpy(), q.w_block_scale.view(torch.uint8).cpu().numpy(),
                                   np.float32(q.w_global_scale.item()))


def _deq_packed(wq, wsf, wg, n, k):
    codes = oracle.unpack_e2m1(wq.view(torch.uint8).cpu().numpy())
    scales = oracle.from_blocked(wsf.view(torch.uint8).reshape(-1).cpu().numpy(), n, k // 16)
    return oracle.dequantize_nvfp4(codes, scales, np.float32(wg.item()))


def oracle_weights(model):
    """Oracle weights of a converted vitfp4.vit model (QuantLinear / FusedNVFP4MLP / FusedNVFP4Block)."""
    from vitfp4.ptq import FusedNVFP4MLP
    cfg = model.config
    d = cfg.embed_dim
    W = {"cfg": dict(d=d, depth=len(model.blocks), heads=cfg.num_heads, patch=cfg.patch_size, img=cfg.img_size,
                     hidden=int(d * cfg.mlp_ratio), ls=None, eps=cfg.layer_norm_eps),
         "patch_w": _np(model.patch_embed.proj.weight).reshape(d, -1), "patch_b": _np(model.patch_embed.proj.bias),
         "cls": _np(model.cls_token).reshape(1, d), "pos": _np(model.pos_embed).reshape(-1, d),
         "norm": (_np(model.norm.weight), _np(model.norm.bias)), "head_w": _np(model.head.weight),
         "head_b": _np(model.head.bias), "blocks": []}
    for blk in model.blocks:
        e = {"norm1": (_np(blk.norm1.weight), _np(blk.norm1.bias)), "norm2": (_np(blk.norm2.weight), _np(blk.norm2.bias)),
             "ls1": _np(getattr(blk.ls1, "gamma", None)), "ls2": _np(getattr(blk.ls2, "gamma", None)),
             "qkv": _deq_qlinear(blk.attn.qkv), "qkv_b": _np(blk.attn.qkv.bias),
             "proj": _deq_qlinear(blk.attn.proj), "proj_b": _np(blk.attn.proj.bias), "gx": None, "gh": None}
        mlp = blk.mlp
        if isinstance(mlp, FusedNVFP4MLP):
            n1 = mlp.w1q.shape[0]
            e["fc1"] = _deq_packed(mlp.w1q, mlp.w1sf, mlp.w1g, n1, mlp.k1)
            e["fc2"] = _deq_packed(mlp.w2q, mlp.w2sf, mlp.w2g, mlp.n2, n1)
            e["fc1_b"], e["fc2_b"] = _np(mlp.b1), _np(mlp.b2)
            if mlp.gx is not None:
                e["gx"], e["gh"] = np.float32(mlp.gx.item()), np.float32(mlp.gh.item())
        else:
            e["fc1"], e["fc2"] = _deq_qlinear(mlp.fc1), _deq_qlinear(mlp.fc2)
            e["fc1_b"], e["fc2_b"] = _np(mlp.fc1.bias), _np(mlp.fc2.bias)
        W["blocks"].append(e)
    return W


def _per_module(prec):
    from vitfp4.ptq import quantize_vit
    model = config1_model(DTYPES[prec]).cuda()
    n, _ = quantize_vit(model, skip_first=0, skip_last=0, w_block_select="six")
    assert n == 48
    return model


# ----------------------------------------------------------------------------- 1. configuration 1
@pytest.mark.parametrize("prec", ["f32", "bf16"])
def test_config1_blocks_vs_reference(prec):
    g = _golden()
    model = _per_module(prec)
    x = block_input(DTYPES[prec]).cuda()
    xn = _np(x)
    with torch.inference_mode():
        for i in BLOCKS:
            out = _np(model.blocks[i](x))
            ref = g[f"c1_{prec}_blk{i}_out"]
            c_out, c_delta = _cos(out, ref), _cos(out - xn, ref - xn)
            print(f"block {i} {prec}: output cos {c_out:.7f}, contribution cos {c_delta:.7f}")
            assert c_out >= BLOCK_OUT_BAR[prec] and c_delta >= BLOCK_DELTA_BAR[prec], (i, c_out, c_delta)


@pytest.mark.parametrize("prec", ["f32", "bf16"])
def test_config1_logits_vs_reference(prec):
    g = _golden()
    model = _per_module(prec)
    with torch.inference_mode():
        out = _np(model(config1_images(DTYPES[prec]).cuda()))
    ref, exact = g[f"c1_{prec}_logits"], g[f"c1_{prec}_exact_logits"]
    spread = _cos(ref, g[f"c1_{prec}_pert_logits"])
    top1 = float((out.argmax(1) == ref.argmax(1)).mean())
    print(f"{prec}: logits cos vs reference {_cos(out, ref):.5f} (reference vs itself one ulp away {spread:.5f}), "
          f"top-1 agreement {top1:.3f}, cos vs unquantized {_cos(out, exact):.5f} (reference {_cos(ref, exact):.5f})")
    assert _cos(out, ref) >= spread - 0.03
    assert abs(_cos(out, exact) - _cos(ref, exact)) <= 0.02


# ----------------------------------------------------------------------------- 2. headline path, per block
def _headline(model):
    from vitfp4.ptq import fuse_mlps, fuse_norms, quantize_vit
    n_mlp = fuse_mlps(model, skip_ends=0)
    quantize_vit(model, skip_first=0, skip_last=0, w_block_select="mse")
    assert fuse_norms(model) == len(model.blocks) == n_mlp
    assert all(b.mlp.exact_gelu for b in model.blocks)          # the reference's GELU by default
    return model


def test_headline_blocks_teacher_forced_vs_oracle():
    model = _headline(config1_model(torch.bfloat16).cuda())
    images = config1_images(torch.bfloat16).cuda()
    seen = {}
    hooks = [b.register_forward_hook(lambda m, i, o, k=k: seen.__setitem__(k, (_np(i[0]), _np(o))))
             for k, b in enumerate(model.blocks)]
    with torch.inference_mode():
        model(images)            # calibrates the MLP globals
        model(images)
    for h in hooks:
        h.remove()
    W = oracle_weights(model)
    res = []
    for k, blk in enumerate(W["blocks"]):
        x_in, out = seen[k]
        ref = vit_oracle.block_forward(blk, W["cfg"], x_in, precision="bf16", mlp="fused")
        res.append((_cos(out, ref), _cos(out - x_in, ref - x_in)))
    print("headline blocks vs oracle (output cos, contribution cos):", [f"{a:.5f}/{b:.5f}" for a, b in res])
    for k, (c_out, c_delta) in enumerate(res):
        assert c_out >= 0.9995 and c_delta >= 0.995, (k, c_out, c_delta)


# ----------------------------------------------------------------------------- 3. configuration 4
def test_vit_l14_logits_vs_oracle():
    from vitfp4 import vit
    model = _headline(vit.build_vit(seed=0, **vit.VIT_L14).cuda().bfloat16().eval())
    gen = torch.Generator().manual_seed(3)
    images = torch.randn(2, 3, 224, 224, generator=gen).bfloat16()
    with torch.inference_mode():
        model(images.cuda())
        out = _np(model(images.cuda()))
    W = oracle_weights(model)
    ref = vit_oracle.forward(W, images.float().numpy(), precision="bf16", mlp="fused")
    print(f"ViT-L/14: logits cos vs oracle {_cos(out, ref):.6f}")
    assert _cos(out, ref) >= 0.999
    assert (out.argmax(1) == ref.argmax(1)).all()
