"""GPU tests of the module layer: QuantLinear, FusedNVFP4MLP / fuse_mlps, the fused LayerNorm cast,
FusedNVFP4Block, and end-to-end ViT logits against the CPU oracle ViT.

Mirrors the reference's tests/test_qlinear.py:9-53 and tests/test_fused_mlp.py:22-123 (their
``requires_sm120`` gate becomes ``gpu``).  Tolerances are stated per test.
"""
import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from conftest import oracle, ROOT
from gpu_util import cos

pytestmark = pytest.mark.gpu


def _cos(a, b):
    return F.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0).item()


# ----------------------------------------------------------------------------- QuantLinear
def test_qlinear_matches_nvfp4_linear():
    from vitfp4.nvfp4 import nvfp4_linear, quantize_to_nvfp4
    from vitfp4.ptq import QuantLinear
    torch.manual_seed(0)
    lin = nn.Linear(256, 128).cuda().bfloat16()
    q = QuantLinear.from_linear(lin)
    x = torch.randn(4, 10, 256, device="cuda", dtype=torch.bfloat16)
    y = q(x)
    assert y.shape == (4, 10, 128)
    wc, wb, wg = quantize_to_nvfp4(lin.weight.data.float(), 16, block_select="mse")
    ref = nvfp4_linear(x.reshape(-1, 256), wc, wb, wg, bias=lin.bias).reshape(4, 10, 128)
    assert torch.equal(y, ref)


def test_qlinear_weights_bit_exact_with_oracle():
    from vitfp4.ptq import QuantLinear
    lin = nn.Linear(192, 96).cuda()
    q = QuantLinear.from_linear(lin)
    c, b, g = oracle.quantize_to_nvfp4(lin.weight.data.cpu().numpy(), 16, block_select="mse")
    assert np.array_equal(q.w_codes.cpu().numpy(), c)
    assert np.array_equal(q.w_block_scale.view(torch.uint8).cpu().numpy(), b)
    assert q.w_global_scale.item() == g


def test_qlinear_close_to_bf16():
    from vitfp4.ptq import QuantLinear
    lin = nn.Linear(512, 512).cuda().bfloat16()
    q = QuantLinear.from_linear(lin)
    x = torch.randn(64, 512, device="cuda", dtype=torch.bfloat16)
    assert _cos(q(x), lin(x)) > 0.99


def test_qlinear_static_global_scale_matches_dynamic_when_equal():
    from vitfp4.nvfp4 import quantize_to_nvfp4
    from vitfp4.ptq import QuantLinear
    lin = nn.Linear(256, 128).cuda().bfloat16()
    q = QuantLinear.from_linear(lin)
    x = torch.randn(4, 256, device="cuda", dtype=torch.bfloat16)
    y_dyn = q(x)
    _, _, gs = quantize_to_nvfp4(x.float(), 16)
    q.set_activation_scale(gs)
    assert torch.equal(y_dyn, q(x)) and q.x_global_scale is not None


def test_qlinear_no_bias_and_state_dict():
    from vitfp4.ptq import QuantLinear
    lin = nn.Linear(128, 64, bias=False).cuda().bfloat16()
    q = QuantLinear.from_linear(lin)
    assert q.bias is None
    x = torch.randn(8, 128, device="cuda", dtype=torch.bfloat16)
    y = q(x)
    assert y.shape == (8, 64)
    sd = q.state_dict()
    assert set(sd) == {"w_codes", "w_block_scale", "w_global_scale"}   # reference buffer names
    q2 = QuantLinear(torch.zeros_like(q.w_codes), torch.zeros_like(q.w_block_scale), torch.zeros((), device="cuda"),
                     None, 128, 64)
    q2(x)                                                   # builds (stale) packed weights
    q2.load_state_dict(sd)                                  # packed cache must follow the new buffers
    assert torch.equal(q2(x), y)


# ----------------------------------------------------------------------------- fused MLP
@pytest.mark.parametrize("M,E", [(8192, 1024), (197, 768), (17, 512)])
def test_fused_mlp_matches_bf16(M, E):
    from vitfp4.ptq import FusedNVFP4MLP
    torch.manual_seed(1)
    x = torch.randn(M, E, device="cuda", dtype=torch.bfloat16)
    fc1 = nn.Linear(E, 4 * E).cuda().bfloat16()
    fc2 = nn.Linear(4 * E, E).cuda().bfloat16()
    ref = fc2(F.gelu(fc1(x)))
    mlp = FusedNVFP4MLP(fc1, fc2)
    out = mlp(x)
    assert mlp.gx is not None and mlp.gh is not None
    assert out.dtype == torch.bfloat16 and _cos(ref, out) >= 0.97     # reference bar
    if M == 8192:
        assert _cos(ref, torch.compile(mlp)(x)) >= 0.97                # custom op survives torch.compile


@pytest.mark.parametrize("exact", [False, True])
def test_fused_mlp_matches_oracle_composition(exact):
    """FusedNVFP4MLP vs the reference's arithmetic (erf-GELU) composed on CPU: cos >= 0.999."""
    from vitfp4.ptq import FusedNVFP4MLP
    torch.manual_seed(2)
    M, E = 512, 256
    x = torch.randn(M, E, device="cuda", dtype=torch.bfloat16)
    fc1, fc2 = nn.Linear(E, 4 * E).cuda().bfloat16(), nn.Linear(4 * E, E).cuda().bfloat16()
    mlp = FusedNVFP4MLP(fc1, fc2, exact_gelu=exact)
    out = mlp(x).detach().float().cpu().numpy()
    xn = x.detach().float().cpu().numpy()
    gx, gh = np.float32(mlp.gx.item()), np.float32(mlp.gh.item())
    w1 = oracle.dequantize_nvfp4(*oracle.quantize_to_nvfp4(fc1.weight.detach().float().cpu().numpy(), 16))
    w2 = oracle.dequantize_nvfp4(*oracle.quantize_to_nvfp4(fc2.weight.detach().float().cpu().numpy(), 16))
    qx = oracle.dequantize_nvfp4(*oracle.quantize_to_nvfp4(xn, 16, global_scale=gx))
    h = oracle.gelu(qx @ w1.T + fc1.bias.detach().float().cpu().numpy())
    qh = oracle.dequantize_nvfp4(*oracle.quantize_to_nvfp4(h, 16, global_scale=gh))
    ref = qh @ w2.T + fc2.bias.detach().float().cpu().numpy()
    assert cos(out, ref) >= 0.999


def _block(act):
    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.fc1, self.act, self.fc2 = nn.Linear(256, 1024), act, nn.Linear(1024, 256)
    return Block()


def test_fuse_mlps_skips_ends():
    from vitfp4.ptq import FusedNVFP4MLP, fuse_mlps

    class Net(nn.Module):
        def __init__(self, n):
            super().__init__()
            self.blocks = nn.ModuleList(_block(nn.GELU()) for _ in range(n))
    model = Net(6).cuda().bfloat16()
    assert fuse_mlps(model, skip_ends=2) == 2
    assert [isinstance(b, FusedNVFP4MLP) for b in model.blocks] == [False, False, True, True, False, False]


def test_fuse_mlps_skips_gated_and_non_gelu():
    from vitfp4.ptq import FusedNVFP4MLP, fuse_mlps

    class Gated(nn.Module):
        def __init__(self):
            super().__init__()
            self.gate_proj, self.up_proj, self.down_proj = nn.Linear(256, 1024), nn.Linear(256, 1024), nn.Linear(1024, 256)

    class Net(nn.Module):
        def __init__(self):
            super().__init__()
            self.blocks = nn.ModuleList([Gated(), _block(nn.GELU(approximate="tanh")), Gated()])
    model = Net().cuda().bfloat16()
    with pytest.warns(UserWarning, match="not known to be erf-GELU"):
        assert fuse_mlps(model, skip_ends=0) == 0
    assert not any(isinstance(b, FusedNVFP4MLP) for b in model.blocks)


# ----------------------------------------------------------------------------- fused LayerNorm cast
@pytest.mark.parametrize("M,K", [(1, 1024), (257, 768), (1000, 1024), (333, 1280), (130, 384)])
@pytest.mark.parametrize("static", [False, True])
def test_ln_cast_matches_unfused(M, K, static):
    from vitfp4.nvfp4 import ops
    torch.manual_seed(M + K)
    x = (torch.randn(M, K, device="cuda") * 3).bfloat16()
    y = torch.randn(M, K, device="cuda").bfloat16()
    gamma = (torch.rand(K, device="cuda") * 0.1).bfloat16()
    ln = nn.LayerNorm(K, eps=1e-6).cuda().bfloat16()
    with torch.no_grad():
        ln.weight.copy_(torch.rand(K) + 0.5)
        ln.bias.copy_(torch.randn(K) * 0.1)
    x_ref = x + y * gamma                                  # bf16 ops, as the unfused block
    h_ref = ln(x_ref)
    gs = ops.global_scale(ops.amax(h_ref)) if static else None
    p_ref, sf_ref, _, g_ref = ops.cast(h_ref, gs, "six")
    p, sf, g, x_new = ops.ln_cast(x, ln.weight, ln.bias, ln.eps, gs=gs, y=y, gamma=gamma)
    torch.cuda.synchronize()
    assert torch.equal(x_new, x_ref)                       # residual + LayerScale bit-exact
    assert abs(g.item() - g_ref.item()) <= 1e-6 * g_ref.item()
    codes, codes_ref = oracle.unpack_e2m1(p.cpu().numpy()), oracle.unpack_e2m1(p_ref.cpu().numpy())
    # LayerNorm reduction order may move a bf16 rounding of h by one ulp: near-identity required
    assert (codes != codes_ref).mean() < 2e-3
    assert (sf.cpu().numpy() != sf_ref.cpu().numpy()).mean() < 2e-3
    p2, sf2, _, _ = ops.ln_cast(x_ref, ln.weight, ln.bias, ln.eps, gs=gs)      # no residual
    assert torch.equal(p2, p) and torch.equal(sf2, sf)
    if not static:
        # the dynamic route's cast pass reads the row statistics its amax pass left in the code
        # rows; casting again with the global it produced recomputes them in one kernel
        p3, sf3, _, _ = ops.ln_cast(x_ref, ln.weight, ln.bias, ln.eps, gs=g)
        assert torch.equal(p3, p) and torch.equal(sf3, sf)


# ----------------------------------------------------------------------------- fused block + model
def _small_vit(depth=4, seed=0):
    import sys
    sys.path.insert(0, ROOT)
    from vitfp4 import vit
    cfg = dict(vit.VIT_S16)
    cfg.update(depth=depth, init_values=1e-1)
    return vit.build_vit(seed=seed, **cfg).cuda().bfloat16().eval()


def _convert(model, attn="bf16", fuse_blocks=False):
    from vitfp4.ptq import enable_quant_attention, fuse_mlps, fuse_norms, quantize_vit, vit_attn_policy
    fuse_mlps(model, skip_ends=0)
    quantize_vit(model, 0, 0)
    if attn == "nvfp4":
        enable_quant_attention(model, vit_attn_policy(len(model.blocks), 0, 0, "blocks"), "nvfp4", "nvfp4")
    if fuse_blocks:
        assert fuse_norms(model) == len(model.blocks)
    return model


@pytest.mark.parametrize("attn", ["bf16", "nvfp4"])
def test_fused_block_matches_unfused_block(attn):
    """One converted block, fused vs per-module: same kernels' numerics, cos >= 0.999."""
    from vitfp4.ptq import FusedNVFP4Block
    torch.manual_seed(5)
    x = torch.randn(8, 197, 384, device="cuda").bfloat16()
    with torch.inference_mode():
        model = _convert(_small_vit(depth=1), attn)
        blk = model.blocks[0]
        a = blk(x)                                   # calibrates the MLP globals
        a = blk(x)
        b = FusedNVFP4Block(blk)(x)
    assert _cos(a, b) >= 0.999, _cos(a, b)


@pytest.mark.parametrize("S", [257, 264, 385])
def test_fused_block_bf16_attention_routes(S):
    """bf16 attention in the fused block equals the per-module block (torch SDPA): S <= 288 runs the
    tcgen05 bf16 kernel (S = 257 with its per-row tail, 264 with a partial 128-row tile); S = 385 =
    3 * 128 + 1 runs cuDNN on queries [0, 384) and on the last one separately and casts both parts
    into one proj operand."""
    from vitfp4.ptq import FusedNVFP4Block
    torch.manual_seed(6)
    x = torch.randn(4, S, 384, device="cuda").bfloat16()
    with torch.inference_mode():
        model = _convert(_small_vit(depth=1), "bf16")
        blk = model.blocks[0]
        a = blk(x)
        a = blk(x)
        b = FusedNVFP4Block(blk)(x)
    assert _cos(a, b) >= 0.999, _cos(a, b)


@pytest.mark.parametrize("gs", [None, 0.003])
def test_cast_split_equals_cast_of_concatenation(gs):
    from vitfp4.nvfp4 import ops
    torch.manual_seed(7)
    main = (torch.randn(6, 256, 1024, device="cuda") * 3).bfloat16()
    tail = (torch.randn(6, 1, 1024, device="cuda") * 5).bfloat16()
    g = None if gs is None else torch.tensor(gs, device="cuda")
    p1, s1, g1 = ops.cast_split(main, tail, gs=g)
    p2, s2, _, g2 = ops.cast(torch.cat([main, tail], 1).reshape(-1, 1024), g, "six")
    torch.cuda.synchronize()
    assert torch.equal(g1, g2) and torch.equal(p1, p2) and torch.equal(s1, s2)


@pytest.mark.parametrize("attn", ["bf16", "nvfp4"])
def test_fused_model_accuracy_matches_unfused(attn):
    """Whole model: FP4 is discontinuous (a one-ulp LayerNorm difference can move an E4M3 block scale
    and flip a block of codes, and this compounds over layers), so fused and per-module logits are
    compared through their accuracy against the bf16 model: no worse than 0.005 below per-module."""
    torch.manual_seed(5)
    x = torch.randn(8, 3, 224, 224, device="cuda").bfloat16()
    with torch.inference_mode():
        exact = _small_vit()(x)
        ref = _convert(_small_vit(), attn)
        fused = _convert(_small_vit(), attn, fuse_blocks=True)
        ref(x)   # calibrate the MLP globals on the same batch in both models
        fused(x)
        a, b = ref(x), fused(x)
    c_ref, c_fused = _cos(a, exact), _cos(b, exact)
    assert _cos(a, b) >= 0.98 and c_fused >= c_ref - 0.005, (_cos(a, b), c_ref, c_fused)


def test_model_logits_vs_oracle():
    """W4A4 ViT-S/16 (depth 4, bf16 attention) logits vs the CPU oracle ViT with the same weights."""
    import sys
    sys.path.insert(0, ROOT + "/oracle")
    import vit_oracle
    torch.manual_seed(6)
    model = _small_vit(depth=4, seed=3)
    W = {"cfg": dict(d=384, depth=4, heads=6, patch=16, img=224, hidden=1536, ls=0.1),
         "patch_w": model.patch_embed.proj.weight.detach().float().reshape(384, -1).cpu().numpy(),
         "cls": model.cls_token.detach().float().reshape(1, 384).cpu().numpy(),
         "pos": model.pos_embed.detach().float().reshape(-1, 384).cpu().numpy(),
         "head_w": model.head.weight.detach().float().cpu().numpy(), "blocks": []}
    for blk in model.blocks:
        d = {}
        for name, lin, mode in (("qkv", blk.attn.qkv, "mse"), ("proj", blk.attn.proj, "mse"),
                                ("fc1", blk.mlp.fc1, "six"), ("fc2", blk.mlp.fc2, "six")):
            w = lin.weight.detach().float().cpu().numpy()
            d[name] = oracle.dequantize_nvfp4(*oracle.quantize_to_nvfp4(w, 16, block_select=mode))
        d["gx"] = d["gh"] = None
        W["blocks"].append(d)
    images = torch.randn(4, 3, 224, 224).bfloat16()
    with torch.inference_mode():
        _convert(model)
        logits = model(images.cuda()).detach().float().cpu().numpy()
    ref = vit_oracle.forward(W, images.float().numpy())
    assert cos(logits, ref) >= 0.99, cos(logits, ref)
    print("logits cos vs oracle", cos(logits, ref))


# ----------------------------------------------------------------------------- composed W4A4 linear
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("static", [False, True])
@pytest.mark.parametrize("M,K,N", [(394, 768, 2304), (257, 3072, 768), (1, 1024, 1024)])
def test_qlinear_forward_matches_oracle(M, K, N, static, dtype):
    """QuantLinear.forward / nvfp4_linear (reference qlinear.py:42-47 -> gemm.py:32-38) against the oracle
    composed from the reference's steps: activation cast (six, dynamic or the static global),
    dequantize-and-matmul (backends/reference.py:6-10), output rounded to x.dtype, + bias in x.dtype.
    The activation codes and scales are bit-exact (held elsewhere); the GEMM's fp32 summation order
    differs, so the fp32 output is held to 1e-3 of max |ref| and cos >= 0.9999, the bf16 output to a
    bf16 step."""
    from vitfp4.nvfp4 import nvfp4_linear
    from vitfp4.ptq import QuantLinear
    torch.manual_seed(M + K)
    lin = nn.Linear(K, N).cuda()
    with torch.no_grad():
        lin.bias.copy_(torch.randn(N) * 0.1)
    lin = lin.to(dtype)
    q = QuantLinear.from_linear(lin)
    x = (torch.randn(M, K, device="cuda") * 2).to(dtype)
    x[:, 3] *= 20.0                                         # an outlier channel
    xn = x.float().cpu().numpy()
    gs = None
    if static:
        gs = np.float32(np.abs(xn).max() / 2688.0 * 0.8)   # a calibrated global that clips the outliers a bit
        q.set_activation_scale(torch.tensor(gs, device="cuda"))
    y = q(x)
    y2 = nvfp4_linear(x, q.w_codes, q.w_block_scale, q.w_global_scale, x_global_scale=q.x_global_scale,
                      bias=q.bias)
    assert y.dtype == dtype and torch.equal(y, y2)
    c, b, g = oracle.quantize_to_nvfp4(xn, 16, global_scale=gs)
    wc, wb, wg = (q.w_codes.cpu().numpy(), q.w_block_scale.view(torch.uint8).cpu().numpy(),
                  np.float32(q.w_global_scale.item()))
    acc = oracle.gemm_reference(c, b, g, wc, wb, wg)
    bias = lin.bias.detach().float().cpu().numpy()
    yn = y.float().cpu().numpy()
    if dtype == torch.float32:
        ref = acc + bias
        assert np.abs(yn - ref).max() <= 1e-3 * np.abs(ref).max() and cos(yn, ref) >= 0.9999
    else:
        ref = oracle.to_bf16(oracle.to_bf16(acc) + bias)
        step = np.abs(ref) * 2.0 ** -7 + 1e-6              # two bf16 roundings
        assert (np.abs(yn - ref) <= step).mean() >= 0.999 and cos(yn, ref) >= 0.9999


# ----------------------------------------------------------------------------- torch.compile contract
def test_custom_ops_trace_under_torch_compile_fullgraph():
    """vitfp4::cast_nvfp4, vitfp4::attention_lowp and vitfp4::fused_block are torch.library custom ops
    with fake implementations (the contract of the reference's fused MLP op, fused_mlp.py:38,58-61), so
    torch.compile(fullgraph=True) traces them without a graph break and runs the same kernels."""
    from vitfp4.nvfp4 import quant_sdpa
    torch.manual_seed(11)
    x = torch.randn(300, 256, device="cuda").bfloat16()
    gs = torch.tensor(0.004, device="cuda")
    cast = torch.compile(lambda t: torch.ops.vitfp4.cast_nvfp4(t, gs, False), fullgraph=True)
    p1, s1 = cast(x)
    p2, s2 = torch.ops.vitfp4.cast_nvfp4(x, gs, False)
    assert torch.equal(p1, p2) and torch.equal(s1, s2)
    q, k, v = (torch.randn(2, 3, 197, 64, device="cuda").bfloat16() for _ in range(3))
    for qk in ("nvfp4", "fp8"):
        att = torch.compile(lambda a, b, c: quant_sdpa(a, b, c, qk=qk, pv=qk), fullgraph=True)
        assert torch.equal(att(q, k, v), quant_sdpa(q, k, v, qk=qk, pv=qk))


def test_fused_model_under_torch_compile():
    """A converted model of fused blocks compiled end to end gives the eager logits (the blocks are opaque
    custom ops; the embedding, final LayerNorm and head are left to the compiler)."""
    torch.manual_seed(12)
    x = torch.randn(4, 3, 224, 224, device="cuda").bfloat16()
    with torch.no_grad():
        model = _convert(_small_vit(depth=2), fuse_blocks=True)
        eager = model(x)                    # calibrates the MLP globals
        eager = model(x)
        compiled = torch.compile(model)(x)
    assert _cos(eager, compiled) >= 0.9999, _cos(eager, compiled)


# ----------------------------------------------------------------------------- packed weight format
def test_qlinear_packed_state_dict_round_trip():
    """persist_packed(): the GEMM-ready bytes travel in state_dict and a loaded module uses them without
    repacking (no pack / swizzle launch); from_packed(): a module built from those bytes alone has the
    reference's codes and scales and computes the same output."""
    from vitfp4.nvfp4 import ops
    from vitfp4.ptq import QuantLinear
    torch.manual_seed(21)
    lin = nn.Linear(384, 1152).cuda().bfloat16()
    q = QuantLinear.from_linear(lin).persist_packed()
    x = torch.randn(197, 384, device="cuda").bfloat16()
    y = q(x)
    sd = q.state_dict()
    assert {"w_packed", "w_sf", "w_codes", "w_block_scale", "w_global_scale", "bias"} <= set(sd)
    q2 = QuantLinear(torch.zeros_like(q.w_codes), torch.zeros_like(q.w_block_scale), torch.zeros((), device="cuda"),
                     torch.zeros_like(q.bias), 384, 1152).persist_packed()
    q2.load_state_dict(sd)
    ops.probe.reset()
    q(x)                                    # packed already: the activation cast and the GEMM only
    n_ready = ops.probe.launches
    ops.probe.reset()
    y2 = q2(x)
    assert ops.probe.launches == n_ready    # nothing repacked after loading
    assert torch.equal(y, y2)
    q3 = QuantLinear.from_packed(sd["w_packed"], sd["w_sf"], sd["w_global_scale"], sd["bias"], 384, 1152)
    assert torch.equal(q3.w_codes, q.w_codes)
    assert torch.equal(q3.w_block_scale.view(torch.uint8), q.w_block_scale.view(torch.uint8))
    assert torch.equal(q3(x), y)
    # without persist_packed the state_dict keeps the reference's buffer names only
    assert "w_packed" not in QuantLinear.from_linear(lin).state_dict()
