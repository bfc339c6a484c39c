"""GPU parity of the NVFP4 cast family (amax, global scale, cast, pack, swizzle) against the
oracle and the reference's golden fixtures — bit-exact codes, scale bytes and global scales."""
import numpy as np
import pytest
import torch

from conftest import golden, oracle
from gpu_util import bf16_tensor, vit_activation

pytestmark = pytest.mark.gpu


def _ops():
    from vitfp4.nvfp4 import ops
    return ops


def _run_cast(x_t, mode, gs=None, gelu=False, bias=None):
    packed, sfs, sfl, g = _ops().cast(x_t, gs, mode, gelu=gelu, bias=bias, swizzled=True, linear=True)
    torch.cuda.synchronize()
    return packed.cpu().numpy(), sfs.cpu().numpy(), sfl.cpu().numpy(), np.float32(g.item())


@pytest.mark.parametrize("name", list(golden()["q_cases"]))
def test_cast_matches_reference_golden(name):
    g = golden()
    x = g[f"q_{name}_x"]
    mse, static, bf16 = g[f"q_{name}_meta"]
    mode = "mse" if mse else "six"
    if int(bf16):
        xt = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    else:
        xt = torch.from_numpy(x).cuda()
    gs = None if static < 0 else torch.tensor(np.float32(static), device="cuda")
    packed, sfs, sfl, gsv = _run_cast(xt, mode, gs)
    codes, bs = g[f"q_{name}_codes"], g[f"q_{name}_bs"]
    assert gsv.tobytes() == np.float32(g[f"q_{name}_gs"]).tobytes()
    assert np.array_equal(sfl, bs), int((sfl != bs).sum())
    assert np.array_equal(packed, oracle.pack_e2m1(codes)), int((packed != oracle.pack_e2m1(codes)).sum())
    assert np.array_equal(sfs, oracle.to_blocked(bs))


@pytest.mark.parametrize("M,K", [(1, 16), (17, 80), (100, 768), (197, 1024), (300, 3072), (1025, 80)])
@pytest.mark.parametrize("mode", ["six", "mse"])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_cast_matches_oracle(M, K, mode, dtype):
    x = vit_activation(M, K, seed=M * 7 + K)
    if dtype == "bf16":
        xt = bf16_tensor(x)
        x = oracle.to_bf16(x)
    else:
        xt = torch.from_numpy(x).cuda()
    packed, sfs, sfl, gsv = _run_cast(xt, mode)
    c, b, g = oracle.quantize_to_nvfp4(x, 16, block_select=mode)
    assert gsv.tobytes() == np.float32(g).tobytes()
    assert np.array_equal(sfl, b), int((sfl != b).sum())
    assert np.array_equal(packed, oracle.pack_e2m1(c)), int((packed != oracle.pack_e2m1(c)).sum())
    assert np.array_equal(sfs, oracle.to_blocked(b))


def test_cast_exact_ties_and_boundaries():
    """Blocks whose max is 6*2^k with members exactly on, and one ulp around, every E2M1
    rounding boundary (global scale 1 -> block scale 2^k, decode exact): the reference rounds
    ties DOWN, so this pins the tie handling of the fast encoder bit-for-bit."""
    rng = np.random.default_rng(11)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    cand = np.concatenate([mids, np.nextafter(mids, 0), np.nextafter(mids, 10), [0.0, -0.0, 6.0, 0.5, 3.0]])
    rows, K = 512, 256
    x = np.empty((rows, K), np.float32)
    for r in range(rows):
        for b in range(K // 16):
            k = rng.integers(-8, 8)
            blk = rng.choice(cand, 16).astype(np.float32) * rng.choice([-1, 1], 16)
            blk[rng.integers(16)] = 6.0
            x[r, 16 * b:16 * b + 16] = blk * np.float32(2.0 ** k)
    xt = torch.from_numpy(x).cuda()
    packed, sfs, sfl, _ = _run_cast(xt, "six", torch.tensor(1.0, device="cuda"))
    c, b, _ = oracle.quantize_to_nvfp4(x, 16, global_scale=np.float32(1.0))
    assert np.array_equal(sfl, b)
    assert np.array_equal(packed, oracle.pack_e2m1(c)), int((packed != oracle.pack_e2m1(c)).sum())


def test_cast_near_boundary_and_underflow_bit_exact():
    """Elements whose quotient x/dec lands on, or within a few ulp of, every E2M1 rounding
    boundary for decode scales with full mantissas (the cast's bracketing fast path must hand
    these blocks to the exact path), bf16 inputs one bf16 step around the boundaries, -0.0 in
    every position, and fp32 blocks whose tiny negative members underflow x/dec to -0.0 (code 0
    in the reference, code 8 for a tiny negative quotient that does not underflow)."""
    rng = np.random.default_rng(21)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    rows, K = 1024, 256
    gs = np.float32(0.37)                                  # decode scales e4m3 * 0.37: full mantissas
    x = np.empty((rows, K), np.float32)
    for r in range(rows):
        for b in range(K // 16):
            amax = np.float32(np.exp2(rng.uniform(-4, 6)))
            bs = oracle.e4m3_decode(oracle.e4m3_encode(np.minimum(amax / np.float32(6) * (np.float32(1) / gs),
                                                                  np.float32(448))))
            dec = np.float32(bs * gs)
            m = rng.choice(mids, 16) * rng.choice([-1, 1], 16)
            q = (m * dec).astype(np.float32)
            steps = rng.integers(-3, 4, 16)
            q = np.array([np.float32(v) if s == 0 else
                          np.nextafter(v, np.float32(np.sign(s) * np.inf), dtype=np.float32) if abs(s) == 1 else
                          np.float32(v) + np.float32(s) * np.spacing(np.float32(v)) for v, s in zip(q, steps)],
                         np.float32)
            q[rng.integers(16)] = amax
            x[r, 16 * b:16 * b + 16] = q
    # fp32 input: full-precision quotients around the boundaries
    gt = torch.tensor(gs, device="cuda")
    packed, _, sfl, _ = _run_cast(torch.from_numpy(x).cuda(), "six", gt)
    c, b, _ = oracle.quantize_to_nvfp4(x, 16, global_scale=gs)
    assert np.array_equal(sfl, b)
    assert np.array_equal(packed, oracle.pack_e2m1(c)), int((packed != oracle.pack_e2m1(c)).sum())
    # bf16 input of the same data, with -0.0 sprinkled in
    xb = oracle.to_bf16(x)
    xb[rng.random(xb.shape) < 0.02] = -0.0
    packed, _, sfl, _ = _run_cast(bf16_tensor(xb), "six", gt)
    c, b, _ = oracle.quantize_to_nvfp4(xb, 16, global_scale=gs)
    assert np.array_equal(sfl, b) and np.array_equal(packed, oracle.pack_e2m1(c))
    # fp32 underflow of the quotient: block max 1e4 (decode scale 448 with gs=1) and tiny negatives
    xu = np.zeros((128, 64), np.float32)
    xu[:, 0] = 1e4
    xu[:, 1:] = -np.float32(1.4e-45) * rng.integers(1, 1000, (128, 63)).astype(np.float32)
    xu[::2, 1:] *= np.float32(1e6)                     # these quotients stay tiny but non-zero
    packed, _, sfl, _ = _run_cast(torch.from_numpy(xu).cuda(), "six", torch.tensor(1.0, device="cuda"))
    c, b, _ = oracle.quantize_to_nvfp4(xu, 16, global_scale=np.float32(1.0))
    assert (c == 0).any() and (c == 8).any()
    assert np.array_equal(sfl, b) and np.array_equal(packed, oracle.pack_e2m1(c))


def test_cast_random_scales_bit_exact():
    """2M elements with per-row magnitudes spanning 2^-30..2^30 (bf16 and fp32 inputs)."""
    rng = np.random.default_rng(12)
    x = (rng.standard_normal((4096, 512)) * np.exp2(rng.uniform(-30, 30, (4096, 1)))).astype(np.float32)
    for mode in ("six",):
        packed, _, sfl, gsv = _run_cast(torch.from_numpy(x).cuda(), mode)
        c, b, g = oracle.quantize_to_nvfp4(x, 16, block_select=mode)
        assert gsv == g and np.array_equal(sfl, b)
        assert np.array_equal(packed, oracle.pack_e2m1(c))
        xb = oracle.to_bf16(x)
        packed, _, sfl, gsv = _run_cast(bf16_tensor(x), mode)
        c, b, g = oracle.quantize_to_nvfp4(xb, 16, block_select=mode)
        assert gsv == g and np.array_equal(sfl, b) and np.array_equal(packed, oracle.pack_e2m1(c))


def test_cast_static_scale_and_strided_rows():
    x = vit_activation(64, 256, seed=3)
    big = np.zeros((64, 384), np.float32)
    big[:, :256] = x
    xt = bf16_tensor(big)[:, :256]            # row stride 384 elements
    gs = np.float32(np.abs(oracle.to_bf16(x)).max() / 2688.0 * 1.3)
    packed, sfs, sfl, gsv = _run_cast(xt, "six", torch.tensor(gs, device="cuda"))
    c, b, _ = oracle.quantize_to_nvfp4(oracle.to_bf16(x), 16, global_scale=gs)
    assert gsv == gs
    assert np.array_equal(sfl, b) and np.array_equal(packed, oracle.pack_e2m1(c))


def test_cast_gelu_and_bias():
    """GELU-fused cast == oracle(GELU(x + b)); erf ulp differences may flip a rare code."""
    x = vit_activation(256, 512, seed=5)
    bias = (np.random.default_rng(1).standard_normal(512) * 0.1).astype(np.float32)
    xt, bt = bf16_tensor(x), bf16_tensor(bias)
    xb = oracle.to_bf16(x) + oracle.to_bf16(bias)
    h = oracle.gelu(xb)
    gs = np.float32(np.abs(h).max() / 2688.0)
    packed, sfs, sfl, _ = _run_cast(xt, "six", torch.tensor(gs, device="cuda"), gelu=True, bias=bt)
    c, b, _ = oracle.quantize_to_nvfp4(h, 16, global_scale=gs)
    code_mismatch = (oracle.unpack_e2m1(packed) != c).mean()
    sf_mismatch = (sfl != b).mean()
    assert code_mismatch < 1e-3 and sf_mismatch < 1e-3, (code_mismatch, sf_mismatch)


def test_amax_and_global_scale():
    ops = _ops()
    x = vit_activation(333, 96, seed=9)
    xt = bf16_tensor(x)
    a = ops.amax(xt)
    assert np.float32(a.item()) == np.abs(oracle.to_bf16(x)).max()
    ag = ops.amax(xt, gelu=True)
    ref = np.abs(oracle.gelu(oracle.to_bf16(x))).max()
    assert abs(ag.item() - ref) <= 1e-6 * ref
    for mode, d in (("six", 2688.0), ("mse", 1536.0)):
        gs = ops.global_scale(a, mode)
        assert np.float32(gs.item()) == np.float32(np.float32(a.item()) / np.float32(d))
    odd = torch.randn(1001, device="cuda")                     # generic (unaligned-length) path
    assert ops.amax(odd).item() == odd.abs().max().item()


def test_pack_unpack_swizzle_golden():
    ops = _ops()
    g = golden()
    codes = torch.from_numpy(g["pack_codes"]).cuda()
    packed = ops.pack_e2m1(codes)
    assert np.array_equal(packed.cpu().numpy(), g["pack_packed"])
    assert torch.equal(ops.unpack_e2m1(packed), codes)
    for R, C in [(1, 1), (17, 3), (128, 4), (130, 5), (300, 48)]:
        out = ops.to_blocked(torch.from_numpy(g[f"blk_{R}x{C}_in"]).cuda())
        assert np.array_equal(out.cpu().numpy(), g[f"blk_{R}x{C}_out"])


def test_quantize_api_matches_reference_shapes():
    from vitfp4.nvfp4 import quantize_to_nvfp4, dequantize_nvfp4
    x = torch.randn(3, 5, 64, device="cuda")
    codes, bs, gs = quantize_to_nvfp4(x, 16)
    assert codes.dtype == torch.uint8 and codes.shape == (3, 5, 64)
    assert bs.dtype == torch.float8_e4m3fn and bs.shape == (3, 5, 4)
    assert gs.dtype == torch.float32 and gs.numel() == 1
    xh = dequantize_nvfp4(codes, bs, gs)
    c = torch.nn.functional.cosine_similarity(x.flatten(), xh.flatten(), dim=0)
    assert c > 0.98
    _, _, g2 = quantize_to_nvfp4(x, 16, global_scale=gs)
    assert torch.equal(gs, g2)


def test_cast_full_size_sampled_rows():
    """BASELINE config-2 cast (M=50432, K=3072): exact global scale and sampled-row parity."""
    M, K = 50432, 3072
    g = torch.Generator(device="cuda").manual_seed(0)
    xt = torch.randn(M, K, device="cuda", generator=g, dtype=torch.float32)
    ch = torch.randperm(K, generator=torch.Generator().manual_seed(0))[:4].cuda()
    xt[:, ch] *= 20
    xt = xt.to(torch.bfloat16)
    packed, sfs, _, gsv = _ops().cast(xt, None, "six")
    amax = np.float32(xt.float().abs().max().item())
    assert np.float32(gsv.item()) == np.float32(amax / np.float32(2688.0))
    rows = torch.randint(0, M, (64,), generator=torch.Generator().manual_seed(1))
    xs = xt[rows.cuda()].float().cpu().numpy()
    c, b, _ = oracle.quantize_to_nvfp4(xs, 16, global_scale=np.float32(gsv.item()))
    assert np.array_equal(packed[rows.cuda()].cpu().numpy(), oracle.pack_e2m1(c))
    sf_full = oracle.from_blocked(sfs.cpu().numpy(), M, K // 16)
    assert np.array_equal(sf_full[rows.numpy()], b)


@pytest.mark.parametrize("M,K,ld,mode,dtype,gelu", [
    (50432, 3072, 3072, "six", "bf16", False),    # BASELINE config-2 cast
    (1025, 80, 80, "mse", "f32", False),
    (300, 768, 1024, "six", "bf16", False),       # strided rows
    (197, 512, 512, "six", "bf16", True),         # GELU + bias prologue
])
def test_cast_index_widths_agree(M, K, ld, mode, dtype, gelu, monkeypatch):
    """The cast runs with 32-bit indices whenever every offset of the call fits; the 64-bit kernel
    (kept for larger tensors, forced here with VF4_CAST_INDEX64) writes the same bytes."""
    g = torch.Generator(device="cuda").manual_seed(M + K)
    full = torch.randn(M, ld, device="cuda", generator=g)
    xt = (full if dtype == "f32" else full.to(torch.bfloat16))[:, :K]
    bias = (torch.randn(K, device="cuda", generator=g) * 0.1).to(xt.dtype) if gelu else None
    gs = torch.tensor(float(xt.float().abs().max()) / 2688.0, device="cuda")
    outs = []
    for force64 in (False, True):
        if force64:
            monkeypatch.setenv("VF4_CAST_INDEX64", "1")
        packed, sfs, sfl, _ = _ops().cast(xt, gs, mode, gelu=gelu, bias=bias, swizzled=True, linear=True)
        torch.cuda.synchronize()
        outs.append((packed.cpu(), sfs.cpu(), sfl.cpu()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
