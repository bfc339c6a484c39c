"""GPU parity of the tcgen05 block-scaled FP4 GEMM against the oracle (the reference's fp32
emulated GEMM, backends/reference.py:6-10).

Tolerances (fp32 accumulation order differs from the emulation, operands are identical):
  fp32 out: max |out - ref| <= 1e-3 * max|ref| and cosine >= 0.9999
  bf16 out: cosine >= 0.9999 and max error <= 1 bf16 ulp of max|ref| (2^-7 relative)
"""
import numpy as np
import pytest
import torch

from conftest import oracle
from gpu_util import cos, oracle_operand, to_cuda_operand, vit_activation

pytestmark = pytest.mark.gpu


def _ops():
    from vitfp4.nvfp4 import ops
    return ops


def _operands(M, N, K, seed=0, a_mode="six", b_mode="mse", dist="normal"):
    rng = np.random.default_rng(seed)
    a = vit_activation(M, K, seed=seed)
    if dist == "heavy":
        a = a * rng.exponential(0.5, size=a.shape).astype(np.float32)
    elif dist == "outlier":
        a[:2] *= 30.0
    b = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    A = oracle_operand(a, a_mode)
    B = oracle_operand(b, b_mode)
    return A, B


def _gemm_cuda(A, B, out_dtype=torch.float32, bias=None):
    ops = _ops()
    ap, asf, ag = to_cuda_operand(A[3], A[4], A[2])
    bp, bsf, bg = to_cuda_operand(B[3], B[4], B[2])
    bt = None if bias is None else torch.from_numpy(bias).cuda().to(torch.bfloat16)
    out = ops.gemm(ap, asf, ag, bp, bsf, bg, bias=bt, out_dtype=out_dtype)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


SHAPES = [  # (M, K, N)
    (128, 64, 128), (256, 512, 768), (256, 1024, 1024), (1024, 1152, 4304), (512, 1408, 6144),
    (17, 512, 768), (100, 1024, 4096), (197, 768, 2304), (333, 3072, 768), (64, 256, 64),
    (130, 96, 144), (1, 32, 16), (257, 1024, 3072),
]


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_gemm_fp32_matches_emulation(M, K, N):
    A, B = _operands(M, N, K, seed=M + N + K)
    out = _gemm_cuda(A, B)
    ref = oracle.gemm_reference(A[0], A[1], A[2], B[0], B[1], B[2])
    err = np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30)
    assert not (out == 0).all()
    assert err <= 1e-3 and cos(out, ref) >= 0.9999, (err, cos(out, ref))


@pytest.mark.parametrize("dist", ["normal", "heavy", "outlier"])
def test_gemm_distributions(dist):
    A, B = _operands(256, 1024, 1024, seed=11, dist=dist)
    out = _gemm_cuda(A, B)
    ref = oracle.gemm_reference(A[0], A[1], A[2], B[0], B[1], B[2])
    assert cos(out, ref) >= 0.9999


@pytest.mark.parametrize("M,K,N", [(256, 512, 768), (197, 1024, 3072), (100, 256, 128)])
def test_gemm_bf16_bias(M, K, N):
    A, B = _operands(M, N, K, seed=5)
    bias = (np.random.default_rng(2).standard_normal(N) * 0.1).astype(np.float32)
    out = _gemm_cuda(A, B, out_dtype=torch.bfloat16, bias=bias)
    ref = oracle.to_bf16(oracle.to_bf16(oracle.gemm_reference(A[0], A[1], A[2], B[0], B[1], B[2]))
                         + oracle.to_bf16(bias))
    assert cos(out, ref) >= 0.9999
    assert np.abs(out - ref).max() <= 2.0 ** -7 * np.abs(ref).max()


def _gelu_tanh(x):
    x = x.astype(np.float64)
    return (0.5 * x * (1 + np.tanh(0.7978845608 * x + 0.0356774081 * x ** 3))).astype(np.float32)


@pytest.mark.parametrize("exact", [False, True])
@pytest.mark.parametrize("M,K,N", [(256, 1024, 4096), (197, 768, 3072), (130, 512, 128)])
def test_gemm_gelu_nvfp4_epilogue(M, K, N, exact):
    """fc1 epilogue NVFP4(GELU(gemm + b1)) with a static global scale, the reference's fused-MLP step
    (fused_mlp.py:47-51).  exact (the default of FusedNVFP4MLP): the GEMM rounded to bf16, + b1 in bf16,
    erf-GELU, the Triton cast's arithmetic -- compared with the oracle's restatement of exactly those
    steps, so only fp32 summation order (which can move a bf16 rounding) and the kernel's erf (within
    2.5e-7 |x|) separate them: codes and scales agree on all but < 2e-4 of the elements.  The tanh
    form (no roundings, hardware tanh) is compared with its own function at < 2e-3."""
    ops = _ops()
    A, B = _operands(M, N, K, seed=7)
    bias = (np.random.default_rng(3).standard_normal(N) * 0.1).astype(np.float32)
    ref_y = oracle.gemm_reference(A[0], A[1], A[2], B[0], B[1], B[2])
    b16 = oracle.to_bf16(bias)
    y1 = oracle.to_bf16(oracle.to_bf16(ref_y) + b16)            # gemm_packed -> bf16, then y1 + b1
    h = oracle.gelu(y1) if exact else _gelu_tanh(ref_y + b16)
    gh = np.float32(np.abs(oracle.to_bf16(h)).max() / 2688.0)
    ap, asf, ag = to_cuda_operand(A[3], A[4], A[2])
    bp, bsf, bg = to_cuda_operand(B[3], B[4], B[2])
    hp, hsf = ops.gemm_gelu_nvfp4(ap, asf, ag, bp, bsf, bg, torch.from_numpy(bias).cuda().bfloat16(),
                                  torch.tensor(gh, device="cuda"), exact=exact)
    torch.cuda.synchronize()
    if exact:
        c, b = oracle.triton_cast_nvfp4(y1, gh, apply_gelu=True)
    else:
        c, b = oracle.triton_cast_nvfp4(h, gh)
    codes = oracle.unpack_e2m1(hp.cpu().numpy())
    sf = oracle.from_blocked(hsf.cpu().numpy(), M, N // 16)
    bar = 2e-4 if exact else 2e-3
    assert (codes != c).mean() < bar, (codes != c).mean()
    assert (sf != b).mean() < bar, (sf != b).mean()
    deq = oracle.dequantize_nvfp4(codes, sf, gh)
    assert cos(deq, oracle.dequantize_nvfp4(c, b, gh)) >= 0.9999
    # either flavour stays within FP4 resolution of the reference's erf-GELU quantization
    ce, be = oracle.triton_cast_nvfp4(y1, gh, apply_gelu=True)
    assert cos(deq, oracle.dequantize_nvfp4(ce, be, gh)) >= 0.998
    # padded scale rows of the last 128-row tile are zero
    full = hsf.cpu().numpy()
    pad = oracle.from_blocked(full, (M + 127) // 128 * 128, N // 16)[M:]
    assert (pad == 0).all()


def test_gelu_erf_matches_torch_exact_gelu():
    """The fc1 epilogue's erf-GELU (vf4_gelu_erf_f32 runs the same device function elementwise)
    against torch's exact F.gelu on the GPU (CUDA erff): |error| <= 4e-7 |x| + 1e-30 over a dense
    sweep of [-12, 12] (A&S 7.1.26 bounds erf's error by 1.5e-7, half of it reaches GELU, plus the
    approximate reciprocal / ex2 and fp32 roundings), the tails, +-inf, NaN and signed zeros."""
    from vitfp4 import _lib
    x = torch.cat([torch.linspace(-12, 12, 2_000_001, device="cuda"),
                   torch.linspace(5.5, 5.6, 10001, device="cuda"), -torch.linspace(5.5, 5.6, 10001, device="cuda"),
                   torch.tensor([0.0, -0.0, 1e-30, -1e-30, 1e4, -1e4], device="cuda")])
    out = torch.empty_like(x)
    _lib.call("vf4_gelu_erf_f32", x.data_ptr(), x.numel(), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    ref = torch.nn.functional.gelu(x.double())
    err = (out.double() - ref).abs()
    assert (err <= 4e-7 * x.double().abs() + 1e-30).all(), float((err / x.double().abs().clamp_min(1e-30)).max())
    # far tails: x itself for large positive x, within 1e-7 of zero for large negative x
    big = x.abs() >= 5.6
    assert torch.equal(out[big & (x > 0)], x[big & (x > 0)]) and (out[big & (x < 0)].abs() <= 1e-7).all()
    special = torch.tensor([float("inf"), float("-inf"), float("nan")], device="cuda")
    o2 = torch.empty_like(special)
    _lib.call("vf4_gelu_erf_f32", special.data_ptr(), 3, o2.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert o2[0].item() == float("inf") and o2[1].item() == 0.0 and o2[2].isnan()   # -inf: the limit


def test_gemm_full_size_sampled_rows():
    """BASELINE config-2 fc2 shape (M=50432, K=3072, N=768): parity on sampled output rows."""
    ops = _ops()
    M, K, N = 50432, 3072, 768
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02)
    ap, asf, _, ag = ops.cast(x, None, "six")
    wp, wsf, wl, wg = ops.cast(w, None, "mse", linear=True)
    out = ops.gemm(ap, asf, ag, wp, wsf, wg, out_dtype=torch.float32)
    torch.cuda.synchronize()
    rows = torch.randint(0, M, (48,), generator=torch.Generator().manual_seed(2))
    a_codes = oracle.unpack_e2m1(ap[rows.cuda()].cpu().numpy())
    a_bs = oracle.from_blocked(asf.cpu().numpy(), M, K // 16)[rows.numpy()]
    b_codes = oracle.unpack_e2m1(wp.cpu().numpy())
    ref = oracle.gemm_reference(a_codes, a_bs, np.float32(ag.item()), b_codes, wl.cpu().numpy(),
                                np.float32(wg.item()))
    got = out[rows.cuda()].cpu().numpy()
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()


@pytest.mark.parametrize("M,K,N", [(256, 1024, 1024), (333, 3072, 768), (1024, 1152, 4304), (300, 512, 512)])
def test_gemm_cta_pair_kernel(M, K, N, monkeypatch):
    """The CTA-pair (cta_group::2, 256x256 tile) kernel, selected with VF4_GEMM_TILE=pair."""
    monkeypatch.setenv("VF4_GEMM_TILE", "pair")
    A, B = _operands(M, N, K, seed=M + K)
    out = _gemm_cuda(A, B)
    ref = oracle.gemm_reference(A[0], A[1], A[2], B[0], B[1], B[2])
    assert np.abs(out - ref).max() <= 1e-3 * np.abs(ref).max() and cos(out, ref) >= 0.9999
    bias = (np.random.default_rng(4).standard_normal(N) * 0.1).astype(np.float32)
    out = _gemm_cuda(A, B, out_dtype=torch.bfloat16, bias=bias)
    refb = oracle.to_bf16(oracle.to_bf16(ref) + oracle.to_bf16(bias))
    assert cos(out, refb) >= 0.9999


@pytest.mark.parametrize("tile", ["", "pair"])
@pytest.mark.parametrize("gamma", [True, False])
@pytest.mark.parametrize("M,K,N", [(256, 1024, 1024), (197, 3072, 768), (130, 512, 128)])
def test_gemm_residual_epilogue(M, K, N, gamma, tile, monkeypatch):
    """fc2 + LayerScale + residual epilogue equals the unfused bf16 steps bit for bit: the bias
    GEMM rounded to bf16, then (y * gamma) and the residual add as bf16 torch ops."""
    if tile:
        monkeypatch.setenv("VF4_GEMM_TILE", tile)
    ops = _ops()
    A, B = _operands(M, N, K, seed=11)
    ap, asf, ag = to_cuda_operand(A[3], A[4], A[2])
    bp, bsf, bg = to_cuda_operand(B[3], B[4], B[2])
    g = torch.Generator(device="cpu").manual_seed(5)
    bias = (torch.randn(N, generator=g) * 0.1).cuda().bfloat16()
    res = torch.randn(M, N, generator=g).cuda().bfloat16()
    gam = (torch.rand(N, generator=g) * 0.5 + 1e-5).cuda().bfloat16() if gamma else None
    y = ops.gemm(ap, asf, ag, bp, bsf, bg, bias=bias, out_dtype=torch.bfloat16)
    ref = res + (y * gam if gamma else y)
    out = ops.gemm_residual(ap, asf, ag, bp, bsf, bg, bias, res, gamma=gam)
    assert torch.equal(out, ref)
    inplace = res.clone()
    ops.gemm_residual(ap, asf, ag, bp, bsf, bg, bias, inplace, gamma=gam, out=inplace)
    assert torch.equal(inplace, ref)


@pytest.mark.parametrize("M,K,N", [(1152, 1024, 4096), (4736, 512, 832), (1300, 768, 2304)])
def test_gemm_resident_b_scales_kernel(M, K, N, monkeypatch):
    """The K <= 1024 kernel that keeps B's scale factors in TMEM (one N tile per CTA, M tiles
    strided) against the emulation, and bit-equal to the streaming kernel on bf16 + bias and
    GELU-NVFP4 outputs (same MMAs, same epilogue)."""
    ops = _ops()
    A, B = _operands(M, N, K, seed=M + N)
    out = _gemm_cuda(A, B)
    ref = oracle.gemm_reference(A[0], A[1], A[2], B[0], B[1], B[2])
    assert np.abs(out - ref).max() <= 1e-3 * np.abs(ref).max() and cos(out, ref) >= 0.9999
    ap, asf, ag = to_cuda_operand(A[3], A[4], A[2])
    bp, bsf, bg = to_cuda_operand(B[3], B[4], B[2])
    bias = (torch.randn(N, generator=torch.Generator().manual_seed(1)) * 0.1).cuda().bfloat16()
    gh = torch.tensor(float(np.abs(ref).max()) / 2688.0, device="cuda")
    ws = [ops.gemm(ap, asf, ag, bp, bsf, bg, bias=bias, out_dtype=torch.bfloat16),
          *ops.gemm_gelu_nvfp4(ap, asf, ag, bp, bsf, bg, bias, gh)]
    monkeypatch.setenv("VF4_GEMM_TILE", "stream")
    st = [ops.gemm(ap, asf, ag, bp, bsf, bg, bias=bias, out_dtype=torch.bfloat16),
          *ops.gemm_gelu_nvfp4(ap, asf, ag, bp, bsf, bg, bias, gh)]
    for a, b in zip(ws, st):
        assert torch.equal(a, b)


@pytest.mark.parametrize("M,K,N", [(300, 2048, 512), (1300, 4096, 1024), (333, 1536, 832), (64, 1088, 256)])
def test_gemm_b_scale_image(M, K, N):
    """The B scale image (each to_blocked atom held four times, per 256-row tile and K64 block) and the
    streaming kernel that copies a K64 block's B scales with one 128x256b tcgen05.cp from it: the
    image equals its definition, and every epilogue (bf16, + bias, fp32, residual) is bit-equal to the
    two-copy kernel; N = 832 has an odd count of 128-row scale blocks (the last tile repeats its first
    atom), K = 1088 a last stage of one K64 block, M = 333 and 300 a partial last row tile."""
    ops = _ops()
    A, B = _operands(M, N, K, seed=K + N)
    ap, asf, ag = to_cuda_operand(A[3], A[4], A[2])
    bp, bsf, bg = to_cuda_operand(B[3], B[4], B[2])
    img = ops.b_scale_image(bsf, N, K)
    n_rb, n_kb, ntn = (N + 127) // 128, (K + 63) // 64, (N + 255) // 256
    atoms = bsf.view(torch.uint8).reshape(n_rb, n_kb, 512)
    if n_rb % 2:
        atoms = torch.cat([atoms, atoms[-1:]], 0)   # the last tile's first atom
    want = atoms.reshape(ntn, 2, n_kb, 512).permute(0, 2, 1, 3).unsqueeze(3).expand(ntn, n_kb, 2, 4, 512)
    assert torch.equal(img.reshape(ntn, n_kb, 2, 4, 512), want)
    g = torch.Generator(device="cpu").manual_seed(7)
    bias = (torch.randn(N, generator=g) * 0.1).cuda().bfloat16()
    res = torch.randn(M, N, generator=g).cuda().bfloat16()
    gam = (torch.rand(N, generator=g) * 0.5 + 1e-5).cuda().bfloat16()
    for kw in ({}, {"bias": bias}, {"out_dtype": torch.float32}):
        assert torch.equal(ops.gemm(ap, asf, ag, bp, bsf, bg, **kw), ops.gemm(ap, asf, ag, bp, bsf, bg, b_image=img, **kw))
    assert torch.equal(ops.gemm_residual(ap, asf, ag, bp, bsf, bg, bias, res, gamma=gam),
                       ops.gemm_residual(ap, asf, ag, bp, bsf, bg, bias, res, gamma=gam, b_image=img))


def test_bounded_wait_gives_up_and_reports():
    """The failure detector in the allowed form: a kernel's bounded mbarrier wait, given a 2 ms limit
    and a barrier nothing arrives on, gives up, records device error 1 (producer data never arrived)
    and returns; the call finishes far below the production 4 s limit, the error word clears when
    read, and the context still runs a GEMM correctly afterwards."""
    import time
    from vitfp4 import _lib
    ops = _ops()
    assert _lib.device_error() == 0                       # also clears anything left over
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    _lib.call("vf4_selftest_wait_timeout", 2_000_000, stream)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert elapsed < 1.0, elapsed
    assert _lib.device_error(clear=True) == 1
    assert _lib.device_error() == 0
    with pytest.raises(_lib.VitFp4Error):
        _lib.call("vf4_selftest_wait_timeout", 0, stream)
    A, B = _operands(130, 256, 512, seed=1)
    ap, asf, ag = to_cuda_operand(A[3], A[4], A[2])
    bp, bsf, bg = to_cuda_operand(B[3], B[4], B[2])
    y = ops.gemm(ap, asf, ag, bp, bsf, bg, out_dtype=torch.float32)
    ref = oracle.gemm_reference(A[0], A[1], A[2], B[0], B[1], B[2])
    assert np.abs(y.cpu().numpy() - ref).max() <= 1e-3 * np.abs(ref).max()
    assert _lib.device_error() == 0
