"""GPU parity of the NVFP4 attention kernels.

The kernels' deliberate differences from the reference's emulated quant_sdpa: the fixed 1/(6*448)
global for P, and P quantized before the 1/rowsum (P = exp(s - max) in [0, 1], exactly 1 at the row
max; the output is divided by the row sum).  Bars:
  * vs a CPU restatement of exactly those semantics (``_oracle_kernel_semantics``): cos >= 0.999
  * vs the reference's quantized output (oracle.quant_sdpa, qk = pv = 'nvfp4'): cos >= 0.995
  * accuracy vs exact fp32 attention no worse than the reference's own minus 0.005, and > 0.95
    (the reference's bar, tests/test_attention.py:60-64)
The per-head-globals mode is a different FP4 noise draw (cos ~0.98 vs the reference), so it is
held to its own oracle and to the reference's accuracy over many heads.
"""
import math

import numpy as np
import pytest
import torch

from conftest import oracle
from gpu_util import cos

pytestmark = pytest.mark.gpu

F32 = np.float32


def _qdq(x, gs, axis=-1):
    """NVFP4 round trip along ``axis`` with a given global scale (zero-padded to 16)."""
    x = np.moveaxis(np.asarray(x, F32), axis, -1)
    k = x.shape[-1]
    pad = (-k) % 16
    if pad:
        x = np.concatenate([x, np.zeros((*x.shape[:-1], pad), F32)], -1)
    c, b, g = oracle.quantize_to_nvfp4(x, 16, global_scale=F32(gs))
    d = oracle.dequantize_nvfp4(c, b, g)[..., :k]
    return np.moveaxis(d, -1, axis)


def _oracle_kernel_semantics(q, k, v, scale, head_globals=False, smooth_k=True, smooth_v=True):
    """The kernels' arithmetic: smooth-K/V (each switchable), NVFP4 Q, K~ (along d) and V~ (along
    tokens) with global scales over the whole tensors (or per head), P with the fixed global 1/2688
    quantized unnormalised (P = exp(s - max) in [0, 1], the 1/rowsum applied to the output)."""
    B, H, S, D = q.shape
    out = np.empty((B, H, S, D), F32)
    g = lambda t: F32(max(np.abs(t).max(), 1e-12) / 2688.0)
    ktt = k - k.mean(2, keepdims=True) if smooth_k else k
    vtt = v - v.mean(2, keepdims=True) if smooth_v else v
    gq_all, gk_all, gv_all = g(q), g(ktt), g(vtt)
    for b in range(B):
        for h in range(H):
            qq, kk, vv = q[b, h], k[b, h], v[b, h]
            kt = kk - kk.mean(0, keepdims=True) if smooth_k else kk
            mu = vv.mean(0, keepdims=True) if smooth_v else np.zeros((1, D), F32)
            vt = vv - mu
            gq, gk, gv = (g(qq), g(kt), g(vt)) if head_globals else (gq_all, gk_all, gv_all)
            s = _qdq(qq, gq) @ _qdq(kt, gk).T * F32(scale)
            vd = _qdq(vt, gv, axis=0)
            p = np.exp(s - s.max(-1, keepdims=True)).astype(F32)
            out[b, h] = (_qdq(p, F32(1.0 / 2688.0)) @ vd) / p.sum(-1, keepdims=True) + mu
    return out


def _qkv(B, H, S, D, seed=0, outlier=True):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, S, D, generator=g)
    k = torch.randn(B, H, S, D, generator=g)
    v = torch.randn(B, H, S, D, generator=g)
    if outlier:  # ViT-like: high-norm tokens and a heavy channel (reference tests/test_attention.py:15-18)
        k[..., :2, :] *= 12.0
        k[..., 7] *= 8.0
        v[..., :2, :] *= 10.0
    return q.bfloat16(), k.bfloat16(), v.bfloat16()


SHAPES = [(2, 4, 64, 64), (1, 2, 197, 64), (2, 3, 257, 64), (1, 2, 1025, 80), (1, 1, 20, 64),
          (1, 2, 130, 128), (2, 2, 385, 64), (1, 1, 1, 64), (1, 2, 48, 64), (2, 3, 320, 64),
          (8, 40, 197, 64)]   # the last one: more heads than SMs, several heads per persistent CTA


@pytest.mark.parametrize("B,H,S,D", SHAPES)
def test_attention_matches_oracles(B, H, S, D):
    from vitfp4.nvfp4 import quant_sdpa
    q, k, v = _qkv(B, H, S, D, seed=S + D)
    scale = 1.0 / math.sqrt(D)
    out = quant_sdpa(q.cuda(), k.cuda(), v.cuda(), qk="nvfp4", pv="nvfp4").float().cpu().numpy()
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref_kernel = _oracle_kernel_semantics(qn, kn, vn, scale)
    ref_sdpa = oracle.quant_sdpa(qn, kn, vn, qk="nvfp4", pv="nvfp4")
    exact = oracle.quant_sdpa(qn, kn, vn, qk="bf16", pv="bf16", smooth_k=False, smooth_v=False)
    assert np.isfinite(out).all()
    c1, c2, c3, c_ref = cos(out, ref_kernel), cos(out, ref_sdpa), cos(out, exact), cos(ref_sdpa, exact)
    assert c1 >= 0.999 and c2 >= 0.995 and c3 > 0.95 and c3 >= c_ref - 0.005, (c1, c2, c3, c_ref)


@pytest.mark.parametrize("packed", [True, False])
@pytest.mark.parametrize("B,H,S,D", [(2, 3, 257, 64), (16, 12, 197, 64), (1, 2, 1025, 80)])
def test_attention_head_globals_mode(B, H, S, D, packed):
    """Per-head global scales (VF4_ATTN_HEAD_GLOBALS): exact to its own semantics, and as accurate
    as the reference on average over many heads (each head is an independent FP4 noise draw)."""
    from vitfp4.nvfp4 import ops
    q, k, v = _qkv(B, H, S, D, seed=7 + S)
    scale = 1.0 / math.sqrt(D)
    out = ops.attention_bhsd(q.cuda(), k.cuda(), v.cuda(), scale, head_globals=True,
                             packed=packed).float().cpu().numpy()
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref_kernel = _oracle_kernel_semantics(qn, kn, vn, scale, head_globals=True)
    exact = oracle.quant_sdpa(qn, kn, vn, qk="bf16", pv="bf16", smooth_k=False, smooth_v=False)
    ref_sdpa = oracle.quant_sdpa(qn, kn, vn, qk="nvfp4", pv="nvfp4")
    assert cos(out, ref_kernel) >= 0.999
    assert cos(out, exact) >= cos(ref_sdpa, exact) - 0.005 and cos(out, exact) > 0.95


@pytest.mark.parametrize("B,H,S,D", [(2, 3, 257, 64), (1, 1, 1, 64), (1, 2, 48, 64), (2, 3, 320, 64),
                                     (8, 40, 197, 64), (3, 16, 129, 64)])
def test_packed_operand_route_equals_inline_route(B, H, S, D):
    """VF4_ATTN_PACKED quantizes the operands in a separate pass into per-head images; with the
    reference's tensor-wide globals the result is the in-kernel route's, bit for bit."""
    from vitfp4 import _lib
    from vitfp4.nvfp4 import ops
    q, k, v = (t.cuda() for t in _qkv(B, H, S, D, seed=11 + S))
    a = ops.attention_bhsd(q, k, v, D ** -0.5, packed=True)
    b = ops.attention_bhsd(q, k, v, D ** -0.5, packed=False)
    qkv = torch.stack([q, k, v], 0).permute(1, 3, 0, 2, 4).reshape(B, S, 3 * H * D).contiguous()
    c = ops.attention_packed_qkv(qkv, H, D ** -0.5, packed=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(c.reshape(B, S, H, D), b.transpose(1, 2))
    assert _lib.device_error() == 0


def test_packed_workspace_size():
    from vitfp4 import _lib
    lib = _lib.lib()
    plain = lib.vf4_attn_workspace_size(4, 16, 257, 64)
    packed = lib.vf4_attn_workspace_size_ex(4, 16, 257, 64, _lib.VF4_ATTN_PACKED)
    assert lib.vf4_attn_workspace_size_ex(4, 16, 257, 64, 0) == plain
    assert packed >= plain + 4 * 16 * 38 * 1024
    # the long-sequence route ignores the flag
    assert lib.vf4_attn_workspace_size_ex(1, 2, 1025, 80, _lib.VF4_ATTN_PACKED) == lib.vf4_attn_workspace_size(1, 2, 1025, 80)
    assert lib.vf4_attn_workspace_size_ex(1, 2, 257, 64, 16) == 0


def test_attention_packed_qkv_path_equals_bhsd():
    from vitfp4.nvfp4 import ops
    B, S, H, D = 3, 257, 4, 64
    qkv = (torch.randn(B, S, 3 * H * D, device="cuda") * 2).bfloat16()
    a = ops.attention_packed_qkv(qkv, H, D ** -0.5)
    q, k, v = qkv.reshape(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
    b = ops.attention_bhsd(q.contiguous(), k.contiguous(), v.contiguous(), D ** -0.5)
    c = ops.attention_bhsd(q, k, v, D ** -0.5)              # strided views, read in place
    torch.cuda.synchronize()
    assert torch.equal(a.reshape(B, S, H, D), b.transpose(1, 2))
    assert torch.equal(b, c)


def test_attention_deterministic_and_no_device_error():
    from vitfp4 import _lib
    from vitfp4.nvfp4 import ops
    q, k, v = (t.cuda() for t in _qkv(2, 2, 257, 64, seed=3))
    a = ops.attention_bhsd(q, k, v, 0.125)
    b = ops.attention_bhsd(q, k, v, 0.125)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert _lib.device_error() == 0


def test_quant_attention_adapter_returns_bshd():
    """HF adapter contract (reference tests/test_qattention.py:20-36): (B,S,H,D) out, None weights;
    unflagged modules run exact SDPA."""
    import torch.nn as nn
    import torch.nn.functional as F
    from vitfp4.ptq.qattention import _quant_attention

    class FakeAttention(nn.Module):
        def __init__(self):
            super().__init__()
            self.scaling = 0.125

    q, k, v = (t.cuda() for t in _qkv(2, 4, 16, 64, seed=4, outlier=False))
    m = FakeAttention()
    m._nvfp4_attn, m._nvfp4_qk, m._nvfp4_pv = True, "nvfp4", "nvfp4"
    out, w = _quant_attention(m, q, k, v, None, scaling=0.125)
    assert w is None and out.shape == (2, 16, 4, 64)
    ref = F.scaled_dot_product_attention(q, k, v, scale=0.125).transpose(1, 2)
    assert F.cosine_similarity(out.flatten().float(), ref.flatten().float(), dim=0) > 0.95
    out2, _ = _quant_attention(FakeAttention(), q, k, v, None, scaling=0.125)
    assert torch.equal(out2, F.scaled_dot_product_attention(q, k, v, scale=0.125).transpose(1, 2).contiguous())


@pytest.mark.parametrize("qk,pv", [("nvfp4", "fp8"), ("fp8", "nvfp4"), ("bf16", "fp8"), ("fp8", "bf16")])
def test_fp8_and_mixed_routes_match_reference(qk, pv):
    """The reference's default route (fp8 / fp8) and the mixed ones run its own arithmetic on the GPU:
    equal to the CPU restatement up to fp32 summation order."""
    from vitfp4.nvfp4 import quant_sdpa
    B, H, S, D = 2, 3, 197, 64
    q, k, v = _qkv(B, H, S, D, seed=31)
    out = quant_sdpa(q.cuda(), k.cuda(), v.cuda(), qk=qk, pv=pv).float().cpu().numpy()
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref = oracle.quant_sdpa(qn, kn, vn, qk=qk, pv=pv)
    exact = oracle.quant_sdpa(qn, kn, vn, qk="bf16", pv="bf16", smooth_k=False, smooth_v=False)
    assert cos(out, ref) >= 0.9999, cos(out, ref)
    assert cos(out, exact) > 0.95


@pytest.mark.parametrize("B,H,S,D", [(2, 3, 257, 64), (1, 4, 197, 64), (1, 1, 1, 64), (1, 2, 48, 64), (8, 40, 197, 64)])
def test_fp8_kernel_matches_reference(B, H, S, D):
    """The FP8 kernel (the reference's default qk = pv = 'fp8' route) against the reference's
    emulated quant_sdpa: same quantization (E4M3 with per-row scales), fp32 accumulation order and
    P scaling (448 * exp(s - max) instead of P / (max P / 448)) differ only by rounding."""
    from vitfp4.nvfp4 import ops, quant_sdpa
    q, k, v = _qkv(B, H, S, D, seed=40 + S)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = ops.attention_fp8_bhsd(qc, kc, vc, D ** -0.5).float().cpu().numpy()
    assert np.array_equal(out, quant_sdpa(qc, kc, vc, qk="fp8", pv="fp8").float().cpu().numpy())
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref = oracle.quant_sdpa(qn, kn, vn, qk="fp8", pv="fp8")
    exact = oracle.quant_sdpa(qn, kn, vn, qk="bf16", pv="bf16", smooth_k=False, smooth_v=False)
    assert np.isfinite(out).all()
    assert cos(out, ref) >= 0.999, cos(out, ref)
    assert cos(out, exact) >= cos(ref, exact) - 0.002


@pytest.mark.parametrize("B,H,S,D", [(1, 2, 1025, 80), (2, 3, 257, 80), (1, 2, 400, 64), (1, 1, 129, 128),
                                     (2, 2, 60, 96), (1, 2, 33, 16), (1, 1, 1408, 80)])
def test_fp8_long_route_matches_reference(B, H, S, D):
    """The long-sequence FP8 route (prep + persistent kernel; ViT-H/14's head dim 80 at 224 and 448 px)
    against the reference's quant_sdpa(qk = pv = 'fp8'): the same quantization of Q, K~, V~ and P, so only
    rounding differs -- per head cos >= 0.999, accuracy vs exact attention within 0.002 of the reference's."""
    from vitfp4.nvfp4 import ops, quant_sdpa
    assert ops.fp8_kernel_ok(S, D)
    q, k, v = _qkv(B, H, S, D, seed=70 + S)
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = ops.attention_fp8_bhsd(qc, kc, vc, D ** -0.5).float().cpu().numpy()
    assert np.array_equal(out, quant_sdpa(qc, kc, vc, qk="fp8", pv="fp8").float().cpu().numpy())
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref = oracle.quant_sdpa(qn, kn, vn, qk="fp8", pv="fp8")
    exact = oracle.quant_sdpa(qn, kn, vn, qk="bf16", pv="bf16", smooth_k=False, smooth_v=False)
    assert np.isfinite(out).all()
    for b in range(B):
        for h in range(H):
            assert cos(out[b, h], ref[b, h]) >= 0.999, (b, h, cos(out[b, h], ref[b, h]))
    assert cos(out, exact) >= cos(ref, exact) - 0.002
    from vitfp4 import _lib
    assert _lib.device_error() == 0


def test_fp8_long_route_many_heads_in_place():
    """More heads than SMs (several heads per persistent CTA, several query tiles per head) read in place
    from the (B, H, S, D) views of a packed qkv projection, as the fused block calls it: against the
    reference's arithmetic run on the GPU (the emulation route), per head cos >= 0.999."""
    from vitfp4.nvfp4 import ops
    from vitfp4.nvfp4.attention import _emulated_sdpa
    B, H, S, D = 16, 16, 1025, 80
    g = torch.Generator(device="cuda").manual_seed(11)
    qkv = torch.randn(B, S, 3 * H * D, device="cuda", generator=g).bfloat16()
    qkv[:, :2] *= 6.0
    q, k, v = qkv.reshape(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
    out = ops.attention_fp8_bhsd(q, k, v, D ** -0.5).float()
    ref = _emulated_sdpa(q, k, v, None, False, D ** -0.5, "fp8", "fp8", True, True)
    c = torch.nn.functional.cosine_similarity(out.reshape(B * H, -1), ref.reshape(B * H, -1), dim=1)
    assert torch.isfinite(out).all()
    assert c.min().item() >= 0.999, c.min().item()


@pytest.mark.parametrize("smooth_k,smooth_v", [(False, False), (True, False), (False, True)])
def test_fp8_long_route_smoothing_switches(smooth_k, smooth_v):
    """Smooth-K / smooth-V switched off on the long-sequence FP8 route, through quant_sdpa and through
    vf4_attn with the workspace vf4_attn_workspace_size_modes asks for (none given: VF4_ERR_ARG, nothing
    launched)."""
    import ctypes
    from vitfp4 import _lib
    from vitfp4.nvfp4 import quant_sdpa
    B, H, S, D = 2, 2, 300, 80
    q, k, v = _qkv(B, H, S, D, seed=8)
    k = (k.float() + 3.0).bfloat16()
    v = (v.float() - 2.0).bfloat16()
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = quant_sdpa(qc, kc, vc, qk="fp8", pv="fp8", smooth_k=smooth_k, smooth_v=smooth_v)
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref = oracle.quant_sdpa(qn, kn, vn, qk="fp8", pv="fp8", smooth_k=smooth_k, smooth_v=smooth_v)
    assert cos(out.float().cpu().numpy(), ref) >= 0.999
    lib = _lib.lib()
    m = _lib.VF4_ATTN_MODE["fp8"]
    flags = (0 if smooth_k else _lib.VF4_ATTN_NO_SMOOTH_K) | (0 if smooth_v else _lib.VF4_ATTN_NO_SMOOTH_V)
    n = int(lib.vf4_attn_workspace_size_modes(B, H, S, D, m, m, flags))
    assert n > 0
    stream = torch.cuda.current_stream().cuda_stream
    o2 = torch.zeros(B, S, H, D, dtype=torch.bfloat16, device="cuda")
    args = (qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, H, S, D, H * S * D, S * D, D, ctypes.c_float(D ** -0.5),
            m, m, flags)
    assert lib.vf4_attn(*args, None, 0, o2.data_ptr(), S * H * D, D, H * D, stream) == 1
    assert (o2 == 0).all()
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    assert lib.vf4_attn(*args, ws.data_ptr(), n, o2.data_ptr(), S * H * D, D, H * D, stream) == 0
    assert torch.equal(o2.transpose(1, 2), out)


# ----------------------------------------------------------------------------- bf16 kernel
def _bf16_errors(q, k, v, scale, got):
    """Max |error| of ``got`` and of torch's own bf16 SDPA against fp32 attention of the same bf16 inputs."""
    import torch.nn.functional as F
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=scale)
    sdpa = F.scaled_dot_product_attention(q, k, v, scale=scale).float()
    return (got.float() - ref).abs().max().item(), (sdpa - ref).abs().max().item()


@pytest.mark.parametrize("kernel", ["slots", "tiles"])
@pytest.mark.parametrize("B,H,S", [(2, 3, 257), (1, 4, 197), (1, 1, 1), (1, 2, 48), (2, 2, 256), (1, 3, 129),
                                   (1, 2, 136), (1, 2, 288), (1, 1, 264), (4, 16, 257), (2, 3, 258),
                                   (1, 2, 2), (1, 3, 16), (2, 2, 128), (24, 16, 257), (20, 16, 197),
                                   (40, 16, 258)])
def test_bf16_kernel_matches_sdpa(B, H, S, kernel, monkeypatch):
    """The bf16 kernels (exact softmax, P rounded to bf16 for the PV MMA, like flash attention)
    against fp32 attention of the same bf16 inputs: no worse than twice torch's own bf16 SDPA
    error (and 4e-3 absolute), on (B, H, S, D) operands and on the strided views of a packed qkv
    projection.  "slots" is the two-slot kernel (S <= 258; keys 256 and 257 on the CUDA cores, query
    rows past 256 in a third tile), "tiles" the single-slot one (S <= 288; S = 129 .. 132 and
    257 .. 260 run its per-row tail).  384, 320 and 640 heads give every CTA several heads (buffer
    reuse and barrier phases across heads)."""
    from vitfp4.nvfp4 import ops
    monkeypatch.setenv("VF4_BF16_ATTN", kernel)
    D = 64
    torch.manual_seed(S + 7 * H)
    qkv = (torch.randn(B, S, 3 * H * D, device="cuda") * 1.5).bfloat16()
    scale = D ** -0.5
    got = ops.attention_bf16_packed_qkv(qkv, H, scale)
    q, k, v = qkv.reshape(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
    err, ref_err = _bf16_errors(q, k, v, scale, got.reshape(B, S, H, D).transpose(1, 2))
    assert torch.isfinite(got).all()
    assert err <= max(2 * ref_err, 4e-3), (err, ref_err)
    # contiguous (B, H, S, D) operands, output in (B, H, S, D) strides
    qc, kc, vc = (t.contiguous() for t in (q, k, v))
    out = torch.empty(B, H, S, D, device="cuda", dtype=torch.bfloat16)
    ops.attention_bf16(qc, kc, vc, B, H, S, D, (H * S * D, S * D, D), scale, out, (H * S * D, S * D, D))
    assert torch.equal(out, got.reshape(B, S, H, D).transpose(1, 2))
    # the output amax the kernel reports is the one the proj's dynamic cast computes
    am = torch.empty((), dtype=torch.float32, device="cuda")
    got2 = ops.attention_bf16_packed_qkv(qkv, H, scale, out_amax=am)
    assert torch.equal(got2, got) and torch.equal(am, ops.amax(got))


@pytest.mark.parametrize("kernel", ["slots", "tiles"])
@pytest.mark.parametrize("S,late", [(256, 200), (257, 131), (197, 190), (258, 257)])
def test_bf16_kernel_late_row_max(S, late, kernel, monkeypatch):
    """A key far past the first 16 whose score exceeds every earlier one by more than 2^32 after
    scaling: the two-slot kernel's running row max jumps there and the P chunks already written are
    rescaled in place (key 257 of S = 258 is one of the keys scored on the CUDA cores)."""
    from vitfp4.nvfp4 import ops
    monkeypatch.setenv("VF4_BF16_ATTN", kernel)
    B, H, D = 2, 2, 64
    torch.manual_seed(S + late)
    qkv = torch.randn(B, S, 3 * H * D, device="cuda") * 0.5
    qkv[:, :, 0] = 12.0                     # q of head 0: a large first coordinate in every row
    qkv[:, late, H * D] = 18.0              # k of head 0 at the late key: q . k ~ 216 there
    qkv = qkv.bfloat16()
    scale = D ** -0.5
    got = ops.attention_bf16_packed_qkv(qkv, H, scale)
    q, k, v = qkv.reshape(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
    err, ref_err = _bf16_errors(q, k, v, scale, got.reshape(B, S, H, D).transpose(1, 2))
    assert torch.isfinite(got).all()
    assert err <= max(2 * ref_err, 4e-3), (err, ref_err)


def test_bf16_kernel_rejects_unsupported_shapes():
    from vitfp4 import _lib
    from vitfp4.nvfp4 import ops
    q = torch.zeros(1, 1, 300, 64, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    with pytest.raises(_lib.VitFp4Error):
        ops.attention_bf16(q, q, q, 1, 1, 300, 64, (300 * 64, 300 * 64, 64), 0.125, out, (300 * 64, 300 * 64, 64))
    assert not ops.bf16_kernel_ok(300, 64) and not ops.bf16_kernel_ok(257, 80) and ops.bf16_kernel_ok(257, 64)


@pytest.mark.parametrize("kernel", ["slots", "tiles"])
@pytest.mark.parametrize("S,row", [(257, 5), (257, 256), (130, 129), (258, 257)])
def test_bf16_kernel_amax_propagates_nan(S, row, kernel, monkeypatch):
    """A NaN in the attention output reaches the fused max |out| as NaN, as the reference's torch amax
    of the SDPA output would give it (a float max would drop it and hand the proj cast a finite global).
    One NaN in v makes every query row's output NaN in that head's column; row picks a tile row or a
    tail row (S = 257 / 130 run the single-slot kernel's per-row tail for the last rows; in the
    two-slot kernel v rows 256 and 257 enter through the extra keys' K = 16 step)."""
    from vitfp4.nvfp4 import ops
    monkeypatch.setenv("VF4_BF16_ATTN", kernel)
    B, H, D = 2, 3, 64
    torch.manual_seed(S)
    qkv = torch.randn(B, S, 3 * H * D, device="cuda").bfloat16()
    qkv[1, row, 2 * H * D + D + 7] = float("nan")          # v of image 1, head 1, token `row`
    am = torch.empty((), dtype=torch.float32, device="cuda")
    got = ops.attention_bf16_packed_qkv(qkv, H, D ** -0.5, out_amax=am)
    torch.cuda.synchronize()
    assert got.isnan().any() and got.float().abs().amax().isnan()
    assert am.isnan(), am
    # and without a NaN the fused amax is finite and equals the output's
    qkv[1, row, 2 * H * D + D + 7] = 0.5
    got = ops.attention_bf16_packed_qkv(qkv, H, D ** -0.5, out_amax=am)
    assert torch.equal(am, got.float().abs().amax())



@pytest.mark.parametrize("smooth_k,smooth_v", [(False, False), (False, True), (True, False)])
@pytest.mark.parametrize("B,H,S,D", [(2, 3, 257, 64), (1, 2, 1025, 80)])
def test_nvfp4_attention_smoothing_switches(B, H, S, D, smooth_k, smooth_v):
    """quant_sdpa(..., smooth_k=False / smooth_v=False) on the FP4 kernels (VF4_ATTN_NO_SMOOTH_K / _V):
    against the kernels' semantics with the same switches (cos >= 0.999) and the reference's
    quant_sdpa with them (>= 0.995); k and v carry a token-constant offset, so the switches matter
    (smoothing exists to take it out of the FP4 ranges, attention.py:57-58, 66-67)."""
    from vitfp4.nvfp4 import quant_sdpa
    q, k, v = _qkv(B, H, S, D, seed=S + 11)
    k = (k.float() + 3.0).bfloat16()
    v = (v.float() - 2.0).bfloat16()
    out = quant_sdpa(q.cuda(), k.cuda(), v.cuda(), qk="nvfp4", pv="nvfp4", smooth_k=smooth_k,
                     smooth_v=smooth_v).float().cpu().numpy()
    on = quant_sdpa(q.cuda(), k.cuda(), v.cuda(), qk="nvfp4", pv="nvfp4").float().cpu().numpy()
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref_kernel = _oracle_kernel_semantics(qn, kn, vn, 1.0 / math.sqrt(D), smooth_k=smooth_k, smooth_v=smooth_v)
    ref_sdpa = oracle.quant_sdpa(qn, kn, vn, qk="nvfp4", pv="nvfp4", smooth_k=smooth_k, smooth_v=smooth_v)
    assert cos(out, ref_kernel) >= 0.999, cos(out, ref_kernel)
    assert cos(out, ref_sdpa) >= 0.995, cos(out, ref_sdpa)
    assert not np.array_equal(out, on)


@pytest.mark.parametrize("smooth_k,smooth_v", [(False, False), (True, False), (False, True)])
def test_fp8_attention_smoothing_switches(smooth_k, smooth_v):
    """The FP8 kernel with smooth-K / smooth-V switched off, through quant_sdpa and the unified vf4_attn
    entry: against the reference's quant_sdpa(qk=pv='fp8') with the same switches, cos >= 0.999."""
    import ctypes
    from vitfp4 import _lib
    from vitfp4.nvfp4 import quant_sdpa
    B, H, S, D = 2, 3, 257, 64
    q, k, v = _qkv(B, H, S, D, seed=5)
    k = (k.float() + 3.0).bfloat16()
    qc, kc, vc = q.cuda(), k.cuda(), v.cuda()
    out = quant_sdpa(qc, kc, vc, qk="fp8", pv="fp8", smooth_k=smooth_k, smooth_v=smooth_v)
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref = oracle.quant_sdpa(qn, kn, vn, qk="fp8", pv="fp8", smooth_k=smooth_k, smooth_v=smooth_v)
    assert cos(out.float().cpu().numpy(), ref) >= 0.999
    # the same through vf4_attn directly, (B, H, S, D) in and (B, S, H, D) out
    o2 = torch.empty(B, S, H, D, dtype=torch.bfloat16, device="cuda")
    flags = (0 if smooth_k else _lib.VF4_ATTN_NO_SMOOTH_K) | (0 if smooth_v else _lib.VF4_ATTN_NO_SMOOTH_V)
    m = _lib.VF4_ATTN_MODE["fp8"]
    _lib.call("vf4_attn", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), B, H, S, D, H * S * D, S * D, D,
              ctypes.c_float(D ** -0.5), m, m, flags, None, 0, o2.data_ptr(), S * H * D, D, H * D,
              torch.cuda.current_stream().cuda_stream)
    assert torch.equal(o2.transpose(1, 2), out)


def test_unified_attention_entry_routes_and_refusals():
    """vf4_attn: nvfp4/nvfp4 equals vf4_attn_nvfp4_ex, bf16/bf16 equals vf4_attn_bf16, mixed modes and
    switches on the per-head-globals route are refused without launching."""
    import ctypes
    from vitfp4 import _lib
    from vitfp4.nvfp4 import ops
    lib = _lib.lib()
    B, H, S, D = 2, 2, 197, 64
    q, k, v = (t.cuda() for t in _qkv(B, H, S, D, seed=9))
    st = (H * S * D, S * D, D)
    ost = (S * H * D, D, H * D)
    stream = torch.cuda.current_stream().cuda_stream

    def run(qk, pv, flags):
        n = int(lib.vf4_attn_workspace_size_modes(B, H, S, D, _lib.VF4_ATTN_MODE[qk], _lib.VF4_ATTN_MODE[pv], flags))
        ws = torch.empty(max(n, 16), dtype=torch.uint8, device="cuda")
        out = torch.zeros(B, S, H, D, dtype=torch.bfloat16, device="cuda")
        status = lib.vf4_attn(q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, S, D, *st, ctypes.c_float(D ** -0.5),
                              _lib.VF4_ATTN_MODE[qk], _lib.VF4_ATTN_MODE[pv], flags, ws.data_ptr(), ws.numel(),
                              out.data_ptr(), *ost, stream)
        return status, out

    s1, o1 = run("nvfp4", "nvfp4", 0)
    assert s1 == 0 and torch.equal(o1, ops.attention_bhsd(q, k, v, D ** -0.5, packed=False).transpose(1, 2))
    s2, o2 = run("bf16", "bf16", 0)
    ref = torch.empty(B, S, H, D, dtype=torch.bfloat16, device="cuda")
    ops.attention_bf16(q, k, v, B, H, S, D, st, D ** -0.5, ref, ost)
    assert s2 == 0 and torch.equal(o2, ref)
    s3, o3 = run("nvfp4", "fp8", 0)
    assert s3 == 6 and (o3 == 0).all()                                  # VF4_ERR_UNSUPPORTED
    s4, _ = run("nvfp4", "nvfp4", _lib.VF4_ATTN_HEAD_GLOBALS | _lib.VF4_ATTN_NO_SMOOTH_K)
    assert s4 == 6


@pytest.mark.parametrize("qk,B,H,S,D", [("fp8", 2, 3, 197, 64), ("fp8", 1, 2, 300, 80), ("nvfp4", 1, 2, 400, 64)])
def test_negative_softmax_scale(qk, B, H, S, D):
    """A negative scale makes the row's largest score the smallest q.k: the FP8 kernels (both routes)
    and the long-sequence FP4 route follow the sign; the fused FP4 kernel refuses it."""
    from vitfp4 import _lib
    from vitfp4.nvfp4 import quant_sdpa
    q, k, v = _qkv(B, H, S, D, seed=90 + S)
    scale = -(D ** -0.5)
    out = quant_sdpa(q.cuda(), k.cuda(), v.cuda(), scale=scale, qk=qk, pv=qk).float().cpu().numpy()
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    ref = (oracle.quant_sdpa(qn, kn, vn, scale=scale, qk=qk, pv=qk) if qk == "fp8"
           else _oracle_kernel_semantics(qn, kn, vn, scale))
    assert np.isfinite(out).all() and cos(out, ref) >= 0.999, cos(out, ref)
    assert _lib.device_error() == 0


def test_negative_scale_refused_where_the_kernel_assumes_a_positive_one():
    import ctypes
    from vitfp4 import _lib
    from vitfp4.nvfp4 import quant_sdpa
    q, k, v = (t.cuda() for t in _qkv(1, 2, 197, 64, seed=3))
    with pytest.raises(_lib.VitFp4Error, match="scale >= 0"):
        quant_sdpa(q, k, v, scale=-0.125, qk="nvfp4", pv="nvfp4")
    out = torch.zeros(1, 197, 2, 64, dtype=torch.bfloat16, device="cuda")
    st = _lib.lib().vf4_attn_bf16(q.data_ptr(), k.data_ptr(), v.data_ptr(), 1, 2, 197, 64, 2 * 197 * 64, 197 * 64, 64,
                                  ctypes.c_float(-0.125), out.data_ptr(), 197 * 2 * 64, 64, 2 * 64, None,
                                  torch.cuda.current_stream().cuda_stream)
    assert st == 6 and (out == 0).all()
