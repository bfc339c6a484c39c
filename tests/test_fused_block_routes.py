"""Attention routing of FusedNVFP4Block on the host (no GPU): which route a bf16 block takes for a
given sequence length, head dim and dtype, with the CUDA kernel entry replaced by a recorder and the
cuDNN routes run by torch's CPU SDPA."""
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F


def _route(qkv, H, D):
    """The fused block's attention routing for an unflagged (bf16-route) block."""
    from vitfp4.ptq.fused_block import _attention_route
    return _attention_route(qkv, H, D ** -0.5, "none", "none")


@pytest.fixture
def kernel_calls(monkeypatch):
    from vitfp4.nvfp4 import ops
    calls = []

    def fake(qkv, num_heads, scale, out_amax=None):
        calls.append((tuple(qkv.shape), num_heads, scale))
        out_amax.fill_(3.0)
        return torch.zeros(qkv.shape[0], qkv.shape[1], qkv.shape[2] // 3, dtype=qkv.dtype)

    monkeypatch.setattr(ops, "attention_bf16_packed_qkv", fake)
    return calls


def _sdpa(qkv, H, D):
    B, S, _ = qkv.shape
    q, k, v = qkv.reshape(B, S, 3, H, D).permute(2, 0, 3, 1, 4).unbind(0)
    return F.scaled_dot_product_attention(q.float(), k.float(), v.float(), scale=D ** -0.5).transpose(1, 2)


@pytest.mark.parametrize("S", [1, 197, 257, 264, 288])
def test_bf16_kernel_route(kernel_calls, S):
    H, D = 2, 64
    qkv = torch.randn(2, S, 3 * H * D).bfloat16()
    tag, out, am = _route(qkv, H, D)
    assert tag == "amax" and out.shape == (2, S, H * D) and am.item() == 3.0
    assert kernel_calls == [((2, S, 3 * H * D), H, D ** -0.5)]


@pytest.mark.parametrize("S,D,dtype", [(385, 64, torch.bfloat16), (400, 64, torch.bfloat16),
                                       (257, 80, torch.bfloat16), (257, 64, torch.float32)])
def test_split_query_route(kernel_calls, S, D, dtype):
    """Outside the kernel (S > 288, head dim != 64, or fp32) with S = 128 k + (1..16): two SDPA calls
    over all keys, queries [0, 128 k) and the rest, whose rows equal one call's."""
    H = 2
    qkv = torch.randn(1, S, 3 * H * D).to(dtype)
    tag, o1, o2 = _route(qkv, H, D)
    s_main = S // 128 * 128
    assert tag == "split" and not kernel_calls
    assert o1.shape == (1, s_main, H * D) and o2.shape == (1, S - s_main, H * D)
    ref = _sdpa(qkv, H, D).reshape(1, S, H * D)
    got = torch.cat([o1, o2], 1).float()
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert (got - ref).abs().max().item() <= tol


def test_whole_call_route(kernel_calls):
    H, D, S = 2, 64, 420                       # S % 128 = 36: one SDPA call
    qkv = torch.randn(1, S, 3 * H * D).bfloat16()
    out = _route(qkv, H, D)
    assert isinstance(out, torch.Tensor) and out.shape == (1, S, H * D) and not kernel_calls


def test_negative_scale_leaves_the_bf16_kernel(kernel_calls):
    """The bf16 kernel takes the row max of the raw scores, which is the softmax's max only for a
    scale >= 0; a negative scale goes to torch SDPA, the reference's own route for bf16 blocks."""
    from vitfp4.ptq.fused_block import _attention_route
    H, D, S = 2, 64, 197
    qkv = torch.randn(1, S, 3 * H * D).bfloat16()
    out = _attention_route(qkv, H, -(D ** -0.5), "none", "none")
    assert not kernel_calls and isinstance(out, torch.Tensor)
