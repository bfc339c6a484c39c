"""The allocation-free attention entry point (vf4_attn_nvfp4_noalloc).

Callers such as an inference server with its own device-memory pool, or a plugin that must not
allocate (or trigger the device synchronisation an allocation can cause) while serving, cannot
hand the attention a workspace from cudaMalloc.  vf4_attn_nvfp4_noalloc runs the same kernels
with a fixed 16 MiB device array inside the library as its scratch.  This file checks, through
the C ABI, that two calls in a row give the same outputs as the workspace entry point
vf4_attn_nvfp4, and that a problem too large for the array is refused without launching.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(name, lib, q, k, v, B, H, S, D, out, ws=None):
    st = (H * S * D, S * D, D)
    ost = (S * H * D, D, H * D)
    stream = torch.cuda.current_stream().cuda_stream
    args = [q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, S, D, *st, ctypes.c_float(D ** -0.5),
            out.data_ptr(), *ost]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    return getattr(lib, name)(*args, stream)


@pytest.mark.parametrize("shapes", [[(2, 4, 257, 64), (1, 2, 1025, 80)],     # fused route, then long-sequence
                                    [(1, 2, 1025, 80), (2, 4, 257, 64)]])    # and the reverse order
def test_noalloc_matches_workspace_entry_point_twice(shapes):
    from vitfp4 import _lib
    lib = _lib.lib()
    for i, (B, H, S, D) in enumerate(shapes):      # two calls in a row, different problems
        g = torch.Generator(device="cuda").manual_seed(10 + i)
        q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).bfloat16() for _ in range(3))
        ws = torch.empty(int(lib.vf4_attn_workspace_size(B, H, S, D)), dtype=torch.uint8, device="cuda")
        ref = torch.empty(B, S, H, D, dtype=torch.bfloat16, device="cuda")
        out = torch.full((B, S, H, D), float("nan"), dtype=torch.bfloat16, device="cuda")
        assert _call("vf4_attn_nvfp4", lib, q, k, v, B, H, S, D, ref, ws) == 0
        assert _call("vf4_attn_nvfp4_noalloc", lib, q, k, v, B, H, S, D, out) == 0, \
            lib.vf4_last_error_string()
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert torch.allclose(out.float(), ref.float(), rtol=0, atol=0), (out.float() - ref.float()).abs().max()
    assert _lib.device_error() == 0


def test_noalloc_refuses_oversized_problem():
    from vitfp4 import _lib
    lib = _lib.lib()
    B, H, S, D = 8, 16, 1025, 80                      # ViT-H/14 @448 heads: ~30 MB of workspace > 16 MiB
    assert lib.vf4_attn_workspace_size(B, H, S, D) > 16 << 20
    q = torch.zeros(B, H, S, D, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(B, S, H, D, dtype=torch.bfloat16, device="cuda")
    status = _call("vf4_attn_nvfp4_noalloc", lib, q, q, q, B, H, S, D, out)
    assert status == 6                                 # VF4_ERR_UNSUPPORTED
    assert b"16777216" in lib.vf4_last_error_string()
    torch.cuda.synchronize()
    assert (out == 0).all()
