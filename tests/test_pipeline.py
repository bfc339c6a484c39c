"""The overlapped host-fed runner: same outputs as the sequential copy -> forward -> read-back loop."""
import pytest
import torch

from vitfp4.pipeline import OverlappedRunner


def test_runner_needs_cuda_device():
    with pytest.raises(RuntimeError):
        OverlappedRunner(torch.nn.Identity(), torch.device("cpu"))


@pytest.mark.gpu
def test_runner_matches_sequential_linear():
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(64, 48), torch.nn.GELU(), torch.nn.Linear(48, 10)).cuda()
    host = [torch.randn(33, 64).pin_memory() for _ in range(5)]
    with torch.inference_mode():
        ref = [model(h.cuda()).float().cpu() for h in host]
        runner = OverlappedRunner(model, torch.device("cuda"))
        for n in (1, 2, 5):                  # one batch, both buffers once, buffers reused
            outs = runner.run(host[:n])
            torch.cuda.synchronize()
            assert len(outs) == n
            for a, b in zip(ref, outs):
                assert torch.equal(a, b)


@pytest.mark.gpu
def test_runner_matches_sequential_w4a4_vit():
    from vitfp4 import vit
    from vitfp4.ptq import fuse_mlps, fuse_norms, quantize_vit
    cfg = dict(vit.VIT_S16)
    cfg["depth"] = 2
    model = vit.build_vit(seed=3, **cfg).to(device="cuda", dtype=torch.bfloat16).eval()
    fuse_mlps(model, skip_ends=0)
    quantize_vit(model, skip_first=0, skip_last=0, w_block_select="mse")
    fuse_norms(model)
    host = [torch.randn(4, 3, 224, 224).bfloat16().pin_memory() for _ in range(3)]
    with torch.inference_mode():
        ref = [model(h.cuda()).float().cpu() for h in host]
        outs = OverlappedRunner(model, torch.device("cuda")).run(host)
        torch.cuda.synchronize()
    for a, b in zip(ref, outs):
        assert torch.equal(a, b)
