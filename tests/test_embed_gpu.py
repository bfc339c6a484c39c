"""Token embedding kernels of the ViT forward: the patch unfold ahead of the patch-projection GEMM and
the class-token / position-embedding assembly, against the torch ops they replace."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,C,H,W,p,kp", [(2, 3, 224, 224, 14, 592), (3, 3, 224, 224, 16, 768), (1, 3, 448, 448, 14, 600),
                                          (2, 4, 32, 48, 8, 256)])
def test_patchify_equals_unfold(B, C, H, W, p, kp):
    from vitfp4.nvfp4 import ops
    x = torch.randn(B, C, H, W, device="cuda").bfloat16()
    got = ops.patchify(x, p, kp)
    K = C * p * p
    ref = x.reshape(B, C, H // p, p, W // p, p).permute(0, 2, 4, 1, 3, 5).reshape(-1, K)
    torch.cuda.synchronize()
    assert torch.equal(got[:, :K], ref)
    assert not got[:, K:].any()


@pytest.mark.parametrize("B,T,D", [(3, 257, 1024), (2, 197, 384), (1, 2, 8)])
def test_embed_tokens_equals_cat_add(B, T, D):
    from vitfp4.nvfp4 import ops
    y = torch.randn(B, T - 1, D, device="cuda").bfloat16()
    cls = torch.randn(1, 1, D, device="cuda").bfloat16()
    pos = torch.randn(1, T, D, device="cuda").bfloat16()
    got = ops.embed_tokens(y, cls, pos)
    ref = torch.cat([cls.expand(B, -1, -1), y], dim=1) + pos
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


def test_vit_embedding_path_matches_torch_ops():
    from vitfp4 import vit
    cfg = dict(vit.VIT_L14)
    cfg["depth"] = 1
    model = vit.build_vit(seed=5, **cfg).to(device="cuda", dtype=torch.bfloat16).eval()
    x = torch.randn(2, 3, 224, 224, device="cuda").bfloat16()
    pe = model.patch_embed
    with torch.inference_mode():
        got = pe(x)
        p = pe.patch
        patches = x.reshape(2, 3, 16, p, 16, p).permute(0, 2, 4, 1, 3, 5).reshape(2, 256, 3 * p * p)
        ref = F.linear(patches.float(), pe.proj.weight.reshape(pe.proj.out_channels, -1).float(),
                       pe.proj.bias.float())
    torch.cuda.synchronize()
    err = (got.float() - ref).abs().max()
    assert err <= 2e-2 * ref.abs().max(), err   # bf16 output rounding of an fp32-accumulated GEMM
