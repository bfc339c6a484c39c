"""block_output_cosines (reference: src/vit_nvfp4/ptq/diagnostics.py:11-42) on CPU models."""
import copy

import torch
import torch.nn as nn


class _Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.blocks = nn.ModuleList(nn.Sequential(nn.Linear(16, 16), nn.GELU()) for _ in range(3))

    def forward(self, x):
        for b in self.blocks:
            x = x + b(x)
        return x


def test_block_output_cosines_localises_a_change():
    from vitfp4.ptq import block_output_cosines
    torch.manual_seed(0)
    ref = _Net()
    q = copy.deepcopy(ref)
    with torch.no_grad():
        q.blocks[1][0].weight.add_(0.3 * torch.randn(16, 16))
    x = torch.randn(4, 16)
    cos = block_output_cosines(ref, q, x)
    assert len(cos) == 3 and abs(cos[0] - 1.0) < 1e-6 and cos[1] < 0.999
    assert block_output_cosines(ref, q, x, block_container="blocks") == cos
