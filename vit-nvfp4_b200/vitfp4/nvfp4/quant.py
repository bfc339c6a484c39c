"""Two-level NVFP4 quantizer (reference: src/vit_nvfp4/nvfp4/quant.py:20-76).

``quantize_to_nvfp4`` runs the CUDA cast kernel, which is bit-exact to the reference's
arithmetic (RTN "six" and Four-Over-Six "mse" block selection, static or dynamic global),
and returns the reference's tensors: unpacked codes, row-major E4M3 scales, fp32 global.
"""
import torch

from . import format as fmt
from . import ops


def quantize_to_nvfp4(x: torch.Tensor, block: int = 16, global_scale: torch.Tensor | None = None,
                      block_select: str = "six"):
    """Returns (codes uint8 (..., K), block_scale float8_e4m3fn (..., K/16), global_scale fp32 0-dim)."""
    assert block == 16, "NVFP4 block is 16"
    assert x.shape[-1] % block == 0, "K must be a multiple of block; pad first"
    assert block_select in ("six", "mse")
    packed, _, sfl, gs = ops.cast(x, global_scale, block_select, swizzled=False, linear=True)
    codes = ops.unpack_e2m1(packed).reshape(x.shape)
    bs = sfl.view(torch.float8_e4m3fn).reshape(*x.shape[:-1], x.shape[-1] // block)
    return codes, bs, gs


def dequantize_nvfp4(codes: torch.Tensor, block_scale_e4m3: torch.Tensor, global_scale: torch.Tensor):
    block = codes.shape[-1] // block_scale_e4m3.shape[-1]
    vals = fmt.code_to_value(codes).reshape(*codes.shape[:-1], block_scale_e4m3.shape[-1], block)
    scale = (block_scale_e4m3.to(torch.float32) * global_scale).unsqueeze(-1)
    return (vals * scale).reshape(codes.shape)
