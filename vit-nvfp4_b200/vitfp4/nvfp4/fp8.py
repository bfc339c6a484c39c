"""FP8 E4M3 per-row quantize-dequantize (reference: src/vit_nvfp4/nvfp4/fp8.py:6-17)."""
import torch

from . import format as fmt


def fp8_e4m3_quant_dequant(x: torch.Tensor) -> torch.Tensor:
    xf = x.to(torch.float32)
    amax = xf.abs().amax(dim=-1, keepdim=True).clamp(min=1e-12)
    scale = amax / fmt.E4M3_MAX
    q = (xf / scale).clamp(-fmt.E4M3_MAX, fmt.E4M3_MAX).to(torch.float8_e4m3fn)
    return q.to(torch.float32) * scale
