"""NVFP4 numeric-format constants and the E2M1 code helpers.

Mirrors src/vit_nvfp4/nvfp4/format.py:3-33 of the reference (Dev-Jahn/vit-nvfp4): the same
constants and the same code <-> value mapping.  These are small tensor utilities (they run on
whatever device their input lives on); the quantizer itself is the CUDA cast kernel.
"""
import torch

E2M1_MAX = 6.0
E4M3_MAX = 448.0
# Four Over Six: the per-tensor global uses 256 so the scale-to-4 candidate stays in E4M3 range
FOS_SCALE_MAX = 256.0

_MAG = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)
_MID = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=torch.float32)


def round_to_e2m1_code(scaled: torch.Tensor) -> torch.Tensor:
    """Nearest E2M1 code (bit3 = sign, bits2..0 = magnitude index); ties to the smaller magnitude."""
    sign = (scaled < 0).to(torch.uint8)
    mag = scaled.abs().clamp(max=E2M1_MAX)
    idx = torch.bucketize(mag, _MID.to(mag.device)).to(torch.uint8)
    return (sign << 3) | idx


def code_to_value(code: torch.Tensor) -> torch.Tensor:
    code = code.to(torch.long)
    sign = 1.0 - 2.0 * ((code >> 3) & 1).to(torch.float32)
    return sign * _MAG.to(code.device)[code & 0x7]
