"""Nibble packing and the 128x4 scale-factor swizzle (reference: src/vit_nvfp4/nvfp4/pack.py:4-58).

``pack_e2m1`` / ``unpack_e2m1`` / ``to_blocked`` run the CUDA kernels of libvitfp4.so;
``pad_to_block`` and ``as_float4_x2`` are shape/dtype utilities.
"""
import torch

from . import ops


def pack_e2m1(codes: torch.Tensor) -> torch.Tensor:
    """Two E2M1 codes per byte: low nibble = even index, high nibble = odd index."""
    assert codes.shape[-1] % 2 == 0 and codes.dtype == torch.uint8
    return ops.pack_e2m1(codes)


def unpack_e2m1(packed: torch.Tensor) -> torch.Tensor:
    return ops.unpack_e2m1(packed)


def pad_to_block(x: torch.Tensor, block: int = 16, dim: int = -1):
    """Right-pad ``x`` with zeros along ``dim`` to a multiple of ``block``; returns (padded, orig_len)."""
    orig = x.shape[dim]
    pad = (-orig) % block
    if pad:
        x = x.movedim(dim, -1)
        x = torch.nn.functional.pad(x, (0, pad))
        x = x.movedim(-1, dim)
    return x, orig


def as_float4_x2(packed: torch.Tensor) -> torch.Tensor:
    return packed.view(torch.float4_e2m1fn_x2)


def to_blocked(input_matrix: torch.Tensor) -> torch.Tensor:
    """(R, C) E4M3 block scales -> flat 128x4-tiled layout (rows padded to 128, columns to 4)."""
    out = ops.to_blocked(input_matrix)
    return out.view(torch.float8_e4m3fn) if input_matrix.dtype == torch.float8_e4m3fn else out
