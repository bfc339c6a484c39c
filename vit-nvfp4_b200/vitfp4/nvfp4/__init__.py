"""NVFP4 core: quantizer, packing, block-scaled FP4 GEMM and low-precision attention.

API mirrors src/vit_nvfp4/nvfp4/__init__.py of the reference (Dev-Jahn/vit-nvfp4); every op
runs the sm_100a kernels of libvitfp4.so.
"""
from .quant import quantize_to_nvfp4, dequantize_nvfp4
from .pack import pack_e2m1, unpack_e2m1, pad_to_block, as_float4_x2, to_blocked
from .gemm import (nvfp4_gemm, nvfp4_linear, register_backend, available_backends, gemm_packed,
                   cast_nvfp4, linear_packed)
from .fp8 import fp8_e4m3_quant_dequant
from .attention import quant_sdpa

__all__ = [
    "quantize_to_nvfp4", "dequantize_nvfp4",
    "pack_e2m1", "unpack_e2m1", "pad_to_block", "as_float4_x2", "to_blocked",
    "nvfp4_gemm", "nvfp4_linear", "register_backend", "available_backends", "gemm_packed",
    "cast_nvfp4", "linear_packed",
    "fp8_e4m3_quant_dequant", "quant_sdpa",
]
