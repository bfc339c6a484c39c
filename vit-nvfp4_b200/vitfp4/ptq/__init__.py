"""Post-training W4A4 conversion and the quantized modules (reference API: src/vit_nvfp4/ptq/__init__.py)."""
from .qlinear import QuantLinear
from .policy import vit_block_policy, block_index
from .qattention import enable_quant_attention, vit_attn_policy
from .fused_mlp import FusedNVFP4MLP, fuse_mlps
from .fused_block import FusedNVFP4Block, fuse_norms
from .convert import quantize_model
from .models import ModelSpec, model_spec, find_block_container, quantize_vit
from .diagnostics import block_output_cosines, tensor_cosine
from .gptq import HessianObserver, gptq_quantize_weight
from .convert_gptq import quantize_model_gptq
from .calibrate import calibrate_activations
from .bias_correction import correct_bias

__all__ = [
    "QuantLinear", "vit_block_policy", "block_index", "enable_quant_attention", "vit_attn_policy",
    "FusedNVFP4MLP", "fuse_mlps", "quantize_model", "ModelSpec", "model_spec", "find_block_container",
    "quantize_vit", "tensor_cosine", "FusedNVFP4Block", "fuse_norms", "HessianObserver", "gptq_quantize_weight",
    "quantize_model_gptq", "block_output_cosines", "calibrate_activations", "correct_bias",
]
