"""W4A4 ``nn.Linear`` replacement (reference: src/vit_nvfp4/ptq/qlinear.py:7-50).

Same constructor, buffers (``w_codes``, ``w_block_scale``, ``w_global_scale``,
``x_global_scale``, ``bias``) and methods as the reference, so converted state_dicts load
unchanged.  The forward runs the CUDA cast of the activation and the tcgen05 FP4 GEMM with a
fused bias epilogue; the weight is packed + swizzled once into non-persistent device buffers
(rebuilt if the weight buffers change) instead of on every call.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..nvfp4 import ops
from ..nvfp4.quant import quantize_to_nvfp4


@torch.library.custom_op("vitfp4::qlinear", mutates_args=())
def qlinear_op(x: torch.Tensor, w_packed: torch.Tensor, w_sf: torch.Tensor, w_gs: torch.Tensor,
               x_gs: torch.Tensor | None, bias: torch.Tensor | None) -> torch.Tensor:
    ap, asf, _, ag = ops.cast(x, x_gs, "six")
    out_dtype = torch.float32 if x.dtype == torch.float32 else torch.bfloat16
    y = ops.gemm(ap, asf, ag, w_packed, w_sf, w_gs, bias=bias, out_dtype=out_dtype)
    return y if y.dtype == x.dtype else y.to(x.dtype)


@qlinear_op.register_fake
def _(x, w_packed, w_sf, w_gs, x_gs, bias):
    return x.new_empty(x.shape[0], w_packed.shape[0])


class QuantLinear(nn.Module):
    """nn.Linear with a statically NVFP4-quantized weight and online NVFP4 activations (W4A4)."""

    def __init__(self, w_codes, w_block_scale, w_global_scale, bias, in_features, out_features):
        super().__init__()
        assert in_features % 16 == 0, "NVFP4 requires in_features (K) divisible by 16"
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("w_codes", w_codes)
        self.register_buffer("w_block_scale", w_block_scale)
        self.register_buffer("w_global_scale", w_global_scale)
        self.register_buffer("x_global_scale", None)   # static activation global (calibrated) or None
        if bias is not None:
            self.register_buffer("bias", bias.detach().clone())
        else:
            self.bias = None
        self.register_buffer("w_packed", None, persistent=False)
        self.register_buffer("w_sf", None, persistent=False)
        self._packed_key = None

    def set_activation_scale(self, scale: torch.Tensor) -> None:
        """Pin a static per-tensor activation global scale."""
        self.x_global_scale = scale.detach().to(torch.float32).reshape(()).clone()

    @classmethod
    def from_linear(cls, linear: nn.Linear, w_block_select: str = "mse") -> "QuantLinear":
        w = linear.weight.data
        codes, bscale, gscale = quantize_to_nvfp4(w.float(), 16, block_select=w_block_select)
        return cls(codes, bscale, gscale, linear.bias, linear.in_features, linear.out_features)

    @staticmethod
    def _version(t: torch.Tensor) -> int:
        try:
            return t._version
        except RuntimeError:   # inference-mode tensors carry no version counter
            return -1

    def _packed_weight(self):
        key = (self.w_codes.data_ptr(), self._version(self.w_codes), self.w_block_scale.data_ptr(),
               self._version(self.w_block_scale), self.w_codes.device)
        if self.w_packed is None or key != self._packed_key:
            self.w_packed = ops.pack_e2m1(self.w_codes.contiguous())
            self.w_sf = ops.to_blocked(self.w_block_scale.contiguous())
            self._packed_key = key
        return self.w_packed, self.w_sf

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out_shape = (*x.shape[:-1], self.out_features)
        wp, wsf = self._packed_weight()
        y = qlinear_op(x.reshape(-1, self.in_features), wp, wsf, self.w_global_scale, self.x_global_scale,
                       self.bias)
        return y.reshape(out_shape)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, nvfp4=W4A4"
