"""W4A4 ``nn.Linear`` replacement (reference: src/vit_nvfp4/ptq/qlinear.py:7-50).

Same constructor, buffers (``w_codes``, ``w_block_scale``, ``w_global_scale``,
``x_global_scale``, ``bias``) and methods as the reference, so converted state_dicts load
unchanged.  The forward runs the CUDA cast of the activation and the tcgen05 FP4 GEMM with a
fused bias epilogue; the weight is packed + swizzled once into device buffers (rebuilt if the
weight buffers change) instead of on every call.

Packed format: ``persist_packed()`` also keeps those GEMM-ready bytes in ``state_dict``
(``w_packed``: ``pack_e2m1`` of the codes, (N, K/2) uint8; ``w_sf``: ``to_blocked`` of the E4M3
scales, flat uint8) so a loaded model runs without repacking, and ``from_packed`` builds a module
from those bytes alone.  The reference stores unpacked codes and repacks on every call
(qlinear.py:19-21, backends/torch_scaled_mm.py:19-22); it has no packed export format.
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

    def _weight_key(self):
        return (self.w_codes.data_ptr(), self._version(self.w_codes), self.w_block_scale.data_ptr(),
                self._version(self.w_block_scale), self.w_codes.device)

    def persist_packed(self, on: bool = True) -> "QuantLinear":
        """Keep (or stop keeping) the packed + swizzled weight in state_dict as w_packed / w_sf."""
        self._packed_weight()
        for name in ("w_packed", "w_sf"):
            if on:
                self._non_persistent_buffers_set.discard(name)
            else:
                self._non_persistent_buffers_set.add(name)
        return self

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        packed = prefix + "w_packed" in state_dict and prefix + "w_sf" in state_dict
        if packed:   # the stored GEMM-ready bytes are taken as they are (allocated here if absent)
            for name in ("w_packed", "w_sf"):
                t = state_dict[prefix + name]
                if getattr(self, name) is None or getattr(self, name).shape != t.shape:
                    setattr(self, name, torch.empty_like(t, device=self.w_codes.device))
            self._non_persistent_buffers_set.difference_update({"w_packed", "w_sf"})
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)
        if packed:
            self._packed_key = self._weight_key()

    @classmethod
    def from_packed(cls, w_packed, w_sf, w_global_scale, bias, in_features, out_features,
                    x_global_scale=None) -> "QuantLinear":
        """A QuantLinear from GEMM-ready bytes: ``w_packed`` (N, K/2) uint8 (or float4_e2m1fn_x2) and
        ``w_sf`` the to_blocked E4M3 scales; the reference's unpacked buffers are derived on the device."""
        wp = w_packed.view(torch.uint8).reshape(out_features, in_features // 2)
        sf = w_sf.view(torch.uint8).reshape(-1)
        nb = in_features // 16
        rp, cp = (out_features + 127) // 128 * 128, (nb + 3) // 4 * 4
        # inverse of to_blocked: tile (rb, cb) at (rb * ncb + cb) * 512, element (r, c) at (r%32)*16 + (r//32)*4 + c
        tiles = sf.reshape(rp // 128, cp // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(rp, cp)
        codes = ops.unpack_e2m1(wp)
        q = cls(codes, tiles[:out_features, :nb].contiguous().view(torch.float8_e4m3fn),
                w_global_scale.reshape(()).float(), bias, in_features, out_features)
        if x_global_scale is not None:
            q.set_activation_scale(x_global_scale)
        q.w_packed, q.w_sf = wp.contiguous(), sf.contiguous()
        q._packed_key = q._weight_key()
        return q

    def _packed_weight(self):
        key = self._weight_key()
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
