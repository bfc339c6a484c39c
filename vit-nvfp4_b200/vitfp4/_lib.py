"""ctypes binding of libvitfp4.so (the sm_100a kernels behind the C ABI in include/vitfp4.h).

There is no fallback: if the library is missing, or the device is not sm_100, every op
raises.  Pointers are taken from torch tensors (``data_ptr()``) and the stream is torch's
current CUDA stream.
"""
from __future__ import annotations

import ctypes
import os
import threading

_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libvitfp4.so")
_lock = threading.Lock()
_lib: ctypes.CDLL | None = None

VF4_BF16, VF4_F32 = 0, 1
VF4_SIX, VF4_MSE = 0, 1
VF4_ATTN_HEAD_GLOBALS = 1
VF4_ATTN_PACKED = 2
VF4_ATTN_NO_SMOOTH_K = 4
VF4_ATTN_NO_SMOOTH_V = 8
VF4_ATTN_MODE = {"bf16": 0, "fp8": 1, "nvfp4": 2}
VF4_EPI_NONE, VF4_EPI_BIAS, VF4_EPI_GELU_NVFP4, VF4_EPI_GELU_ERF_NVFP4, VF4_EPI_BIAS_RESIDUAL = 0, 1, 2, 3, 4

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64

# name -> argtypes (all return int status unless listed in _RESTYPE)
SIGNATURES: dict[str, list] = {
    "vf4_version": [],
    "vf4_last_error_string": [],
    "vf4_device_error": [_I],
    "vf4_selftest_wait_timeout": [ctypes.c_uint64, _P],
    "vf4_amax": [_P, _I, _L, _I, _P, _P],
    "vf4_gelu_erf_f32": [_P, _L, _P, _P],
    "vf4_global_scale": [_P, _I, _P, _P],
    "vf4_cast_nvfp4": [_P, _I, _L, _L, _L, _P, _I, _I, _P, _P, _P, _P, _P, _P],
    "vf4_ln_cast_nvfp4": [_P, _P, _P, _P, _P, _P, ctypes.c_float, _L, _L, _P, _P, _P, _P, _P],
    "vf4_pack_e2m1": [_P, _L, _L, _P, _P],
    "vf4_unpack_e2m1": [_P, _L, _L, _P, _P],
    "vf4_to_blocked": [_P, _L, _L, _P, _P],
    "vf4_gemm_nvfp4": [_P, _P, _P, _P, _P, _P, _L, _L, _L, _P, _I, _P, _I, _P, _P, _P, _P],
    "vf4_gemm_nvfp4_residual": [_P, _P, _P, _P, _P, _P, _L, _L, _L, _P, _P, _P, _P, _P],
    "vf4_gemm_nvfp4_ex": [_P, _P, _P, _P, _P, _P, _P, _L, _L, _L, _P, _I, _P, _I, _P, _P, _P, _P, _P, _P],
    "vf4_b_scale_image": [_P, _L, _L, _P, _P],
    "vf4_b_scale_image_bytes": [_L, _L],
    "vf4_attn_workspace_size": [_L, _L, _L, _L],
    "vf4_attn_workspace_size_ex": [_L, _L, _L, _L, _I],
    "vf4_patchify": [_P, _L, _L, _L, _L, _L, _L, _P, _P],
    "vf4_cast_nvfp4_split": [_P, _L, _P, _L, _L, _L, _P, _P, _P, _P, _P],
    "vf4_embed_tokens": [_P, _P, _P, _L, _L, _L, _P, _P],
    "vf4_attn_nvfp4": [_P, _P, _P, _L, _L, _L, _L, _L, _L, _L, ctypes.c_float, _P, _L, _L, _L, _P, _L, _P],
    "vf4_attn_nvfp4_ex": [_P, _P, _P, _L, _L, _L, _L, _L, _L, _L, ctypes.c_float, _P, _L, _L, _L, _I, _P, _L, _P],
    "vf4_attn_fp8": [_P, _P, _P, _L, _L, _L, _L, _L, _L, _L, ctypes.c_float, _P, _L, _L, _L, _P],
    "vf4_attn_bf16": [_P, _P, _P, _L, _L, _L, _L, _L, _L, _L, ctypes.c_float, _P, _L, _L, _L, _P, _P],
    "vf4_attn_nvfp4_noalloc": [_P, _P, _P, _L, _L, _L, _L, _L, _L, _L, ctypes.c_float, _P, _L, _L, _L, _P],
    "vf4_attn": [_P, _P, _P, _L, _L, _L, _L, _L, _L, _L, ctypes.c_float, _I, _I, _I, _P, _L, _P, _L, _L, _L, _P],
    "vf4_attn_workspace_size_modes": [_L, _L, _L, _L, _I, _I, _I],
    "vf4_gptq_block": [_P, _L, _P, _L, _P, _L, _P, _L, _L, _L, _P, _L, _P, _L, _P],
}
_RESTYPE = {"vf4_last_error_string": ctypes.c_char_p, "vf4_attn_workspace_size": ctypes.c_int64,
            "vf4_attn_workspace_size_ex": ctypes.c_int64, "vf4_attn_workspace_size_modes": ctypes.c_int64,
            "vf4_b_scale_image_bytes": ctypes.c_int64}


class VitFp4Error(RuntimeError):
    pass


def library_path() -> str:
    return _PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(_PATH):
                    raise VitFp4Error(
                        f"{_PATH} is not built; run `python -m vitfp4._build` (nvcc, sm_100a). "
                        "vitfp4 has no CPU or eager fallback.")
                cdll = ctypes.CDLL(_PATH)
                for name, args in SIGNATURES.items():
                    fn = getattr(cdll, name)
                    fn.argtypes = args
                    fn.restype = _RESTYPE.get(name, ctypes.c_int)
                _lib = cdll
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().vf4_last_error_string().decode(errors="replace")
        raise VitFp4Error(f"{what} failed (status {status}): {msg}")


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args), name)


def device_error(clear: bool = True) -> int:
    """Device-side error word of all kernel families (0 = none). Synchronizes."""
    return int(lib().vf4_device_error(1 if clear else 0))
