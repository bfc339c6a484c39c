"""vitfp4 — B200-native (sm_100a) NVFP4 W4A4 inference path for Vision Transformers.

Python host code over hand-written CUDA kernels (libvitfp4.so, C ABI in include/vitfp4.h).
"""
from . import nvfp4  # noqa: F401

__version__ = "0.1.0"
