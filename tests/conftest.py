"""Shared test setup: import paths, the oracle, golden fixtures and the ``gpu`` marker."""
import functools
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "vit-nvfp4_b200")
for p in (PKG_DIR, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _load_oracle():
    spec = importlib.util.spec_from_file_location("nvfp4_oracle", os.path.join(ROOT, "oracle", "nvfp4_oracle.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


oracle = _load_oracle()


@functools.lru_cache(maxsize=1)
def golden():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden_nvfp4.npz")))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
