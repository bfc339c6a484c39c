"""Accuracy metrics (reference: src/vit_nvfp4/ptq/diagnostics.py:5-8)."""
import torch
import torch.nn.functional as F


def tensor_cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    return float(F.cosine_similarity(a.flatten().float(), b.flatten().float(), dim=0))
