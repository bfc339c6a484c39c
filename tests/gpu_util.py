"""Helpers shared by the GPU parity tests: seeded inputs, oracle-side operand preparation."""
import numpy as np
import torch

from conftest import oracle


def bf16_tensor(x: np.ndarray) -> torch.Tensor:
    """fp32 numpy -> bf16 CUDA tensor (RNE, same rounding as the oracle's to_bf16)."""
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to("cuda").to(torch.bfloat16)


def f32_of_bf16(x: np.ndarray) -> np.ndarray:
    return oracle.to_bf16(x)


def vit_activation(M, K, seed=0, outlier_frac=0.001, scale=1.0):
    """BASELINE config-2 style activations: N(0,1) with ceil(0.1% K) channels scaled x20."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((M, K), dtype=np.float32) * np.float32(scale)
    n_out = max(1, int(np.ceil(outlier_frac * K)))
    ch = rng.permutation(K)[:n_out]
    x[:, ch] *= np.float32(20.0)
    return x


def oracle_operand(x: np.ndarray, mode="six", gs=None):
    """Oracle-quantize x (M, K) -> (codes, bs_bits, gs, packed, sf_swizzled) as numpy."""
    c, b, g = oracle.quantize_to_nvfp4(x, 16, global_scale=gs, block_select=mode)
    return c, b, g, oracle.pack_e2m1(c), oracle.to_blocked(b)


def to_cuda_operand(packed, sfs, gs):
    return (torch.from_numpy(packed).cuda(), torch.from_numpy(sfs).cuda(),
            torch.tensor(np.float32(gs), device="cuda"))


def cos(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))
