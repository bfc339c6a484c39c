"""GPTQ weight quantization to NVFP4 on the GPU (reference: src/vit_nvfp4/ptq/gptq.py:17-129).

Same API and output as the reference: ``HessianObserver`` accumulates H = sum x x^T over the
calibration inputs of one Linear; ``gptq_quantize_weight(weight, H, block=16, percdamp=0.01,
blocksize=128)`` returns ``(codes, block_scale_e4m3, global_scale)`` in the format of
``quantize_to_nvfp4``.  The per-16 block scales and the global are those of round-to-nearest
("six") quantization of the original weight, frozen; GPTQ only chooses the codes, quantizing the
input columns in order and pushing each column's error, through the upper Cholesky factor of the
damped inverse Hessian, onto the columns not yet quantized.

Where the work runs: the block scales and global come from the CUDA cast kernel; the Hessian
preparation (dead columns, damping, Cholesky factorisations) and the update of the later columns
after each block of ``blocksize`` columns (one GEMM) are torch / cuSOLVER / cuBLAS calls in fp32;
the column loop inside a block -- the reference's Python loop of small torch ops per column
(gptq.py:101-122) -- is one launch of the ``vf4_gptq_block`` kernel per block, a warp per weight
row.  Given the same Hinv the codes are bit-identical to the reference's; across devices the
Cholesky factors and the GEMMs round differently, so codes can differ where a value sits on a
rounding boundary.
"""
from __future__ import annotations

import torch

from ..nvfp4 import ops


class HessianObserver:
    """Running H = sum over calibration rows of x x^T for a Linear with ``in_features`` inputs."""

    def __init__(self, in_features: int):
        self.in_features = in_features
        self.H = torch.zeros(in_features, in_features, dtype=torch.float32)
        self.nsamples = 0

    @torch.no_grad()
    def observe(self, x: torch.Tensor) -> None:
        rows = x.detach().reshape(-1, self.in_features).to(torch.float32)
        if rows.shape[0] == 0:
            return
        if self.H.device != rows.device:
            self.H = self.H.to(rows.device)
        self.H += rows.t() @ rows
        self.nsamples += rows.shape[0]


def _fp32_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a @ b in full fp32 whatever the process-wide TF32 setting (the reference's CPU matmul is fp32)."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return a @ b
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def inverse_hessian_factor(H: torch.Tensor, W: torch.Tensor, percdamp: float = 0.01) -> torch.Tensor:
    """The upper Cholesky factor of (H + damping)^-1 that drives the column updates.

    Inputs with no calibration energy (H[j, j] == 0) get H[j, j] = 1 and their weight column zeroed
    in place in ``W``; the diagonal is then damped by ``percdamp`` times its mean (gptq.py:79-94)."""
    H = H.clone()
    K = H.shape[0]
    dead = torch.diagonal(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    idx = torch.arange(K, device=H.device)
    H[idx, idx] += percdamp * torch.diagonal(H).mean()
    inv = torch.cholesky_inverse(torch.linalg.cholesky(H))
    return torch.linalg.cholesky(inv, upper=True).contiguous()


@torch.no_grad()
def gptq_quantize_weight(weight: torch.Tensor, H: torch.Tensor, block: int = 16, percdamp: float = 0.01,
                         blocksize: int = 128):
    """GPTQ-quantize one (N, K) Linear weight to NVFP4 given its (K, K) calibration Hessian.

    Returns (codes uint8 (N, K), block_scale float8_e4m3fn (N, K/16), global_scale fp32 0-dim) on the
    weight's (CUDA) device."""
    if block != 16:
        raise ValueError("NVFP4 blocks are 16 wide")
    if blocksize % 16 or not 16 <= blocksize <= 128:
        raise ValueError("blocksize must be a multiple of 16 in [16, 128] (one kernel launch per block)")
    W = weight.detach().to(torch.float32).clone()
    if not W.is_cuda:
        raise RuntimeError("gptq_quantize_weight runs on the GPU (CUDA weight required)")
    N, K = W.shape
    if K % 16:
        raise ValueError("NVFP4 needs in_features divisible by 16")
    # frozen scales: round-to-nearest "six" quantization of the original weight
    _, _, bscale, gscale = ops.cast(W, None, "six", swizzled=False, linear=True)
    Hinv = inverse_hessian_factor(H.to(W.device, torch.float32), W, percdamp)
    codes = torch.empty(N, K, dtype=torch.uint8, device=W.device)
    for i1 in range(0, K, blocksize):
        i2 = min(i1 + blocksize, K)
        err = torch.empty(N, i2 - i1, dtype=torch.float32, device=W.device)
        ops.gptq_block(W[:, i1:], Hinv[i1:i2, i1:i2], bscale, gscale, i1, i2 - i1, codes, err)
        if i2 < K:
            W[:, i2:] -= _fp32_matmul(err, Hinv[i1:i2, i2:])
    return codes, bscale.view(torch.float8_e4m3fn), gscale
