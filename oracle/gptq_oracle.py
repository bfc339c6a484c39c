"""CPU oracle for GPTQ weight quantization to NVFP4.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the ``vitfp4`` package, its CUDA library
or its C ABI) imports, links or executes this file; only ``tests/`` uses it, as the checker.

It restates in numpy float32 the reference's GPTQ (Dev-Jahn/vit-nvfp4,
``src/vit_nvfp4/ptq/gptq.py:53-129``):

* frozen scales ............ per-16 E4M3 block scales and the fp32 global of round-to-nearest
                             ("six") quantization of the original weight (gptq.py:37-50, 72-77)
* Hessian preparation ...... dead inputs (H[j, j] == 0: H[j, j] = 1, weight column zeroed),
                             damping by percdamp * mean(diag H), Hinv = upper Cholesky factor of
                             (H)^-1 (gptq.py:79-94)
* column loop .............. per block of ``blocksize`` columns, for each column i in order:
                             code = e2m1(w_i / s), q = value(code) * s, err = (w_i - q) / Hinv[i, i],
                             w[:, i:] -= err * Hinv[i, i:] (product rounded, then the subtraction);
                             after the block W[:, i2:] -= Err @ Hinv[i1:i2, i2:] (gptq.py:101-126)
* output codes ............. e2m1(Q / s), the reference's re-encoding of the dequantized result
                             (gptq.py:128-131)

Parity is PINNED by ``tests/golden/make_golden_gptq.py``, which runs the reference's own
``gptq_quantize_weight`` on CPU and stores its codes together with the inverse-Hessian factor its
steps produce: given that factor the column loop here reproduces the reference's codes bit for bit
(``tests/test_gptq_oracle.py``).  The Cholesky steps here use numpy's LAPACK and the cross-block
update numpy's matmul, which round differently from torch's; only the column loop is exact.
"""
from __future__ import annotations

import numpy as np

import nvfp4_oracle as nv

F32 = np.float32


def frozen_scales(W: np.ndarray):
    """(block-scale E4M3 bits (N, K/16), decode scale fp32 (N, K/16), global fp32) of RTN 'six'."""
    _, bs, gs = nv.quantize_to_nvfp4(np.asarray(W, F32), 16, block_select="six")
    return bs, (nv.e4m3_decode(bs) * F32(gs)).astype(F32), F32(gs)


def prepare_hinv(H: np.ndarray, W: np.ndarray, percdamp: float = 0.01) -> np.ndarray:
    """gptq.py:79-94 on a copy of H; zeroes the dead columns of W in place."""
    H = np.array(H, dtype=F32, copy=True)
    K = H.shape[0]
    dead = np.diagonal(H) == 0
    H[dead, dead] = F32(1.0)
    W[:, dead] = F32(0.0)
    idx = np.arange(K)
    H[idx, idx] += F32(percdamp) * F32(np.mean(np.diagonal(H), dtype=F32))
    L = np.linalg.cholesky(H).astype(F32)
    Linv = np.linalg.inv(L).astype(F32)
    Hi = (Linv.T @ Linv).astype(F32)
    return np.linalg.cholesky(Hi).T.astype(F32)   # upper factor U with U^T U = Hi


def column_block(W1: np.ndarray, Hinv1: np.ndarray, dq: np.ndarray):
    """The reference's inner loop over one block: W1 (N, c) fp32 (copied), Hinv1 (c, c), dq (N, c) the
    decode scale of each element's 16-block.  Returns (Q1 dequantized (N, c), Err1 (N, c))."""
    W1 = np.array(W1, dtype=F32, copy=True)
    N, c = W1.shape
    Q1 = np.zeros_like(W1)
    E1 = np.zeros_like(W1)
    with np.errstate(divide="ignore", invalid="ignore"):
        for i in range(c):
            w = W1[:, i].copy()
            s = dq[:, i]
            q = (nv.code_to_value(nv.round_to_e2m1_code((w / s).astype(F32))) * s).astype(F32)
            e = ((w - q).astype(F32) / Hinv1[i, i]).astype(F32)
            Q1[:, i] = q
            E1[:, i] = e
            W1[:, i:] = (W1[:, i:] - (e[:, None] * Hinv1[i, i:][None, :]).astype(F32)).astype(F32)
    return Q1, E1


def reencode(Q: np.ndarray, dq: np.ndarray) -> np.ndarray:
    """gptq.py:128-131: E2M1 codes of the dequantized GPTQ result."""
    with np.errstate(divide="ignore", invalid="ignore"):
        return nv.round_to_e2m1_code((Q / dq).astype(F32))


def gptq_quantize_weight(W: np.ndarray, H: np.ndarray, percdamp: float = 0.01, blocksize: int = 128,
                         Hinv: np.ndarray | None = None):
    """gptq.py:53-131.  Returns (codes uint8 (N, K), block-scale E4M3 bits (N, K/16), global fp32).
    ``Hinv`` given: use it instead of preparing one here (dead columns of W are still zeroed)."""
    W = np.array(W, dtype=F32, copy=True)
    N, K = W.shape
    bs, dqb, gs = frozen_scales(W)
    if Hinv is None:
        Hinv = prepare_hinv(H, W, percdamp)
    else:
        W[:, np.diagonal(np.asarray(H)) == 0] = F32(0.0)
    dq = np.repeat(dqb, 16, axis=1)
    Q = np.zeros_like(W)
    for i1 in range(0, K, blocksize):
        i2 = min(i1 + blocksize, K)
        Q1, E1 = column_block(W[:, i1:i2], Hinv[i1:i2, i1:i2], dq[:, i1:i2])
        Q[:, i1:i2] = Q1
        if i2 < K:
            W[:, i2:] = (W[:, i2:] - (E1 @ Hinv[i1:i2, i2:]).astype(F32)).astype(F32)
    return reencode(Q, dq), bs, gs
