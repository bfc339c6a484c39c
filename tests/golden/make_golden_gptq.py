"""Generate the golden fixture that pins the GPTQ oracle (and the GPU column loop) to the reference.

Run once in a container that holds the reference source tree (Dev-Jahn/vit-nvfp4):

    python tests/golden/make_golden_gptq.py --reference-src <path-to>/vit-nvfp4/src

It runs the reference's own ``gptq_quantize_weight`` (src/vit_nvfp4/ptq/gptq.py:53) and
``quantize_to_nvfp4`` (src/vit_nvfp4/nvfp4/quant.py:20) on CPU for seeded weights and calibration
Hessians and writes ``tests/golden/golden_gptq.npz``.  The inverse-Hessian factor each call uses is
recorded by wrapping ``torch.linalg.cholesky`` while the reference runs (its last call, with
upper=True, returns that factor), so tests can feed the same factor to the oracle's and the GPU's
column loops.  The GPU box never runs this script; the tests only read the committed ``.npz``.

Cases:
  a  N=48,  K=128 (one 128-column block), one dead input column, weight outliers
  b  N=96,  K=256 (two blocks: exercises the cross-block update)
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_gptq.npz")


def _case(seed: int, N: int, K: int, M: int, dead: list[int]):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(N, K, generator=g) * 0.05
    W[3, 7] = 0.9                       # outliers: some blocks' scales far from the rest
    W[10, 40:44] = -0.6
    X = torch.randn(M, K, generator=g)
    X[:, 17] *= 6.0                     # a heavy input channel
    for j in dead:
        X[:, j] = 0.0
    return W, X.t() @ X


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("VIT_NVFP4_REFERENCE_SRC"),
                    help="the reference's src/ directory (or set VIT_NVFP4_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("pass --reference-src <vit-nvfp4>/src or set VIT_NVFP4_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)
    from vit_nvfp4.nvfp4.quant import quantize_to_nvfp4
    from vit_nvfp4.ptq import gptq as ref_gptq

    torch.set_num_threads(1)
    out: dict[str, np.ndarray] = {}
    for name, (seed, N, K, M, dead) in {"a": (1, 48, 128, 512, [5]), "b": (2, 96, 256, 1024, [])}.items():
        W, H = _case(seed, N, K, M, dead)
        seen = []
        real = torch.linalg.cholesky

        def recorder(A, *a, **kw):
            r = real(A, *a, **kw)
            seen.append(r.clone())
            return r

        torch.linalg.cholesky = recorder
        try:
            codes, bs, gs = ref_gptq.gptq_quantize_weight(W.clone(), H.clone(), block=16)
        finally:
            torch.linalg.cholesky = real
        rc, rbs, rgs = quantize_to_nvfp4(W.float(), 16)
        out[f"{name}_W"] = W.numpy()
        out[f"{name}_H"] = H.numpy()
        out[f"{name}_Hinv"] = seen[-1].numpy()
        out[f"{name}_codes"] = codes.numpy().astype(np.uint8)
        out[f"{name}_bs"] = bs.view(torch.uint8).numpy()
        out[f"{name}_gs"] = np.float32(gs.item())
        out[f"{name}_rtn_codes"] = rc.numpy().astype(np.uint8)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
