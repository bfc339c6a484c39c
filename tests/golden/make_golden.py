"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once in a container that holds the reference source tree (Dev-Jahn/vit-nvfp4):

    python tests/golden/make_golden.py --reference-src <path-to>/vit-nvfp4/src

It imports the reference package, runs its own CPU functions on seeded inputs and
writes ``tests/golden/golden_nvfp4.npz``.  The GPU box never runs this script; the
tests only read the committed ``.npz``.

Reference functions exercised (file:line in the reference project):
  format.round_to_e2m1_code ........ src/vit_nvfp4/nvfp4/format.py:17
  quant.quantize_to_nvfp4 .......... src/vit_nvfp4/nvfp4/quant.py:20  (six, mse, static global)
  pack.pack_e2m1 / to_blocked ...... src/vit_nvfp4/nvfp4/pack.py:4, :39
  backends.reference.gemm .......... src/vit_nvfp4/nvfp4/backends/reference.py:6
  attention.quant_sdpa ............. src/vit_nvfp4/nvfp4/attention.py:53
  fp8.fp8_e4m3_quant_dequant ....... src/vit_nvfp4/nvfp4/fp8.py:6
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_nvfp4.npz")


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def _edge_block_matrix() -> torch.Tensor:
    """Rows of hand-picked 16-element blocks: ties, zero blocks, tiny, huge, signed zeros."""
    rows = []
    mids = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0]
    # row 0: a 6.0-max block whose other values land exactly on E2M1 midpoints (scale 1)
    r = [6.0] + mids + [-m for m in mids] + [0.0]
    rows.append(r[:16] + [0.0] * 48)
    # row 1: all-zero blocks and a block of signed zeros
    rows.append([0.0] * 32 + [-0.0] * 16 + [0.0] * 16)
    # row 2: single tiny non-zero in otherwise-zero blocks, plus a huge block
    rows.append([1e-30] + [0.0] * 15 + [-3e-8] + [0.0] * 15 + [1e4] * 16 + [7.0, -7.0] * 8)
    # row 3: values whose block scale lands on E4M3 subnormals / the 448 clamp
    rows.append([2.0 ** -12] * 16 + [2.0 ** -20] * 16 + [3.0 ** i for i in range(16)] + [0.1 * i for i in range(16)])
    return torch.tensor(rows, dtype=torch.float32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("VIT_NVFP4_REFERENCE_SRC"),
                    help="the reference's src/ directory (or set VIT_NVFP4_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("pass --reference-src <vit-nvfp4>/src or set VIT_NVFP4_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)
    from vit_nvfp4.nvfp4 import format as fmt
    from vit_nvfp4.nvfp4 import gemm as G
    from vit_nvfp4.nvfp4.quant import quantize_to_nvfp4, dequantize_nvfp4
    from vit_nvfp4.nvfp4.pack import pack_e2m1, to_blocked
    from vit_nvfp4.nvfp4.attention import quant_sdpa
    from vit_nvfp4.nvfp4.fp8 import fp8_e4m3_quant_dequant
    G._BACKENDS.pop("torch_scaled_mm_v2", None)   # CPU: use the fp32 emulation backend

    torch.set_num_threads(1)
    out: dict[str, np.ndarray] = {}

    # --- E2M1 rounding points (format.py:17) ---
    pts = torch.tensor([0.0, -0.0, 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 0.6, 0.8, 1.2, 5.5, 7.0, -0.6,
                        -0.75, -5.0, 6.0, -6.0, 1e9, -1e9, float("inf"), float("-inf"), float("nan"),
                        0.2499999, 0.2500001, 4.9999995, 5.0000005], dtype=torch.float32)
    out["e2m1_in"] = pts.numpy()
    out["e2m1_codes"] = fmt.round_to_e2m1_code(pts).numpy()

    # --- E4M3 RNE conversion (torch .to(float8_e4m3fn)) over a dense sweep ---
    g = torch.Generator().manual_seed(7)
    sweep = torch.cat([
        torch.exp2(torch.empty(6000).uniform_(-14, 9, generator=g)),
        torch.arange(0, 512, dtype=torch.float32) * 2.0 ** -10,          # subnormal grid + ties
        torch.tensor([448.0, 447.99, 440.0, 432.0, 2.0 ** -6, 2.0 ** -7, 2.0 ** -10, 3 * 2.0 ** -11]),
    ]).float()
    out["e4m3_in"] = sweep.numpy()
    out["e4m3_bits"] = sweep.to(torch.float8_e4m3fn).view(torch.uint8).numpy()

    # --- quantize_to_nvfp4 cases (quant.py:20) ---
    cases = []
    gq = torch.Generator().manual_seed(0)

    def add(name, x, mode, static=None, bf16=False):
        xin = x.to(torch.bfloat16).float() if bf16 else x.float()
        gs_arg = None if static is None else torch.tensor(static, dtype=torch.float32)
        c, b, gsv = quantize_to_nvfp4(xin, 16, global_scale=gs_arg, block_select=mode)
        cases.append(name)
        out[f"q_{name}_x"] = _bf16_bits(xin) if bf16 else xin.numpy()
        out[f"q_{name}_codes"] = c.numpy()
        out[f"q_{name}_bs"] = b.view(torch.uint8).numpy()
        out[f"q_{name}_gs"] = np.array(gsv.float().reshape(()).item(), np.float32)
        out[f"q_{name}_meta"] = np.array([1 if mode == "mse" else 0, -1.0 if static is None else static, int(bf16)],
                                         np.float64)

    for mode in ("six", "mse"):
        add(f"edge_{mode}", _edge_block_matrix(), mode)
        add(f"m1k16_{mode}", torch.randn(1, 16, generator=gq), mode)
        add(f"m17k80_{mode}", torch.randn(17, 80, generator=gq) * 3, mode, bf16=True)
        add(f"m100k64_{mode}", torch.randn(100, 64, generator=gq), mode, bf16=True)
        x = torch.randn(197, 128, generator=gq)
        x[:, 5] *= 20.0                                                      # outlier channel
        add(f"m197k128_{mode}", x, mode, bf16=True)
        add(f"m8k3072_{mode}", torch.randn(8, 3072, generator=gq) * 0.02, mode)
        heavy = torch.randn(64, 256, generator=gq) * torch.empty(64, 256).exponential_(0.5, generator=gq)
        add(f"heavy_{mode}", heavy, mode, bf16=True)
    x = torch.randn(33, 96, generator=gq)
    add("static_six", x, "six", static=float(x.abs().max() / 2688.0 * 1.7))
    add("static_mse", x, "mse", static=float(x.abs().max() / 1536.0 * 0.8))
    out["q_cases"] = np.array(cases)

    # --- pack_e2m1 / to_blocked (pack.py:4,39) ---
    codes = torch.randint(0, 16, (5, 64), generator=gq, dtype=torch.uint8)
    out["pack_codes"] = codes.numpy()
    out["pack_packed"] = pack_e2m1(codes).numpy()
    for R, C in [(1, 1), (17, 3), (128, 4), (130, 5), (300, 48)]:
        sf = torch.randint(0, 255, (R, C), generator=gq, dtype=torch.uint8)
        out[f"blk_{R}x{C}_in"] = sf.numpy()
        out[f"blk_{R}x{C}_out"] = to_blocked(sf.view(torch.float8_e4m3fn)).view(torch.uint8).numpy()

    # --- reference GEMM (backends/reference.py:6) ---
    a = torch.randn(64, 256, generator=gq)
    b = torch.randn(48, 256, generator=gq)
    a[:2] *= 30.0
    aq = quantize_to_nvfp4(a, 16)
    bq = quantize_to_nvfp4(b, 16, block_select="mse")
    out["gemm_a"] = a.numpy()
    out["gemm_b"] = b.numpy()
    out["gemm_out"] = G.nvfp4_gemm(*aq, *bq, out_dtype=torch.float32, backend="reference").numpy()

    # --- emulated attention (attention.py:53) ---
    for name, (B, H, S, D) in {"s20d64": (1, 2, 20, 64), "s33d80": (2, 1, 33, 80)}.items():
        q = torch.randn(B, H, S, D, generator=gq)
        k = torch.randn(B, H, S, D, generator=gq)
        v = torch.randn(B, H, S, D, generator=gq)
        k[..., :2, :] *= 12.0
        v[..., :2, :] *= 10.0
        out[f"att_{name}_q"], out[f"att_{name}_k"], out[f"att_{name}_v"] = q.numpy(), k.numpy(), v.numpy()
        for qk, pv in (("nvfp4", "nvfp4"), ("fp8", "fp8"), ("bf16", "bf16")):
            out[f"att_{name}_{qk}_{pv}"] = quant_sdpa(q, k, v, qk=qk, pv=pv).numpy()
    xr = torch.randn(6, 40, generator=gq) * 5
    out["fp8_in"], out["fp8_out"] = xr.numpy(), fp8_e4m3_quant_dequant(xr).numpy()

    # --- ATen's 16-wide mean order (the FoS MSE reduction) ---
    e = torch.rand(512, 16, generator=gq) * torch.exp2(torch.randint(-20, 4, (512, 1), generator=gq).float())
    out["mean_in"], out["mean_out"] = e.numpy(), e.mean(dim=-1).numpy()

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes, {len(out)} arrays, torch {torch.__version__})")


if __name__ == "__main__":
    main()
