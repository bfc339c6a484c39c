"""Generate the end-to-end golden logits that pin whole-model parity to the reference.

Run once in a container that holds the reference source tree (Dev-Jahn/vit-nvfp4):

    python tests/golden/make_golden_vit.py --reference-src <path-to>/vit-nvfp4/src

a ViT-S/16 (12 blocks, width 384, 6 heads, GELU MLP 1536, 224x224 input,
197 tokens, 1000 classes) with N(0, 0.02) weights, zero biases and LayerNorm (1, 0) -- built by
``vitfp4.vit.build_vit(seed=0, **VIT_S16)``, plain torch modules -- converted by the REFERENCE's
``quantize_vit(model, skip_first=0, skip_last=0, w_block_select="six")`` (every block Linear becomes
its ``QuantLinear`` with RTN weights and dynamic NVFP4 activations) and run by the reference's CPU
backend (``backends/reference.py``: dequantize, fp32 matmul) on a batch of 8 N(0, 1) images drawn
from ``torch.Generator().manual_seed(0)``.  Two precisions:

  c1_f32   the configuration as stated (fp32 model and images)
  c1_bf16  the same model and images in bf16 (the reference rounds each QuantLinear output to bf16
           and adds the bf16 bias, torch's bf16 LayerNorm / GELU / SDPA in between)

Besides the logits of each, the fixture records:
  *_exact_logits   the same model before conversion (bf16/fp32 weights and activations), the
                   yardstick for "same accuracy as the reference"
  *_pert_logits    the converted reference model on the images with every element moved one ulp up
                   in its dtype (torch.nextafter): how far the reference's own logits move under a
                   last-bit change of its input.  W4A4 rounding
                   is discontinuous and this random-init model has no LayerScale, so such a change
                   flips codes that compound over the 12 blocks; end-to-end comparisons are bounded
                   by this, and block-level comparisons on identical inputs carry the tight bar
  *_blk{i}_out     converted block i of the reference on one synthetic block input
                   (``block_input(dtype)``: N(0, 1) of shape (1, 197, 384), seed 1), for i in BLOCKS

The GPU box never runs this script; the tests rebuild the same model and images from the same
seeds (torch's CPU generator) and read only the committed ``golden_vit.npz``.

Reference functions exercised (file:line in the reference project):
  ptq.models.quantize_vit ......... src/vit_nvfp4/ptq/models.py:74-79
  ptq.qlinear.QuantLinear ......... src/vit_nvfp4/ptq/qlinear.py:7-50
  nvfp4.gemm.nvfp4_linear ......... src/vit_nvfp4/nvfp4/gemm.py:32-38
  backends.reference.gemm ......... src/vit_nvfp4/nvfp4/backends/reference.py:6-10
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "golden_vit.npz")
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "vit-nvfp4_b200"))

BATCH = 8
SEED = 0
BLOCKS = (0, 11)


def config1_model(dtype: torch.dtype):
    """The configuration-1 ViT-S/16 (plain torch modules, CPU) in ``dtype``."""
    from vitfp4 import vit
    return vit.build_vit(seed=SEED, **vit.VIT_S16).to(dtype).eval()


def config1_images(dtype: torch.dtype) -> torch.Tensor:
    g = torch.Generator().manual_seed(SEED)
    return torch.randn(BATCH, 3, 224, 224, generator=g).to(dtype)


def block_input(dtype: torch.dtype) -> torch.Tensor:
    g = torch.Generator().manual_seed(1)
    return torch.randn(1, 197, 384, generator=g).to(dtype)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", default=os.environ.get("VIT_NVFP4_REFERENCE_SRC"),
                    help="the reference's src/ directory (or set VIT_NVFP4_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.reference_src:
        ap.error("pass --reference-src <vit-nvfp4>/src or set VIT_NVFP4_REFERENCE_SRC")
    sys.path.insert(0, args.reference_src)
    from vit_nvfp4.nvfp4 import gemm as G
    from vit_nvfp4.ptq.models import quantize_vit
    G._BACKENDS.pop("torch_scaled_mm_v2", None)   # CPU: the fp32 emulation backend

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out: dict[str, np.ndarray] = {}
    for tag, dtype in (("c1_f32", torch.float32), ("c1_bf16", torch.bfloat16)):
        model = config1_model(dtype)
        images = config1_images(dtype)
        with torch.inference_mode():
            out[f"{tag}_exact_logits"] = model(images).float().numpy()
        n, spec = quantize_vit(model, skip_first=0, skip_last=0, w_block_select="six")
        assert n == 48 and spec.block_container == "blocks", (n, spec)
        with torch.inference_mode():
            logits = model(images).float()
            pert = torch.nextafter(images, torch.full_like(images, float("inf")))
            out[f"{tag}_pert_logits"] = model(pert).float().numpy()
            for i in BLOCKS:
                out[f"{tag}_blk{i}_out"] = model.blocks[i](block_input(dtype)).float().numpy()
        out[f"{tag}_logits"] = logits.numpy()
        top2 = logits.topk(2, dim=-1).values
        print(f"{tag}: {n} QuantLinears, logits |max| {logits.abs().max():.4f}, "
              f"smallest top-1/top-2 gap {(top2[:, 0] - top2[:, 1]).min():.5f}")
    out["meta_torch"] = np.array(torch.__version__)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({os.path.getsize(OUT)} bytes)")


if __name__ == "__main__":
    main()
