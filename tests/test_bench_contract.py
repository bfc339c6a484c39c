"""Host-side pieces of bench.py's JSON contract: algorithmic bytes and the roofline objects (no GPU)."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


def test_gemm_algorithmic_bytes():
    m, n, k = 263168, 1024, 4096
    ops = (m + n) * (k // 2 + k // 16)
    assert bench.gemm_algorithmic_bytes("gemm_bias", m, n, k) == ops + m * n * 2
    assert bench.gemm_algorithmic_bytes("gemm_residual", m, n, k) == ops + 2 * m * n * 2
    assert bench.gemm_algorithmic_bytes("gemm_gelu_nvfp4", m, 4096, 1024) == \
        (m + 4096) * (512 + 64) + m * (2048 + 256)
    # bf16 attention: q, k, v read and the output written once
    assert bench.gemm_algorithmic_bytes("attn_bf16", 16384, 257, 64) == 16384 * 257 * 64 * 2 * 4


@pytest.mark.parametrize("measured", [True, False])
def test_roofline_entry_peaks_and_traffic(measured):
    bf16 = 1645.7 if measured else bench.FALLBACK_PEAKS["bf16_tflops"]
    # fc2 at 2.8 PF: 240 launches of 2 M N K flops in 192 ms
    m, n, k = 263168, 1024, 4096
    flops = 240 * 2.0 * m * n * k
    g = bench.roofline_entry(f"gemm_residual_{m}x{n}x{k}", flops, 192.0, bf16, measured)
    assert g["peak"] == round(4 * bf16, 1) and g["unit"] == "TFLOP/s" and g["bound"] == "tensor"
    assert abs(g["frac"] - g["achieved"] / g["peak"]) < 1e-3
    assert g["traffic"] is not None and g["traffic"] < 2 * g["algorithmic_bytes"]
    assert ("of measured" in g["peak_source"]) == measured and ("of fallback" in g["peak_source"]) != measured
    # the bf16 attention kernel is held to the bf16 peak
    a = bench.roofline_entry("attn_bf16_16384x257x64", 240 * 4.0 * 16384 * 257 ** 2 * 64, 199.0, bf16, measured)
    assert a["peak"] == round(bf16, 1) and 0 < a["frac"] < 1
    assert a["traffic"] is not None and a["algorithmic_bytes"] == 16384 * 257 * 64 * 8
    # kinds without an ncu capture report no traffic
    assert bench.roofline_entry("gemm_bias_4096x768x768", 1e12, 1.0, bf16, measured)["traffic"] is None
