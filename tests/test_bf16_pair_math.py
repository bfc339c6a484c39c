"""CPU proof behind the bf16 pair arithmetic of the kernels (``add_bf16x2`` / ``mul_bf16x2`` in
vf4_common.cuh, used by the GEMM bf16 epilogues, the residual LayerNorm cast and the fc1 epilogue).

The kernels replace torch's bf16 ops -- an fp32 operation, then one rounding to bf16 -- by
``add.rn.bf16x2`` / ``mul.rn.bf16x2``, which round the exact result once.  The two agree when the
fp32 step is exact or cannot move the value across a bf16 rounding midpoint:
  * a product of two bf16 values has at most 16 significant bits, so its fp32 value is exact
    (outside fp32's subnormal range);
  * a sum of two bf16 values is exact in fp32 unless their exponents differ by more than 16, and then
    it lies within 2^-16 relative of the larger operand, far from any bf16 midpoint.
Checked here on random bf16 pairs over a wide exponent range, on exponent gaps around 16, and on
values next to bf16 midpoints, against the exactly rounded result (float64 holds the exact sums and
products of these operands).
"""
import numpy as np


def _bf16_bits_to_f64(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def _rne_bf16_from_f32(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bf16 bits, nearest-even (finite inputs)."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _rne_bf16_from_f64(x: np.ndarray) -> np.ndarray:
    """Round exact float64 values to bf16 bits, nearest-even, in one step (normal range)."""
    m, e = np.frexp(x)                         # x = m * 2^e, 0.5 <= |m| < 1
    q = np.round(m * 256.0)                    # 8 significant bits; np.round is half-to-even
    return _rne_bf16_from_f32((q * np.exp2(e - 8)).astype(np.float32))   # exact in fp32 (8 bits)


def _random_bf16(rng, n, emin=-60, emax=60):
    sign = rng.integers(0, 2, n).astype(np.uint16) << 15
    exp = (rng.integers(emin, emax, n) + 127).astype(np.uint16) << 7
    man = rng.integers(0, 128, n).astype(np.uint16)
    return sign | exp | man


def test_bf16_pair_mul_equals_fp32_then_round():
    rng = np.random.default_rng(0)
    a, b = _random_bf16(rng, 2_000_000), _random_bf16(rng, 2_000_000)
    fa, fb = _bf16_bits_to_f64(a), _bf16_bits_to_f64(b)
    exact = fa * fb                                            # exact: 16 significant bits
    torch_way = _rne_bf16_from_f32((fa.astype(np.float32) * fb.astype(np.float32)))
    single = _rne_bf16_from_f64(exact)
    assert np.array_equal(torch_way, single)


def test_bf16_pair_add_equals_fp32_then_round():
    rng = np.random.default_rng(1)
    n = 2_000_000
    a = _random_bf16(rng, n, -20, 20)
    # b: the same exponent range, plus exponent gaps of 14..20 below a (where the fp32 sum starts
    # to round) with both signs
    b = _random_bf16(rng, n, -20, 20)
    gap = rng.integers(14, 21, n).astype(np.int64)
    ea = ((a >> 7) & 0xFF).astype(np.int64)
    eb = np.clip(ea - gap, 1, 254).astype(np.uint16)
    b_gap = (rng.integers(0, 2, n).astype(np.uint16) << 15) | (eb << 7) | rng.integers(0, 128, n).astype(np.uint16)
    for bb in (b, b_gap):
        fa, fb = _bf16_bits_to_f64(a), _bf16_bits_to_f64(bb)
        exact = fa + fb                                        # exact in float64 (gap <= 20 bits)
        torch_way = _rne_bf16_from_f32(fa.astype(np.float32) + fb.astype(np.float32))
        nz = exact != 0
        single = _rne_bf16_from_f64(exact[nz])
        assert np.array_equal(torch_way[nz], single)


def test_bf16_rounding_helpers_agree_on_midpoints():
    """The single-rounding reference itself: values exactly on and next to bf16 midpoints."""
    rng = np.random.default_rng(2)
    base = _bf16_bits_to_f64(_random_bf16(rng, 10_000, -10, 10))
    ulp = np.abs(base) * 2.0 ** -7
    for off in (0.5, 0.5 - 2.0 ** -12, 0.5 + 2.0 ** -12):
        x = base + off * ulp * np.sign(base)
        assert np.array_equal(_rne_bf16_from_f64(x), _rne_bf16_from_f32(x.astype(np.float32)))
