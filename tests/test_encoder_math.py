"""CPU proofs for the arithmetic shortcuts of the CUDA quantizer (vf4_common.cuh).

1. ``div6_rn``: RN(a / 6) by one Markstein correction step equals IEEE division for every fp32
   significand in [1, 2) (exhaustive; every other normal a is a power-of-two scaling of these).
2. ``encode16_bracket``: codes taken from the brackets a = RN(x * lo), b = RN(x * hi),
   lo/hi = RN(inv * (1 -+ 2^-20)), are accepted only when the nearest-even E2M1 codes of a and
   b agree; then they equal the reference's round-half-down code of RN(x / dec).  Checked here
   with the reciprocal perturbed by up to 4 ulp (the hardware approximation is within 1 ulp),
   on quotients placed on and around every rounding boundary.
"""
from fractions import Fraction

import numpy as np

from conftest import oracle

F32 = np.float32


def _rn32(x64: np.ndarray) -> np.ndarray:
    return x64.astype(np.float32)


def test_div6_markstein_exhaustive_significands():
    a = (np.arange(1 << 23, 1 << 24, dtype=np.int64).astype(np.float64) / float(1 << 23)).astype(np.float32)
    y = F32(1.0) / F32(6.0)
    assert y.view(np.uint32) == 0x3E2AAAAB
    q0 = _rn32(a.astype(np.float64) * np.float64(y))                 # exact product, one rounding
    r64 = a.astype(np.float64) - 6.0 * q0.astype(np.float64)           # exact in float64
    r = _rn32(r64)
    assert np.array_equal(r.astype(np.float64), r64)                   # the FMA residual is exact
    s64 = q0.astype(np.float64) + r.astype(np.float64) * np.float64(y)  # r*y exact; sum rounded once
    q1 = _rn32(s64)
    want = a / F32(6.0)
    # float64 -> float32 double rounding can only matter next to a float32 midpoint: redo those exactly
    lo = np.minimum(q1, np.nextafter(q1, F32(-np.inf)))
    hi = np.nextafter(q1, F32(np.inf))
    near = (np.abs(s64 - (q1.astype(np.float64) + lo.astype(np.float64)) / 2) < 4 * np.spacing(s64)) | \
           (np.abs(s64 - (q1.astype(np.float64) + hi.astype(np.float64)) / 2) < 4 * np.spacing(s64))
    for i in np.flatnonzero(near):
        exact = Fraction(float(q0[i])) + Fraction(float(r[i])) * Fraction(float(y))
        cands = [F32(q1[i]), np.nextafter(q1[i], F32(-np.inf)), np.nextafter(q1[i], F32(np.inf))]
        q1[i] = min(cands, key=lambda c: (abs(Fraction(float(c)) - exact), int(c.view(np.uint32)) & 1))
    bad = np.flatnonzero(q1 != want)
    assert bad.size == 0, (bad.size, a[bad[:4]])


_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _cvt_rne_e2m1(v: np.ndarray) -> np.ndarray:
    """Nearest-even E2M1 code with saturation (the hardware converter), finite inputs."""
    m = np.minimum(np.abs(v.astype(np.float64)), 6.0)
    d = np.abs(m[..., None] - _GRID)
    best = d.min(-1, keepdims=True)
    cand = np.where(d == best, np.arange(8), 99)
    even = np.where(cand % 2 == 0, cand, 99).min(-1)
    idx = np.where((d == best).sum(-1) > 1, even, cand.min(-1))
    return (np.signbit(v).astype(np.int64) << 3) | idx


def _bracket_codes(x: np.ndarray, dec: np.float32, inv_err_ulp: int):
    inv = F32(1.0) / dec
    for _ in range(abs(inv_err_ulp)):
        inv = np.nextafter(inv, F32(np.inf) if inv_err_ulp > 0 else F32(-np.inf))
    lo = F32(inv * F32(1.0 - 2.0 ** -20))
    hi = F32(inv * F32(1.0 + 2.0 ** -20))
    a = (x.astype(np.float64) * np.float64(lo)).astype(np.float32) + F32(0.0)   # +0: -0 -> +0
    b = (x.astype(np.float64) * np.float64(hi)).astype(np.float32) + F32(0.0)
    ca, cb = _cvt_rne_e2m1(a), _cvt_rne_e2m1(b)
    return ca, ca == cb


def test_bracket_codes_equal_reference_when_accepted():
    rng = np.random.default_rng(7)
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], np.float32)
    n_rejected = n_random = n_random_ok = 0
    for trial in range(400):
        dec = F32(np.exp2(rng.uniform(-20, 17)) * rng.uniform(1, 2))
        m = rng.choice(mids, 256) * rng.choice([-1, 1], 256)
        q = (m.astype(np.float64) * dec).astype(np.float32)
        steps = rng.integers(-6, 7, 256)
        x = q.copy()
        for i, s in enumerate(steps):
            for _ in range(abs(s)):
                x[i] = np.nextafter(x[i], F32(np.sign(s) * np.inf))
        x = np.concatenate([x, (rng.standard_normal(256) * 3 * dec).astype(np.float32), np.array([0.0, -0.0], np.float32)])
        ref = oracle.round_to_e2m1_code(x / dec)
        for err in (-4, -1, 0, 1, 4):
            codes, ok = _bracket_codes(x, dec, err)
            assert np.array_equal(codes[ok], ref[ok]), (trial, err)
            n_rejected += int((~ok).sum())
            n_random += 256
            n_random_ok += int(ok[256:512].sum())
    # near-boundary quotients go to the exact path; random data almost never does
    assert n_rejected > 0 and n_random_ok > 0.999 * n_random
