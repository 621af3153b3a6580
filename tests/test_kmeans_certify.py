"""The rounding-interval test of the tensor-core k-means assignment, on CPU.

kmeans_tc.cu certifies bf16(acc) = bf16(a) for the exact sequential dot acc
when the tensor-core dot a lies more than E inside the bf16 rounding interval
of bf16(a) (`cand_sim`).  This restates that predicate with numpy float32
arithmetic and checks, on random and adversarial values (powers of two, both
interval edges, tiny and negative values), that whenever it says "safe" every
float32 within E of a rounds to the same bf16.
"""

import numpy as np


def _bf16(x):
    """Round float32 to bf16 (nearest even), returned as float32."""
    b = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def _safe(a, E):
    """The device predicate (cand_sim) for float32 a and error bound E."""
    f = np.float32
    bf = _bf16(a)
    ab = np.abs(bf).view(np.uint32)
    ok_range = (ab >= (8 << 23)) & (ab < 0x7F800000)
    ulp = ((ab & 0x7F800000) - (7 << 23)).astype(np.uint32).view(np.float32)
    dn = np.where((ab & 0x007F0000) != 0, ulp, f(0.5) * ulp).astype(np.float32)
    d = (np.abs(a).astype(np.float32) - np.abs(bf)).astype(np.float32)
    lhs1 = (d + E).astype(np.float32)
    lhs2 = (E - d).astype(np.float32)
    return ok_range & (lhs1 < f(0.5) * ulp) & (lhs2 < f(0.5) * dn)


def _check(a, E):
    a = np.asarray(a, np.float32)
    E = np.asarray(E, np.float32)
    s = _safe(a, E)
    if not s.any():
        return 0
    a, E = a[s], E[s]
    # both ends of [a - E, a + E] and points inside; rounding is monotone, so
    # the ends decide, the inside points guard the test itself
    a64, E64 = a.astype(np.float64), E.astype(np.float64)
    for t in (-1.0, -0.999, -0.5, 0.0, 0.5, 0.999, 1.0):
        x = (a64 + t * E64).astype(np.float32)
        # the float32 values an exact dot can take lie inside the real
        # interval: step back toward a where rounding left it
        out = np.abs(x.astype(np.float64) - a64) > E64
        x = np.where(out, np.nextafter(x, a), x).astype(np.float32)
        np.testing.assert_array_equal(_bf16(x), _bf16(a))
    return int(s.sum())


def test_certify_random_values():
    rng = np.random.default_rng(0)
    a = (rng.standard_normal(2_000_000) * 200).astype(np.float32)
    E = (np.abs(a) * np.float32(2.0 ** -12) * rng.uniform(0.1, 3.0, a.size)).astype(np.float32)
    assert _check(a, E) > 1_000_000


def test_certify_near_powers_of_two_and_edges():
    rng = np.random.default_rng(1)
    out = 0
    for e in range(-20, 20):
        p = np.float32(2.0 ** e)
        ulp = np.float32(2.0 ** (e - 7))
        # around the power of two (spacing halves below it) and around the
        # midpoints just above and below it
        centres = np.array([p, p + ulp / 2, p - ulp / 4, p + ulp, p - ulp / 2], np.float32)
        offs = rng.uniform(-1.0, 1.0, (centres.size, 4000)).astype(np.float32) * ulp
        a = (centres[:, None] + offs).reshape(-1).astype(np.float32)
        for sign in (1.0, -1.0):
            aa = (a * np.float32(sign)).astype(np.float32)
            E = (rng.uniform(0.0, 0.6, aa.size) * ulp).astype(np.float32)
            out += _check(aa, E)
    assert out > 10_000


def test_certify_refuses_tiny_and_ambiguous():
    f = np.float32
    # below 2^-119 the predicate always recomputes
    assert not _safe(np.array([f(2.0 ** -125)]), np.array([f(0.0)])).any()
    assert not _safe(np.array([f(0.0)]), np.array([f(0.0)])).any()
    # a value on a rounding midpoint is never certified, whatever E
    mid = np.float32(1.0 + 2.0 ** -8)       # halfway between bf16 1.0 and 1.0078125
    assert not _safe(np.array([mid]), np.array([f(0.0)])).any()
    # an error bound as wide as half a bf16 step is never certified
    assert not _safe(np.array([f(1.5)]), np.array([f(2.0 ** -8)])).any()
