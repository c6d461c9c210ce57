"""Properties of the packed moment word and the compressed-gradient residual
(the oracle's statement of both formats).  CPU only."""

import numpy as np
import pytest

from oracle import oracle as O


def _all_finite_patterns(rng, n):
    bits = rng.integers(0, 1 << 31, n, dtype=np.uint32)
    bits = bits[bits <= 0x7F800000]
    return bits


def test_roundtrip_exact_for_every_non_nan_value():
    rng = np.random.default_rng(0)
    mags = np.concatenate([
        _all_finite_patterns(rng, 1 << 20),
        np.arange(0, 1 << 17, dtype=np.uint32),                    # zero, denormals
        np.arange(0x7F7E0000, 0x7F800001, dtype=np.uint32),        # top of the range, +Inf
        (np.arange(0, 1 << 16, dtype=np.uint32) | 0x3F800000),     # every low half at 1.0
        (np.arange(0, 1 << 16, dtype=np.uint32) | 0x3F7F0000),     # every low half below 1.0
    ])
    for sign in (0, 0x80000000):
        x = (mags | np.uint32(sign)).view(np.float32)
        w = O.pack_first(x)
        back = O.unpack_first(w)
        np.testing.assert_array_equal(back.view(np.uint32), x.view(np.uint32))


def test_high_half_is_round_to_nearest_ties_away():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(1 << 18) * 1e-3).astype(np.float32)
    w = O.pack_first(x)
    hi = (w >> 16).astype(np.uint32) << 16
    approx = hi.view(np.float32).astype(np.float64)
    err = np.abs(approx - x.astype(np.float64))
    ulp_bf16 = np.spacing(np.abs(x)).astype(np.float64) * 65536
    assert np.all(err <= ulp_bf16 / 2)
    # exact ties round away from zero
    tie = np.array([0x3F808000, 0x3F818000, 0xBF808000], np.uint32).view(np.float32)
    np.testing.assert_array_equal(O.pack_first(tie) >> 16, [0x3F81, 0x3F82, 0xBF81])


def test_every_residual_pattern_decodes_within_half_a_bf16_ulp():
    lo = np.arange(0, 1 << 16, dtype=np.uint32)
    for hi in (0x3F80, 0x0081, 0x7F7F, 0x1234):
        w = (np.uint32(hi) << 16) | lo
        x = O.unpack_first(w).astype(np.float64)
        h = np.float64(np.array([hi << 16], np.uint32).view(np.float32)[0])
        ulp = np.spacing(np.float32(h)) * 65536.0
        assert np.all(np.abs(x - h) <= ulp / 2 + 1e-45)


def test_decode_clamps_out_of_range_residuals():
    w = np.array([0x0000FFFF, 0x7F800001, 0x7F807FFF, 0x80008000], np.uint32)
    x = O.unpack_first(w).view(np.uint32)
    np.testing.assert_array_equal(x, [0x00000000, 0x7F800000, 0x7F800000, 0x80000000])


def test_nan_stays_nan():
    x = np.array([0x7FC00000, 0x7F800001, 0xFFFFFFFF], np.uint32).view(np.float32)
    back = O.unpack_first(O.pack_first(x))
    assert np.all(np.isnan(back))


def test_second_moment_payload_bit_kept():
    rng = np.random.default_rng(2)
    v = np.abs(rng.standard_normal(4096).astype(np.float32)) * 1e-6
    payload = rng.integers(0, 2, 4096, dtype=np.uint32)
    phys = v.view(np.uint32) | (payload << 31)
    w = O.pack_second(phys)
    np.testing.assert_array_equal(w >> 31, payload)
    np.testing.assert_array_equal(O.unpack_second(w), phys)


def test_compress_error_feedback_is_exact():
    """sum over steps of the compressed values == sum of gradients minus the
    final residual, up to the FP32 rounding of each s = g + e."""
    rng = np.random.default_rng(3)
    n = 1 << 14
    c = np.zeros(n, np.uint16)
    q = np.zeros(n, np.uint16)
    total_c = np.zeros(n, np.float64)
    total_g = np.zeros(n, np.float64)
    steps = 20
    for _ in range(steps):
        g = (rng.standard_normal(n) * 1e-3).astype(np.float32)
        e_prev = O.ef_residual(c, q)
        s = (g + e_prev).astype(np.float32)
        O.compress_ef(g, c, q)
        cv = (c.astype(np.uint32) << 16).view(np.float32)
        # s == c + e exactly
        np.testing.assert_array_equal((cv.astype(np.float64) + O.ef_residual(c, q)), s.astype(np.float64))
        total_c += cv
        total_g += g
    drift = np.abs(total_g - total_c - O.ef_residual(c, q))
    assert drift.max() <= steps * 1e-3 * 2.0 ** -23 * 8


def test_compress_nonfinite_resets_residual():
    g = np.array([np.inf, np.nan, 1.0], np.float32)
    c = np.zeros(3, np.uint16)
    q = np.zeros(3, np.uint16)
    O.compress_ef(g, c, q)
    e = O.ef_residual(c, q)
    np.testing.assert_array_equal(e, [0.0, 0.0, 0.0])


def test_grad_stats():
    rng = np.random.default_rng(4)
    g = rng.standard_normal(1000).astype(np.float32)
    g[7] = np.inf
    g[9] = np.nan
    s, a, bad = O.grad_stats(g)
    assert bad == 2 and a == np.inf and np.isnan(s)
    g2 = g.copy()
    g2[[7, 9]] = 0
    s2, a2, bad2 = O.grad_stats(g2)
    assert bad2 == 0 and a2 == np.abs(g2).max()
    assert s2 == pytest.approx(float(np.sum(g2.astype(np.float64) ** 2)), rel=1e-12)
