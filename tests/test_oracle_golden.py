"""The oracle against the reference's own outputs (golden vectors made by
importing remote/torch_fiber.py).  CPU only."""

import numpy as np
import pytest

import golden_io as G
from oracle import oracle as O

MODES = {
    "fiber_mt": [O.MODE_SIGNFIBER, O.MODE_PACKED],
    "plain_mt": [O.MODE_PLAIN],
    "ragged_stress": [O.MODE_SIGNFIBER, O.MODE_PACKED],
    "c1_small": [O.MODE_SIGNFIBER, O.MODE_PACKED],
}


@pytest.mark.parametrize("name,mode", [(n, m) for n, ms in MODES.items() for m in ms])
def test_oracle_matches_reference(name, mode):
    d = G.load(name)
    p, m, v, steps = G.oracle_replay(d, mode)
    np.testing.assert_array_equal(steps, d["steps"])
    em, ev = G.expected_words(d, mode == O.MODE_PACKED)
    # moments and payload bits: bit-exact against the reference
    np.testing.assert_array_equal(m, em)
    np.testing.assert_array_equal(v, ev)
    # params: bit-exact against the reference run with a correctly rounded sqrt
    np.testing.assert_array_equal(p.view(np.uint32), d["p_ieee_sqrt"].view(np.uint32))
    # and within the stated tolerance of the stock reference
    ok, worst = G.p_matches_stock(p, d)
    assert ok, worst


def test_stock_reference_sqrt_is_the_only_difference():
    """The stock reference's p differs from the IEEE one only where torch's
    CPU sqrt rounded differently, on a small fraction of elements."""
    d = G.load("c1_small")
    diff = d["p"].view(np.uint32) != d["p_ieee_sqrt"].view(np.uint32)
    assert 0 < diff.mean() < 0.02


def test_payload_survives_in_reference_outputs():
    d = G.load("fiber_mt")
    np.testing.assert_array_equal((d["v"] >> 31).astype(np.uint8), d["payload"])
    d = G.load("ragged_stress")
    np.testing.assert_array_equal(d["v"] >> 31, d["v0_words"] >> 31)


def test_per_tensor_step_counters():
    d = G.load("fiber_mt")
    assert list(d["steps"]) == [6, 6, 5, 6]
    d = G.load("ragged_stress")
    assert d["steps"][0] == 3 and d["steps"][5] == 3 and d["steps"][1] == 4


@pytest.mark.parametrize("name", G.LOWP_CASES)
@pytest.mark.parametrize("mode", [O.MODE_SIGNFIBER, O.MODE_PACKED])
def test_oracle_reduced_precision_params(name, mode):
    """bf16/fp16 parameters (remote/torch_fiber.py:45, 114-116): FP32 moments
    bit-exact, parameters bit-exact against the IEEE-sqrt reference; against
    the stock reference a few elements are one ulp of the 16-bit type off."""
    d = G.load(name)
    p, m, v, steps = G.oracle_replay(d, mode)
    np.testing.assert_array_equal(steps, d["steps"])
    em, ev = G.expected_words(d, mode == O.MODE_PACKED)
    np.testing.assert_array_equal(m, em)
    np.testing.assert_array_equal(v, ev)
    np.testing.assert_array_equal(p, d["p_ieee_sqrt"])
    ulp = G.lowp_ulp_distance(p, d["p"])
    assert ulp.max() <= 1 and (ulp > 0).mean() < 0.02
