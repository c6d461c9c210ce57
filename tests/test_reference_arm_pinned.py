"""The CPU path that bench.py times as the reference (its ``--impl reference``
arm and the ``cpu_baseline`` leg): oracle/torch_port.step_fp32, the
reference's step (remote/torch_fiber.py:83-116) restated op for op as
PyTorch CPU ops.  Replayed over the golden cases made by importing the
reference itself, it must give the stock reference's p, m and v bit for
bit -- including the parameters, where the reference's own (not correctly
rounded) CPU square root decides the last bit.  CPU only."""

import numpy as np
import pytest
import torch

import golden_io as G
from oracle import torch_port


@pytest.mark.parametrize("name", G.CASES)
def test_torch_port_is_the_stock_reference_bit_for_bit(name):
    d = G.load(name)
    p, m, v = G.initial_state(d, packed=False)
    p = torch.from_numpy(p.copy())
    m = torch.from_numpy(m.view(np.float32).copy())
    v = torch.from_numpy(v.view(np.float32).copy())
    off = G.offsets(d)
    n = len(d["sizes"])
    group = G.group_of(d)
    fiber = bool(d["fiber"])
    steps = [0] * n
    for s in range(d["grads"].shape[0]):
        for i in range(n):
            if d["none_mask"][s, i]:  # no gradient: the parameter is skipped (:79-80)
                continue
            steps[i] += 1
            sl = slice(int(off[i]), int(off[i + 1]))
            g = torch.from_numpy(np.ascontiguousarray(d["grads"][s, sl]))
            torch_port.step_fp32(p[sl], g, m[sl], v[sl], group["lr"], group["betas"],
                                 group["eps"], group["weight_decay"], steps[i], fiber=fiber)
    np.testing.assert_array_equal(steps, d["steps"])
    np.testing.assert_array_equal(p.numpy().view(np.uint32), d["p"].view(np.uint32))
    np.testing.assert_array_equal(m.numpy().view(np.uint32), d["m"].view(np.uint32))
    np.testing.assert_array_equal(v.numpy().view(np.uint32), d["v"].view(np.uint32))
