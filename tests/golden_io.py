"""Loading the golden vectors (made from the reference by make_golden.py) and
replaying them through the oracle.  Test infrastructure only."""

from __future__ import annotations

import os

import numpy as np

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CASES = ("fiber_mt", "plain_mt", "ragged_stress", "c1_small")
LOWP_CASES = ("bf16_params", "f16_params")


def param_dtype(d) -> str:
    return str(d["dtype"]) if "dtype" in d else "f32"


def load(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as d:
        return {k: d[k] for k in d.files}


def group_of(d) -> dict:
    return dict(lr=float(d["lr"]), betas=tuple(float(b) for b in d["betas"]),
                eps=float(d["eps"]), weight_decay=float(d["weight_decay"]))


def offsets(d) -> np.ndarray:
    return np.concatenate([[0], np.cumsum(d["sizes"])]).astype(np.int64)


def initial_state(d, packed: bool):
    """(p, m words, v words) before step 1, in the requested moment format."""
    total = int(d["sizes"].sum())
    p = d["p0"].copy()
    if "m0" in d:
        if packed:
            return p, d["m0_words"].copy(), d["v0_words"].copy()
        return p, d["m0"].copy(), d["v0"].copy()
    m = np.zeros(total, np.uint32)
    v = np.zeros(total, np.uint32)
    if "payload" in d:
        v |= d["payload"].astype(np.uint32) << 31
    return p, m, v


def oracle_replay(d, mode: int):
    """Run the oracle over a golden case; returns (p, m, v, steps)."""
    packed = mode == O.MODE_PACKED
    p, m, v = initial_state(d, packed)
    off = offsets(d)
    n = len(d["sizes"])
    ts = [dict(p=p[off[i]:off[i + 1]], m=m[off[i]:off[i + 1]], v=v[off[i]:off[i + 1]])
          for i in range(n)]
    steps = [0] * n
    grads = d["grads"]
    for s in range(grads.shape[0]):
        gl = [None if d["none_mask"][s, i] else grads[s, off[i]:off[i + 1]] for i in range(n)]
        O.multi_tensor_step(mode, ts, gl, group_of(d), steps, param_dtype=param_dtype(d))
    return p, m, v, np.array(steps, np.int64)


def lowp_to_f32(bits: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return (bits.astype(np.uint32) << 16).view(np.float32)
    return bits.view(np.float16).astype(np.float32)


def lowp_ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in ulps of the 16-bit type, on the monotone integer line."""
    ai = a.view(np.int16).astype(np.int64)
    bi = b.view(np.int16).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFF), bi)
    return np.abs(ai - bi)


def expected_words(d, packed: bool):
    """Reference final (m, v) words, packed with the spec's encoder when asked."""
    if packed:
        return O.pack_first(d["m"].view(np.float32)), O.pack_second(d["v"])
    return d["m"], d["v"]


def update_bound(d) -> np.ndarray:
    """Per element, the sum over steps of one ulp of that step's update
    (-lr/bc1 * m / den), from the oracle.  The stock reference's square root
    is within one ulp, so its p may differ from an IEEE-rounded p by about
    this much in total."""
    p, m, v = initial_state(d, False)
    off = offsets(d)
    n = len(d["sizes"])
    bound = np.zeros(p.size, np.float64)
    steps = [0] * n
    group = group_of(d)
    mode = O.MODE_SIGNFIBER if bool(d["fiber"]) else O.MODE_PLAIN
    for s in range(d["grads"].shape[0]):
        for i in range(n):
            if d["none_mask"][s, i]:
                continue
            sl = slice(off[i], off[i + 1])
            steps[i] += 1
            h = O.reference_hyper(group["lr"], group["betas"], group["eps"], group["weight_decay"],
                                  steps[i])
            p_before = p[sl].copy()
            O.step(mode, h, p[sl], np.ascontiguousarray(d["grads"][s, sl]), m[sl], v[sl])
            upd = np.abs(p[sl].astype(np.float64) - p_before.astype(np.float64) * h.decay)
            bound[sl] += np.spacing(np.maximum(upd, 1e-45).astype(np.float32)).astype(np.float64)
    return bound


def p_matches_stock(p, d) -> tuple[bool, float]:
    """p against the stock reference: within 2 ulp of p, plus the
    accumulated one-ulp-of-update slack of the reference's square root."""
    ref = d["p"]
    diff = np.abs(p.astype(np.float64) - ref.astype(np.float64))
    tol = 2.0 * np.spacing(np.abs(ref)).astype(np.float64) + 2.0 * update_bound(d)
    worst = float(np.max(diff / tol)) if diff.size else 0.0
    return bool(np.all(diff <= tol)), worst
