"""dfc_zero_fused_step_ef: the ZeRO-1 fused step with the next bucket's
gradient compression in the same grid, on one GPU.

Two ranks are laid out in this GPU's own memory (every buffer local, every
access in bounds, nothing waits), as one launch sees them: rank 0 steps its
segments, reading both ranks' compressed gradients and storing into both
parameter copies, while the same grid compresses another gradient range.
The results must equal, bit for bit, those of dfc_zero_fused_step followed
by dfc_compress_ef on the same inputs; the step is also checked against the
oracle given g = comp_0 + comp_1 (FP32, rank order) and the compression
against the oracle's compression.  Cases: one CTA per tile and a capped
grid whose CTAs walk many tiles; more compression tiles than step tiles and
fewer; ragged and misaligned segments (the per-element path); a set error
flag (the step touches nothing, the compression still runs); no segments
at all; the launch as a barrier's programmatic dependent, behind a barrier
that passes and one that gives up (a signal array nothing writes, 2 ms).
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _ptrs(*ts):
    return (ctypes.c_uint64 * len(ts))(*[t.data_ptr() for t in ts])


def _case(cuda, seed, step_sizes, n_comp):
    """Buffers of one case, the same for the same seed: the step over
    segments of the given sizes (packed into one flat range with gaps), the
    compression over n_comp elements whose (comp, resid) state comes from an
    earlier compression."""
    rng = np.random.default_rng(seed)
    offsets, off = [], 0
    for k, n in enumerate(step_sizes):
        off += 4 * k + (k % 3)          # gaps, some offsets not a multiple of 4
        offsets.append(off)
        off += n
    total = off + 64
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    comps = [dev((rng.standard_normal(total) * 1e-3).astype(np.float32)).to(torch.bfloat16)
             .view(torch.int16) for _ in range(2)]
    p0 = dev((rng.standard_normal(total) * 0.02).astype(np.float32))
    m, v = [], []
    for n in step_sizes:
        mf = (rng.standard_normal(n) * 1e-3).astype(np.float32)
        vf = (rng.random(n) * 1e-6).astype(np.float32)
        m.append(dev(O.pack_first(mf).view(np.int32)))
        v.append(dev(O.pack_second(vf.view(np.uint32)).view(np.int32)))
    hc = np.zeros(n_comp, np.uint16)
    hq = np.zeros(n_comp, np.uint16)
    O.compress_ef((rng.standard_t(3, n_comp) * 1e-3).astype(np.float32), hc, hq)
    cg = dev((rng.standard_t(3, n_comp) * 1e-3).astype(np.float32))
    cc = dev(hc.view(np.int16))
    cq = dev(hq.view(np.int16))
    return offsets, comps, p0, m, v, cg, cc, cq


def _segs(offsets, sizes, m, v):
    from t3st_b200 import _lib

    segs = np.zeros(len(sizes), dtype=_lib.PEERSEG_DTYPE)
    for k, (o, n) in enumerate(zip(offsets, sizes)):
        segs[k] = (o, n, m[k].data_ptr(), v[k].data_ptr(), k % 2, 0)
    return segs


def _hypers():
    from t3st_b200 import kernels
    from t3st_b200.torch_fiber import hyper_row

    return kernels.hypers([hyper_row(1e-3, (0.9, 0.999), 1e-8, 0.01, 3, grad_scale=0.5),
                           hyper_row(5e-4, (0.8, 0.99), 1e-6, 0.0, 7, grad_scale=0.5)])


def _run(cuda, step_sizes, n_comp, ctas, fused, error=False, seed=1, flags=0, barrier=None):
    """barrier: None, or "pass" / "give up": a dfc_peer_barrier of rank 0 of
    two on the same stream first, whose other rank has already arrived /
    never arrives (2 ms limit)."""
    from t3st_b200 import _lib

    lib = _lib.lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    offsets, comps, p0, m, v, cg, cc, cq = _case(cuda, seed, step_sizes, n_comp)
    params = [p0.clone(), p0.clone()]
    segs = _segs(offsets, step_sizes, m, v)
    hyp = _hypers()
    flag = torch.full((1,), 2 if error else 0, dtype=torch.int32, device=cuda)
    if barrier is not None:
        mine = torch.zeros(2, dtype=torch.int32, device=cuda)
        other = torch.zeros(2, dtype=torch.int32, device=cuda)
        if barrier == "pass":
            mine[1] = 1  # rank 1's epoch 1 is already in rank 0's array
        torch.cuda.synchronize()
        _lib.check("dfc_peer_barrier", lib.dfc_peer_barrier(
            _ptrs(mine, other), 2, 0, 1, flag.data_ptr(), 2_000_000, stream))
    if fused:
        nxt = np.zeros(1, dtype=_lib.COMPRESSRANGE_DTYPE)
        nxt[0] = (cg.data_ptr(), cc.data_ptr(), cq.data_ptr(), n_comp)
        _lib.check("dfc_zero_fused_step_ef", lib.dfc_zero_fused_step_ef(
            _ptrs(*comps), _ptrs(*params), None, None, 2, 0,
            _lib.ptr(segs) if len(segs) else None, len(segs), _lib.ptr(hyp), 2,
            _lib.MODE_PACKED, None, flag.data_ptr(), _lib.ptr(nxt), flags, ctas, stream))
    else:
        if not error:
            _lib.check("dfc_zero_fused_step", lib.dfc_zero_fused_step(
                _ptrs(*comps), _ptrs(*params), None, None, 2, 0,
                _lib.ptr(segs) if len(segs) else None, len(segs), _lib.ptr(hyp), 2,
                _lib.MODE_PACKED, None, flag.data_ptr(), ctas, stream))
        _lib.check("dfc_compress_ef", lib.dfc_compress_ef(
            cg.data_ptr(), cc.data_ptr(), cq.data_ptr(), n_comp, 0, stream))
    torch.cuda.synchronize()
    out = {"p0": params[0], "p1": params[1], "cc": cc, "cq": cq}
    for k in range(len(step_sizes)):
        out[f"m{k}"], out[f"v{k}"] = m[k], v[k]
    return {k: t.cpu().numpy().copy() for k, t in out.items()}, p0.cpu().numpy(), comps


CASES = [
    # (segment sizes, compression elements, CTAs per SM)
    ([6144 + 5, 2048, 37, 4096 * 3 + 1], 2048 * 11 + 12, 0),   # more compression tiles
    ([300 * 2048, 77], 2048 * 3 + 4, 0),                       # more step tiles
    ([300 * 2048, 5], 500 * 2048, 1),                          # capped: CTAs walk tiles
    ([], 2048 * 7 + 8, 0),                                     # compression only
]


@pytest.mark.parametrize("sizes,n_comp,ctas", CASES)
def test_fused_compression_equals_the_two_calls(cuda, sizes, n_comp, ctas):
    got, p0, comps = _run(cuda, sizes, n_comp, ctas, fused=True)
    want, _, _ = _run(cuda, sizes, n_comp, ctas, fused=False)
    for key in want:
        np.testing.assert_array_equal(got[key].view(np.uint32 if got[key].itemsize == 4
                                                    else np.uint16),
                                      want[key].view(np.uint32 if want[key].itemsize == 4
                                                     else np.uint16), err_msg=key)
    # the step against the oracle, for the first segment
    if sizes:
        offsets = _case(cuda, 1, sizes, n_comp)[0]
        o, n = offsets[0], sizes[0]
        c = [x[o:o + n].view(torch.bfloat16).float().cpu().numpy() for x in comps]
        gsum = (c[0] + c[1]).astype(np.float32)
        hy = O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.01, 3, grad_scale=0.5)
        p = p0[o:o + n].copy()
        _, _, _, m, v, _, _, _ = _case(cuda, 1, sizes, n_comp)
        sm = m[0].cpu().numpy().view(np.uint32).copy()
        sv = v[0].cpu().numpy().view(np.uint32).copy()
        O.step(O.MODE_PACKED, hy, p, gsum, sm, sv)
        np.testing.assert_array_equal(got["p0"][o:o + n].view(np.uint32), p.view(np.uint32))
        np.testing.assert_array_equal(got["p1"][o:o + n].view(np.uint32), p.view(np.uint32))
        np.testing.assert_array_equal(got["m0"].view(np.uint32), sm)
        np.testing.assert_array_equal(got["v0"].view(np.uint32), sv)
    # the compression against the oracle's
    _, _, _, _, _, cg, cc, cq = _case(cuda, 1, sizes, n_comp)
    oc = cc.cpu().numpy().view(np.uint16).copy()
    oq = cq.cpu().numpy().view(np.uint16).copy()
    O.compress_ef(cg.cpu().numpy(), oc, oq)
    np.testing.assert_array_equal(got["cc"].view(np.uint16), oc)
    np.testing.assert_array_equal(got["cq"].view(np.uint16), oq)


def test_error_flag_skips_the_step_but_not_the_compression(cuda):
    sizes, n_comp = [6144 + 5, 2048], 2048 * 5 + 8
    got, p0, _ = _run(cuda, sizes, n_comp, 0, fused=True, error=True)
    want, _, _ = _run(cuda, sizes, n_comp, 0, fused=False, error=True)  # compression only
    np.testing.assert_array_equal(got["p0"].view(np.uint32), p0.view(np.uint32))
    np.testing.assert_array_equal(got["p1"].view(np.uint32), p0.view(np.uint32))
    _, _, _, m, v, _, _, _ = _case(cuda, 1, sizes, n_comp)
    for k in range(len(sizes)):
        np.testing.assert_array_equal(got[f"m{k}"], m[k].cpu().numpy())
        np.testing.assert_array_equal(got[f"v{k}"], v[k].cpu().numpy())
    np.testing.assert_array_equal(got["cc"], want["cc"])
    np.testing.assert_array_equal(got["cq"], want["cq"])


@pytest.mark.parametrize("sizes,n_comp,ctas", [CASES[0], CASES[2]])
def test_launch_after_a_barrier_that_passes(cuda, sizes, n_comp, ctas):
    """DFC_FUSED_AFTER_BARRIER behind a barrier whose other rank has arrived:
    the grid starts as the barrier's programmatic dependent (compression
    tiles at once, step tiles after the barrier); results equal the two
    separate calls bit for bit."""
    from t3st_b200 import _lib

    got, _, _ = _run(cuda, sizes, n_comp, ctas, fused=True, flags=_lib.FUSED_AFTER_BARRIER,
                     barrier="pass")
    want, _, _ = _run(cuda, sizes, n_comp, ctas, fused=False)
    for key in want:
        np.testing.assert_array_equal(got[key], want[key], err_msg=key)


def test_launch_after_a_barrier_that_gives_up(cuda):
    """The same behind a barrier that gives up after 2 ms: the step tiles wait
    for the barrier, see its flag and touch nothing; the compression is
    done."""
    from t3st_b200 import _lib

    sizes, n_comp = [6144 + 5, 2048], 2048 * 5 + 8
    got, p0, _ = _run(cuda, sizes, n_comp, 0, fused=True, flags=_lib.FUSED_AFTER_BARRIER,
                      barrier="give up")
    want, _, _ = _run(cuda, sizes, n_comp, 0, fused=False, error=True)  # compression only
    np.testing.assert_array_equal(got["p0"].view(np.uint32), p0.view(np.uint32))
    np.testing.assert_array_equal(got["p1"].view(np.uint32), p0.view(np.uint32))
    _, _, _, m, v, _, _, _ = _case(cuda, 1, sizes, n_comp)
    for k in range(len(sizes)):
        np.testing.assert_array_equal(got[f"m{k}"], m[k].cpu().numpy())
        np.testing.assert_array_equal(got[f"v{k}"], v[k].cpu().numpy())
    np.testing.assert_array_equal(got["cc"], want["cc"])
    np.testing.assert_array_equal(got["cq"], want["cq"])
