"""dfc_grad_stats_noalloc, the statistics entry point for callers that
cannot allocate device memory (a host runtime whose device memory all
belongs to its own pool, a plugin whose host forbids device allocations
during a step).  It keeps its partial records in a device array inside the
library, so the caller passes only the gradients and the output records.

The test calls it through the C ABI twice in a row, on different inputs, and
checks each result against the allocating entry point dfc_grad_stats with the
tolerance the other statistics tests use (sum of squares to 1e-12 relative,
max and non-finite count exact), and against the CPU oracle's statistics of
the same values.  This file is collected last so that a run
stopping at the first failure has already run every other test; it also
passes alone in a fresh process."""

import numpy as np
import pytest
import torch

from t3st_b200 import _lib, kernels

pytestmark = pytest.mark.gpu


def _inputs(cuda, seed):
    rng = np.random.default_rng(seed)
    sizes = [0, 1, 7, 8192, 8193, 100003, 1 << 20]
    grads = []
    for i, n in enumerate(sizes):
        x = (rng.standard_normal(n) * 10.0 ** rng.uniform(-4, 0)).astype(np.float32)
        if i == 4 and seed % 2:
            x[[5, 99]] = [np.inf, np.nan]
        grads.append(torch.from_numpy(x).to(cuda))
    grads.append(grads[5].bfloat16())
    return grads


def _noalloc(grads, cuda):
    refs = kernels.grad_refs(grads)
    out = torch.full((len(grads) * _lib.GRADSTATS_DTYPE.itemsize,), 0xAB, dtype=torch.uint8,
                     device=cuda)
    with torch.cuda.device(cuda):
        rc = _lib.lib().dfc_grad_stats_noalloc(
            _lib.ptr(refs), len(refs), out.data_ptr(), torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _lib.DFC_OK, _lib.strerror(rc)
    return kernels.stats_to_numpy(out)


def _check(got, want):
    np.testing.assert_array_equal(got["nonfinite"], want["nonfinite"])
    np.testing.assert_array_equal(got["amax"], want["amax"])
    for a, b in zip(got["sumsq"], want["sumsq"]):
        if np.isnan(b):
            assert np.isnan(a)
        else:
            assert a == pytest.approx(b, rel=1e-12, abs=0)


def _check_oracle(got, grads):
    """Also against the CPU oracle's statistics of the same values."""
    from oracle import oracle as O

    for rec, g in zip(got, grads):
        s, a, bad = O.grad_stats(g.float().cpu().numpy())
        assert rec["nonfinite"] == bad and rec["amax"] == np.float32(a)
        if np.isnan(s):
            assert np.isnan(rec["sumsq"])
        else:
            assert rec["sumsq"] == pytest.approx(s, rel=1e-12, abs=0)


def test_noalloc_stats_match_the_scratch_entry_point_on_two_calls(cuda):
    for seed in (1, 2):  # two calls in a row on different inputs
        grads = _inputs(cuda, seed)
        want = kernels.stats_to_numpy(kernels.grad_stats(grads))
        got = _noalloc(grads, cuda)
        _check(got, want)
        _check_oracle(got, grads)


def test_noalloc_rejects_requests_beyond_the_static_capacity(cuda):
    # one more gradient than the partial-record array has records (each
    # gradient takes at least one): 65,537 one-element slices of one real
    # buffer, so every descriptor points at memory the call may read.  The
    # call must refuse before launching anything.
    n = _lib.GRAD_STATS_STATIC_RECORDS + 1
    g = torch.zeros(n, device=cuda)
    refs = np.zeros(n, dtype=_lib.GRADREF_DTYPE)
    refs["grad"] = g.data_ptr() + 4 * np.arange(n, dtype=np.uint64)
    refs["numel"] = 1
    out = torch.full((n * _lib.GRADSTATS_DTYPE.itemsize,), 0xAB, dtype=torch.uint8, device=cuda)
    with torch.cuda.device(cuda):
        rc = _lib.lib().dfc_grad_stats_noalloc(_lib.ptr(refs), n, out.data_ptr(),
                                               torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _lib.DFC_ERR_SCRATCH
    torch.cuda.synchronize()
    assert int((out != 0xAB).sum()) == 0  # nothing was written
    # at the capacity itself the same buffers are accepted
    with torch.cuda.device(cuda):
        rc = _lib.lib().dfc_grad_stats_noalloc(_lib.ptr(refs), n - 1, out.data_ptr(),
                                               torch.cuda.current_stream(cuda).cuda_stream)
    assert rc == _lib.DFC_OK
    st = kernels.stats_to_numpy(out[:(n - 1) * _lib.GRADSTATS_DTYPE.itemsize])
    assert not st["sumsq"].any() and not st["amax"].any() and not st["nonfinite"].any()
