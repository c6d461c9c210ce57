"""The C-ABI library loads, exports what the header declares and rejects bad
arguments before touching the GPU.  CPU only: every call here fails
validation, so no CUDA call is made.  The validation tests pass made-up
device addresses; they are skipped wherever a GPU is visible, so that a
regression in the validation order could never send such an address to a
kernel on a real device."""

import ctypes
import os
import re

import numpy as np
import pytest

from t3st_b200 import _lib

# made-up device addresses below: never where a kernel could run
no_device = pytest.mark.skipif(
    __import__("torch").cuda.is_available(),
    reason="passes made-up device addresses; runs only where no GPU is visible")

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "dfc_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dfc_\w+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(_lib.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_version_and_strerror():
    lib = _lib.lib()
    assert lib.dfc_abi_version() == _lib.ABI_VERSION
    for code in range(-9, 1):
        assert _lib.strerror(code) not in ("", "unknown status")
    assert _lib.strerror(-100) == "unknown status"


def test_struct_sizes_match_header():
    text = open(HEADER).read()
    for name, dt in (("DfcSegment", _lib.SEGMENT_DTYPE), ("DfcHyper", _lib.HYPER_DTYPE),
                     ("DfcGradRef", _lib.GRADREF_DTYPE), ("DfcGradStats", _lib.GRADSTATS_DTYPE)):
        m = re.search(r"(\d+) bytes\.\s*\*/\s*typedef struct " + name, text)
        assert m and int(m.group(1)) == dt.itemsize, name


def _seg(**kw):
    s = np.zeros(1, dtype=_lib.SEGMENT_DTYPE)
    s[0] = (0x10000, 0x20000, 0x30000, 0x40000, 16, 0, 0, 0)
    for k, v in kw.items():
        s[0][k] = v
    return s


@no_device
def test_step_rejects_bad_arguments_before_launch():
    lib = _lib.lib()
    h = np.zeros(1, dtype=_lib.HYPER_DTYPE)
    P = _lib.ptr
    assert lib.dfc_mt_step(None, -1, None, 0, 0, None, None) == _lib.DFC_ERR_SIZE
    assert lib.dfc_mt_step(None, 0, None, 0, 7, None, None) == _lib.DFC_ERR_MODE
    assert lib.dfc_mt_step(None, 0, None, 0, 0, None, None) == _lib.DFC_OK
    assert lib.dfc_mt_step(None, 1, P(h), 1, 0, None, None) == _lib.DFC_ERR_NULL
    cases = [
        (_seg(numel=-1), _lib.DFC_ERR_SIZE),
        (_seg(param=0), _lib.DFC_ERR_NULL),
        (_seg(grad=0), _lib.DFC_ERR_NULL),
        (_seg(hyper=1), _lib.DFC_ERR_HYPER),
        (_seg(hyper=-1), _lib.DFC_ERR_HYPER),
        (_seg(grad_dtype=3), _lib.DFC_ERR_DTYPE),
        (_seg(param_dtype=7), _lib.DFC_ERR_DTYPE),
        (_seg(param=0x10001, param_dtype=1), _lib.DFC_ERR_ALIGN),
        (_seg(param=0x10002), _lib.DFC_ERR_ALIGN),
        (_seg(exp_avg_sq=0x40001), _lib.DFC_ERR_ALIGN),
        (_seg(grad=0x20002), _lib.DFC_ERR_ALIGN),
        (_seg(grad=0x20001, grad_dtype=1), _lib.DFC_ERR_ALIGN),
    ]
    for segs, want in cases:
        assert lib.dfc_mt_step(P(segs), 1, P(h), 1, 1, None, None) == want
    # a bad segment after good ones: nothing is launched
    two = np.concatenate([_seg(), _seg(numel=-5)])
    assert lib.dfc_mt_step(P(two), 2, P(h), 1, 1, None, None) == _lib.DFC_ERR_SIZE


@no_device
def test_other_entry_points_reject_bad_arguments():
    lib = _lib.lib()
    assert lib.dfc_compress_ef(None, None, None, -1, 0, None) == _lib.DFC_ERR_SIZE
    assert lib.dfc_compress_ef(None, None, None, 0, 0, None) == _lib.DFC_OK
    assert lib.dfc_compress_ef(None, 0x1000, 0x2000, 4, 0, None) == _lib.DFC_ERR_NULL
    assert lib.dfc_compress_ef(0x1002, 0x1000, 0x2000, 4, 0, None) == _lib.DFC_ERR_ALIGN
    assert lib.dfc_compress_ef(0x1000, 0x1001, 0x2000, 4, 0, None) == _lib.DFC_ERR_ALIGN
    assert lib.dfc_pack_moments(None, -1, 0, None) == _lib.DFC_ERR_SIZE
    assert lib.dfc_pack_moments(None, 4, 0, None) == _lib.DFC_ERR_NULL
    assert lib.dfc_unpack_moments(0x1001, 4, 1, None) == _lib.DFC_ERR_ALIGN

    refs = np.zeros(2, dtype=_lib.GRADREF_DTYPE)
    refs[0] = (0x1000, 10000, 0, 0)
    refs[1] = (0x2000, 1, 1, 0)
    need = lib.dfc_grad_stats_scratch_bytes(_lib.ptr(refs), 2)
    assert need == 3 * _lib.GRADSTATS_DTYPE.itemsize  # 2 tiles + 1 tile of 8192
    assert lib.dfc_grad_stats(_lib.ptr(refs), 2, 0x5000, 0x6000, need - 1, None) == _lib.DFC_ERR_SCRATCH
    assert lib.dfc_grad_stats(_lib.ptr(refs), 2, None, 0x6000, need, None) == _lib.DFC_ERR_NULL
    refs[1]["grad_dtype"] = 5
    assert lib.dfc_grad_stats(_lib.ptr(refs), 2, 0x5000, 0x6000, need, None) == _lib.DFC_ERR_DTYPE
    assert lib.dfc_clip_coef(None, -1, 1.0, None, None, None) == _lib.DFC_ERR_SIZE

    ranges = np.zeros(2, dtype=_lib.WORDRANGE_DTYPE)
    ranges[0] = (0x1000, 10)
    ranges[1] = (0x2000, 6)
    assert lib.dfc_fiber_read(_lib.ptr(ranges), 2, 0, 17, 0x9000, None) == _lib.DFC_ERR_RANGE
    assert lib.dfc_fiber_read(_lib.ptr(ranges), 2, 10, 7, 0x9000, None) == _lib.DFC_ERR_RANGE
    assert lib.dfc_fiber_read(_lib.ptr(ranges), 2, -1, 1, 0x9000, None) == _lib.DFC_ERR_RANGE
    assert lib.dfc_fiber_write(_lib.ptr(ranges), 2, 0, 16, None, None) == _lib.DFC_ERR_NULL
    ranges[1]["words"] = 0x2002
    assert lib.dfc_fiber_write(_lib.ptr(ranges), 2, 0, 16, 0x9000, None) == _lib.DFC_ERR_ALIGN

    comps = (ctypes.c_uint64 * 2)(0x10000, 0x20000)
    params = (ctypes.c_uint64 * 2)(0x30000, 0x40000)
    segs = np.zeros(1, dtype=_lib.PEERSEG_DTYPE)
    segs[0] = (0, 64, 0x50000, 0x60000, 0, 0)
    h = np.zeros(1, dtype=_lib.HYPER_DTYPE)

    def fused(error_flag, n_peers=2, rank=0):
        return lib.dfc_zero_fused_step(comps, params, None, None, n_peers, rank, _lib.ptr(segs), 1,
                                       _lib.ptr(h), 1, _lib.MODE_PACKED, None, error_flag, 0, None)

    assert fused(0x70002) == _lib.DFC_ERR_ALIGN  # the barrier's error flag is an int
    assert fused(0x70000, n_peers=9) == _lib.DFC_ERR_SIZE
    assert fused(0x70000, rank=2) == _lib.DFC_ERR_SIZE
    segs[0]["hyper"] = 1
    assert fused(0x70000) == _lib.DFC_ERR_HYPER
    segs[0]["hyper"] = 0

    # the same step with the next bucket's compression in its grid: the
    # compression range is checked before anything launches
    nxt = np.zeros(1, dtype=_lib.COMPRESSRANGE_DTYPE)

    def fused_ef(rng, n_segs=1, flags=0):
        return lib.dfc_zero_fused_step_ef(comps, params, None, None, 2, 0, _lib.ptr(segs), n_segs,
                                          _lib.ptr(h), 1, _lib.MODE_PACKED, None, 0x70000,
                                          None if rng is None else _lib.ptr(rng), flags, 0, None)

    nxt[0] = (0x80000, 0x90000, 0xA0000, 6)
    assert fused_ef(nxt) == _lib.DFC_ERR_SIZE       # not a whole number of quads
    nxt[0] = (0x80000, 0x90000, 0xA0000, -4)
    assert fused_ef(nxt) == _lib.DFC_ERR_SIZE
    nxt[0] = (0, 0x90000, 0xA0000, 8)
    assert fused_ef(nxt) == _lib.DFC_ERR_NULL
    nxt[0] = (0x80008, 0x90000, 0xA0000, 8)
    assert fused_ef(nxt) == _lib.DFC_ERR_ALIGN      # gradients need 16 bytes
    nxt[0] = (0x80000, 0x90004, 0xA0000, 8)
    assert fused_ef(nxt) == _lib.DFC_ERR_ALIGN      # halves need 8
    nxt[0] = (0x80000, 0x90000, 0xA0000, 8)
    segs[0]["hyper"] = 1
    assert fused_ef(nxt) == _lib.DFC_ERR_HYPER      # the step's own checks still apply
    assert fused_ef(None) == _lib.DFC_ERR_HYPER
    segs[0]["hyper"] = 0
    assert fused_ef(nxt, flags=2) == _lib.DFC_ERR_MODE  # unknown flag bit
    nxt[0] = (0, 0, 0, 0)                            # nothing to compress, no segments: no-op
    assert fused_ef(nxt, n_segs=0) == _lib.DFC_OK
    assert fused_ef(None, n_segs=0) == _lib.DFC_OK


def test_library_is_self_contained():
    """The .so needs no PyTorch library: its dynamic dependencies are the C
    runtime only (the CUDA runtime is linked in statically)."""
    import subprocess

    out = subprocess.run(["ldd", _lib.LIB_PATH], capture_output=True, text=True).stdout
    assert "torch" not in out and "libc10" not in out
