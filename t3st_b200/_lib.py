"""ctypes binding of libdfc_b200.so (the C ABI declared in include/dfc_b200.h).

There is no fallback: if the library is missing or cannot load, every
optimizer entry point raises.  The library holds no PyTorch types; tensors
cross the boundary as raw device pointers, the stream as
``torch.cuda.current_stream().cuda_stream``.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

LIB_PATH = _build.LIB_PATH

# ---- status codes / enums (mirror include/dfc_b200.h) ----
ABI_VERSION = 3
DFC_OK = 0
DFC_ERR_NULL = -1
DFC_ERR_ALIGN = -2
DFC_ERR_SIZE = -3
DFC_ERR_DTYPE = -4
DFC_ERR_MODE = -5
DFC_ERR_HYPER = -6
DFC_ERR_CUDA = -7
DFC_ERR_RANGE = -8
DFC_ERR_SCRATCH = -9

# partial records available to dfc_grad_stats_noalloc (include/dfc_b200.h)
GRAD_STATS_STATIC_RECORDS = 65536

# replay records (include/dfc_b200.h)
REPLAY_RECORD_BYTES = 1552
REPLAY_PIXELS = 3072
RECORD_OK, RECORD_BAD_MAGIC, RECORD_BAD_CRC = 0, 1, 2

MODE_PLAIN = 0
MODE_SIGNFIBER = 1
MODE_PACKED = 2

DTYPE_F32 = 0
DTYPE_BF16 = 1
DTYPE_F16 = 2
GRAD_F32, GRAD_BF16, GRAD_F16 = DTYPE_F32, DTYPE_BF16, DTYPE_F16

# numpy mirrors of the descriptor structs (same byte layout as the C structs)
SEGMENT_DTYPE = np.dtype([("param", "<u8"), ("grad", "<u8"), ("exp_avg", "<u8"),
                          ("exp_avg_sq", "<u8"), ("numel", "<i8"), ("hyper", "<i4"),
                          ("grad_dtype", "<i2"), ("param_dtype", "<i2")])
HYPER_FIELDS = ("beta1", "one_minus_beta1", "beta2", "one_minus_beta2", "sqrt_bc2", "eps",
                "decay", "neg_step_size", "grad_scale")
HYPER_DTYPE = np.dtype([(f, "<f4") for f in HYPER_FIELDS] + [("reserved", "<f4", (3,))])
GRADREF_DTYPE = np.dtype([("grad", "<u8"), ("numel", "<i8"), ("grad_dtype", "<i4"),
                          ("reserved", "<i4")])
GRADSTATS_DTYPE = np.dtype([("sumsq", "<f8"), ("amax", "<f4"), ("reserved", "<i4"),
                            ("nonfinite", "<i8")])
WORDRANGE_DTYPE = np.dtype([("words", "<u8"), ("count", "<i8")])
PEERSEG_DTYPE = np.dtype([("offset", "<i8"), ("numel", "<i8"), ("exp_avg", "<u8"),
                          ("exp_avg_sq", "<u8"), ("hyper", "<i4"), ("reserved", "<i4")])
COMPRESSRANGE_DTYPE = np.dtype([("grad", "<u8"), ("comp", "<u8"), ("resid", "<u8"),
                                ("numel", "<i8")])
MAX_PEERS = 8
FUSED_AFTER_BARRIER = 1  # dfc_zero_fused_step_ef flag
assert SEGMENT_DTYPE.itemsize == 48 and HYPER_DTYPE.itemsize == 48
assert GRADREF_DTYPE.itemsize == 24 and GRADSTATS_DTYPE.itemsize == 24
assert WORDRANGE_DTYPE.itemsize == 16 and PEERSEG_DTYPE.itemsize == 40
assert COMPRESSRANGE_DTYPE.itemsize == 32

# Names of every entry point the header declares (checked by the CPU tests).
EXPORTS = (
    "dfc_abi_version", "dfc_strerror", "dfc_last_cuda_error", "dfc_mt_step",
    "dfc_pack_moments", "dfc_unpack_moments", "dfc_compress_ef",
    "dfc_grad_stats_scratch_bytes", "dfc_grad_stats", "dfc_clip_coef",
    "dfc_fiber_read", "dfc_fiber_write", "dfc_grad_stats_noalloc",
    "dfc_zero_fused_step", "dfc_zero_fused_step_ef", "dfc_peer_barrier",
    "dfc_multicast_sum_bf16",
    "dfc_replay_encode", "dfc_replay_decode",
)


class DfcError(RuntimeError):
    """A non-zero status from libdfc_b200.so."""

    def __init__(self, fn: str, status: int, detail: str = ""):
        self.status = status
        msg = f"{fn} failed: {strerror(status)} ({status})"
        if detail:
            msg += f": {detail}"
        super().__init__(msg)


_lib = None


def _declare(h: ctypes.CDLL) -> None:
    P, I32, I64, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
    sig = {
        "dfc_abi_version": ([], ctypes.c_int),
        "dfc_strerror": ([ctypes.c_int], ctypes.c_char_p),
        "dfc_last_cuda_error": ([], ctypes.c_int),
        "dfc_mt_step": ([P, I32, P, I32, I32, P, P], ctypes.c_int),
        "dfc_pack_moments": ([P, I64, I32, P], ctypes.c_int),
        "dfc_unpack_moments": ([P, I64, I32, P], ctypes.c_int),
        "dfc_compress_ef": ([P, P, P, I64, I32, P], ctypes.c_int),
        "dfc_grad_stats_scratch_bytes": ([P, I32], SZ),
        "dfc_grad_stats": ([P, I32, P, P, SZ, P], ctypes.c_int),
        "dfc_clip_coef": ([P, I32, ctypes.c_float, P, P, P], ctypes.c_int),
        "dfc_fiber_read": ([P, I32, I64, I64, P, P], ctypes.c_int),
        "dfc_fiber_write": ([P, I32, I64, I64, P, P], ctypes.c_int),
        "dfc_grad_stats_noalloc": ([P, I32, P, P], ctypes.c_int),
        "dfc_zero_fused_step": ([P, P, P, P, I32, I32, P, I32, P, I32, I32, P, P, I32, P],
                                ctypes.c_int),
        "dfc_zero_fused_step_ef": ([P, P, P, P, I32, I32, P, I32, P, I32, I32, P, P, P,
                                    ctypes.c_uint32, I32, P], ctypes.c_int),
        "dfc_peer_barrier": ([P, I32, I32, ctypes.c_uint32, P, I64, P], ctypes.c_int),
        "dfc_multicast_sum_bf16": ([P, P, I64, P], ctypes.c_int),
        "dfc_replay_encode": ([P, I64, P, P, I64, P, I64, P], ctypes.c_int),
        "dfc_replay_decode": ([P, I64, I64, P, P, P, P, P], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(h, name)
        fn.argtypes = args
        fn.restype = res


def lib() -> ctypes.CDLL:
    """Load libdfc_b200.so, building it first if it is absent (needs nvcc)."""
    global _lib
    if _lib is None:
        path = LIB_PATH
        if not os.path.exists(path):
            path = _build.build()
        try:
            h = ctypes.CDLL(path)
        except OSError as e:  # pragma: no cover - depends on the machine
            raise ImportError(f"cannot load {path}: {e}") from e
        _declare(h)
        if h.dfc_abi_version() != ABI_VERSION:
            raise ImportError(f"{path}: unexpected ABI version {h.dfc_abi_version()}")
        _lib = h
    return _lib


_host = None


def host():
    """The native host plan module (t3st_b200._dfc_host), built first if it
    is absent (needs g++ and PyTorch's headers)."""
    global _host
    if _host is None:
        import importlib

        import torch  # noqa: F401  (the extension links against libtorch_python)

        if not os.path.exists(_build.HOST_PATH):
            _build.build_host()
        _host = importlib.import_module("t3st_b200._dfc_host")
    return _host


def mt_step_address() -> int:
    """Address of dfc_mt_step in the loaded library (for the host plan)."""
    return ctypes.cast(lib().dfc_mt_step, ctypes.c_void_p).value


def strerror(status: int) -> str:
    return lib().dfc_strerror(status).decode()


def check(fn: str, status: int) -> None:
    if status != DFC_OK:
        detail = ""
        if status == DFC_ERR_CUDA:
            detail = f"cudaError {lib().dfc_last_cuda_error()}"
        raise DfcError(fn, status, detail)


def ptr(a: np.ndarray) -> int:
    return a.ctypes.data
