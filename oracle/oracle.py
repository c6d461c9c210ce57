"""CPU oracle for the DFC-AdamW step -- TEST INFRASTRUCTURE ONLY.

Only the test-suite, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import this module; the product package never does.

Two restatements of the reference live here:

* ``dfc_oracle.c`` (loaded through ctypes): element-wise C with explicit
  rounding -- the bit-level checker for the CUDA kernels.
* ``reference_hyper`` / ``multi_tensor_step``: the host-side scalar math and
  the per-parameter bookkeeping of ``DFCAdamW.step`` (remote/torch_fiber.py:
  74-117): per-tensor step counter that advances only when a gradient exists
  (:79-86), bias corrections formed in double (:110-111), f32 rounding of
  each scalar where PyTorch hands a Python float to an FP32 kernel.

Parity of the C restatement against the reference itself is pinned by the
golden vectors in ``tests/golden`` (made by importing the reference).
"""

from __future__ import annotations

import ctypes
import math
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "dfc_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")

MODE_PLAIN = 0
MODE_SIGNFIBER = 1
MODE_PACKED = 2

F32, BF16, F16 = 0, 1, 2
DTYPES = {"f32": F32, "bf16": BF16, "f16": F16}

CFLAGS = ["-O2", "-fPIC", "-shared", "-std=c11", "-ffp-contract=off", "-fno-fast-math",
          "-fexcess-precision=standard"]


def build(force: bool = False) -> str:
    """Compile dfc_oracle.c into liboracle.so beside it (gcc, no build system)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + f".tmp{os.getpid()}"
        subprocess.run(["gcc", *CFLAGS, "-o", tmp, SRC, "-lm"], check=True)
        os.replace(tmp, LIB)
    return LIB


class _Hyper(ctypes.Structure):
    _fields_ = [(name, ctypes.c_float) for name in (
        "beta1", "one_minus_beta1", "beta2", "one_minus_beta2",
        "sqrt_bc2", "eps", "decay", "neg_step_size", "grad_scale")]


_lib = None


def lib():
    global _lib
    if _lib is None:
        handle = ctypes.CDLL(build())
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        handle.orc_step.argtypes = [ctypes.c_int, ctypes.POINTER(_Hyper), P, ctypes.c_int, P,
                                    ctypes.c_int, P, P, I64]
        for name in ("orc_pack_first", "orc_unpack_first", "orc_pack_second", "orc_unpack_second"):
            getattr(handle, name).argtypes = [P, P, I64]
        handle.orc_compress_ef.argtypes = [P, P, P, I64]
        handle.orc_ef_residual.argtypes = [P, P, P, I64]
        handle.orc_grad_stats.argtypes = [P, I64, P, P, P]
        handle.orc_enc_mag.argtypes = [ctypes.c_uint32]
        handle.orc_enc_mag.restype = ctypes.c_uint32
        handle.orc_dec_mag.argtypes = [ctypes.c_uint32]
        handle.orc_dec_mag.restype = ctypes.c_uint32
        _lib = handle
    return _lib


def _f32(x: float) -> float:
    return float(np.float32(x))


@dataclass(frozen=True)
class Hyper:
    """FP32 scalars of one (param group, step) pair, as the reference forms them."""

    beta1: float
    one_minus_beta1: float
    beta2: float
    one_minus_beta2: float
    sqrt_bc2: float
    eps: float
    decay: float
    neg_step_size: float
    grad_scale: float = 1.0

    def ctype(self) -> _Hyper:
        return _Hyper(*(getattr(self, f) for f, _ in _Hyper._fields_))


def reference_hyper(lr, betas, eps, weight_decay, step, grad_scale=1.0) -> Hyper:
    """Scalars of remote/torch_fiber.py:75-116 for one parameter at ``step``.

    bias corrections in double (:110-111); ``mul_(beta)``, ``add_(alpha=1-beta1)``,
    ``addcmul_(value=1-beta2)``, ``div_(sqrt(bc2))``, ``add_(eps)``,
    ``mul_(1-lr*wd)`` (only when wd != 0, :114; multiplying by 1.0 is exact so
    the skip is restated as decay=1) and ``addcdiv_(value=-lr/bc1)`` each round
    their double scalar once to f32.
    """
    beta1, beta2 = betas
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    return Hyper(
        beta1=_f32(beta1),
        one_minus_beta1=_f32(1.0 - beta1),
        beta2=_f32(beta2),
        one_minus_beta2=_f32(1.0 - beta2),
        sqrt_bc2=_f32(math.sqrt(bc2)),
        eps=_f32(eps),
        decay=_f32(1.0 - lr * weight_decay) if weight_decay else 1.0,
        neg_step_size=_f32(-(lr / bc1)),
        grad_scale=_f32(grad_scale),
    )


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def step(mode: int, hyper: Hyper, p: np.ndarray, g: np.ndarray, m: np.ndarray, v: np.ndarray,
         param_dtype: str = "bf16", grad_dtype: str = "bf16") -> None:
    """In-place element-wise step.  p: float32, or uint16 bits of a
    ``param_dtype`` ("bf16"/"f16") parameter; g: float32, or uint16 bits of a
    ``grad_dtype`` gradient; m, v uint32 words (FP32 bit patterns, or packed
    words in MODE_PACKED)."""
    n = p.size
    assert m.dtype == np.uint32 and v.dtype == np.uint32
    assert g.size == n and m.size == n and v.size == n
    pdt = F32 if p.dtype == np.float32 else DTYPES[param_dtype]
    gdt = F32 if g.dtype == np.float32 else DTYPES[grad_dtype]
    if pdt != F32:
        assert p.dtype == np.uint16
    if gdt != F32:
        assert g.dtype == np.uint16
    h = hyper.ctype()
    rc = lib().orc_step(mode, ctypes.byref(h), _ptr(p), pdt, _ptr(g), gdt, _ptr(m), _ptr(v), n)
    if rc != 0:
        raise ValueError(f"oracle step failed: {rc}")


def pack_first(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, np.uint32)
    lib().orc_pack_first(_ptr(x), _ptr(out), x.size)
    return out


def unpack_first(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint32)
    out = np.empty(w.shape, np.float32)
    lib().orc_unpack_first(_ptr(w), _ptr(out), w.size)
    return out


def pack_second(physical_bits: np.ndarray) -> np.ndarray:
    """FP32 sign-fiber word (payload in bit 31) -> packed word (payload kept)."""
    b = np.ascontiguousarray(physical_bits, dtype=np.uint32)
    out = np.empty(b.shape, np.uint32)
    lib().orc_pack_second(_ptr(b), _ptr(out), b.size)
    return out


def unpack_second(w: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, dtype=np.uint32)
    out = np.empty(w.shape, np.uint32)
    lib().orc_unpack_second(_ptr(w), _ptr(out), w.size)
    return out


def compress_ef(g: np.ndarray, c: np.ndarray, q: np.ndarray) -> None:
    """In place: c (bf16 bits, uint16), q (residual field, uint16)."""
    assert g.dtype == np.float32 and c.dtype == np.uint16 and q.dtype == np.uint16
    lib().orc_compress_ef(_ptr(g), _ptr(c), _ptr(q), g.size)


def ef_residual(c: np.ndarray, q: np.ndarray) -> np.ndarray:
    out = np.empty(c.shape, np.float32)
    lib().orc_ef_residual(_ptr(c), _ptr(q), _ptr(out), c.size)
    return out


def grad_stats(g: np.ndarray) -> tuple[float, float, int]:
    g = np.ascontiguousarray(g, dtype=np.float32)
    s = ctypes.c_double()
    a = ctypes.c_float()
    bad = ctypes.c_int64()
    lib().orc_grad_stats(_ptr(g), g.size, ctypes.byref(s), ctypes.byref(a), ctypes.byref(bad))
    return s.value, a.value, bad.value


def multi_tensor_step(mode, tensors, grads, group, steps, param_dtype="bf16"):
    """Reference bookkeeping over a parameter list (remote/torch_fiber.py:74-117).

    tensors: list of dicts with 'p' (float32, or uint16 bits of param_dtype), 'm', 'v'
             (uint32 words), updated in place.
    grads:   list of arrays of the parameter's type, or None (None skips the
             tensor, step not advanced).
    group:   dict(lr, betas, eps, weight_decay[, grad_scale]).
    steps:   list[int] per-tensor step counters, advanced in place.
    """
    for i, (t, g) in enumerate(zip(tensors, grads)):
        if g is None:
            continue
        steps[i] += 1
        h = reference_hyper(group["lr"], group["betas"], group["eps"], group["weight_decay"],
                            steps[i], group.get("grad_scale", 1.0))
        step(mode, h, t["p"], np.ascontiguousarray(g), t["m"], t["v"], param_dtype, param_dtype)


def f32_ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """|a - b| in FP32 ulps on the monotone integer line (sign-magnitude ->
    two's complement), so the distance is meaningful across zero."""
    ai = np.ascontiguousarray(a, dtype=np.float32).view(np.int32).astype(np.int64)
    bi = np.ascontiguousarray(b, dtype=np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)
