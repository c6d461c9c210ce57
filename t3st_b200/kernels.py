"""Tensor-level calls into libdfc_b200.so.

Each function takes CUDA tensors, checks their dtype and device, builds the
host descriptor arrays of the C ABI and launches on the current stream of
the tensors' device.  Nothing here falls back to PyTorch arithmetic.
"""

from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from . import _lib

DTYPE_CODES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
               torch.float16: _lib.DTYPE_F16}
_GRAD_CODES = DTYPE_CODES


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need_cuda(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("t3st_b200 kernels take CUDA tensors only")
        if t.device != dev:
            raise RuntimeError("all tensors of one call must share a device")
    return dev


def _words(t: torch.Tensor) -> torch.Tensor:
    if t.dtype not in (torch.float32, torch.int32, torch.uint32):
        raise TypeError("moment words must be a 32-bit tensor")
    return t


def segments(params: Sequence[torch.Tensor], grads: Sequence[torch.Tensor],
             exp_avgs: Sequence[torch.Tensor], exp_avg_sqs: Sequence[torch.Tensor],
             hyper_index: Sequence[int]) -> np.ndarray:
    """Segment descriptors for dfc_mt_step (host array)."""
    n = len(params)
    if not (len(grads) == len(exp_avgs) == len(exp_avg_sqs) == len(hyper_index) == n):
        raise ValueError("segment lists differ in length")
    segs = np.zeros(n, dtype=_lib.SEGMENT_DTYPE)
    for i in range(n):
        p, g, m, v = params[i], grads[i], _words(exp_avgs[i]), _words(exp_avg_sqs[i])
        pcode = DTYPE_CODES.get(p.dtype)
        if pcode is None:
            raise TypeError("parameters must be FP32, bf16 or fp16")
        code = DTYPE_CODES.get(g.dtype)
        if code is None:
            raise TypeError("gradients must be FP32, bf16 or fp16")
        if not (p.numel() == g.numel() == m.numel() == v.numel()):
            raise ValueError("segment tensors differ in size")
        if not (p.is_contiguous() and g.is_contiguous() and m.is_contiguous() and v.is_contiguous()):
            raise ValueError("segment tensors must be contiguous")
        segs[i] = (p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(),
                   int(hyper_index[i]), code, pcode)
    return segs


def hypers(rows: Sequence[tuple]) -> np.ndarray:
    """Hyper-set array from rows of (beta1, 1-beta1, beta2, 1-beta2, sqrt_bc2,
    eps, decay, neg_step_size[, grad_scale]) -- doubles, rounded to f32 here."""
    out = np.zeros(len(rows), dtype=_lib.HYPER_DTYPE)
    for i, r in enumerate(rows):
        r = tuple(r)[:9]
        if len(r) == 8:
            r = r + (1.0,)
        for f, x in zip(_lib.HYPER_FIELDS, r):
            out[i][f] = x
    return out


def mt_step_raw(segs: np.ndarray, hyp: np.ndarray, mode: int, device: torch.device,
                device_grad_scale: torch.Tensor | None = None) -> None:
    """One dfc_mt_step call with prepared descriptor arrays."""
    scale_ptr = None
    if device_grad_scale is not None:
        if device_grad_scale.dtype != torch.float32 or not device_grad_scale.is_cuda:
            raise TypeError("device_grad_scale must be a CUDA float32 tensor")
        scale_ptr = device_grad_scale.data_ptr()
    with torch.cuda.device(device):
        _lib.check("dfc_mt_step", _lib.lib().dfc_mt_step(
            _lib.ptr(segs), len(segs), _lib.ptr(hyp), len(hyp), mode, scale_ptr, _stream(device)))


def mt_step(params, grads, exp_avgs, exp_avg_sqs, hyper_rows, hyper_index, mode: int,
            device_grad_scale: torch.Tensor | None = None) -> None:
    """Fused multi-tensor step over lists of contiguous CUDA tensors."""
    dev = _need_cuda(*params, *grads, *exp_avgs, *exp_avg_sqs)
    mt_step_raw(segments(params, grads, exp_avgs, exp_avg_sqs, hyper_index), hypers(hyper_rows),
                mode, dev, device_grad_scale)


def pack_moments(words: torch.Tensor, second: bool) -> None:
    dev = _need_cuda(words)
    with torch.cuda.device(dev):
        _lib.check("dfc_pack_moments", _lib.lib().dfc_pack_moments(
            _words(words).data_ptr(), words.numel(), int(second), _stream(dev)))


def unpack_moments(words: torch.Tensor, second: bool) -> None:
    dev = _need_cuda(words)
    with torch.cuda.device(dev):
        _lib.check("dfc_unpack_moments", _lib.lib().dfc_unpack_moments(
            _words(words).data_ptr(), words.numel(), int(second), _stream(dev)))


def compress_ef(grad: torch.Tensor, comp: torch.Tensor, resid: torch.Tensor,
                ctas_per_sm: int = 0) -> None:
    """bf16 compression with error feedback, in place on (comp, resid);
    ctas_per_sm > 0 caps the grid (room for a kernel beside it)."""
    dev = _need_cuda(grad, comp, resid)
    if grad.dtype != torch.float32:
        raise TypeError("grad must be FP32")
    if comp.element_size() != 2 or resid.element_size() != 2:
        raise TypeError("comp and resid must be 16-bit tensors")
    if not (grad.numel() == comp.numel() == resid.numel()):
        raise ValueError("sizes differ")
    if not (grad.is_contiguous() and comp.is_contiguous() and resid.is_contiguous()):
        raise ValueError("tensors must be contiguous")
    with torch.cuda.device(dev):
        _lib.check("dfc_compress_ef", _lib.lib().dfc_compress_ef(
            grad.data_ptr(), comp.data_ptr(), resid.data_ptr(), grad.numel(), int(ctas_per_sm),
            _stream(dev)))


def grad_refs(grads: Sequence[torch.Tensor]) -> np.ndarray:
    refs = np.zeros(len(grads), dtype=_lib.GRADREF_DTYPE)
    for i, g in enumerate(grads):
        code = DTYPE_CODES.get(g.dtype)
        if code is None:
            raise TypeError("gradients must be FP32, bf16 or fp16")
        if not g.is_contiguous():
            raise ValueError("gradients must be contiguous")
        refs[i] = (g.data_ptr(), g.numel(), code, 0)
    return refs


def grad_stats(grads: Sequence[torch.Tensor]) -> torch.Tensor:
    """Per-gradient (sumsq, amax, nonfinite) records as a uint8 CUDA tensor of
    n*24 bytes; view with ``stats_to_numpy`` after a copy to the host."""
    dev = _need_cuda(*grads)
    refs = grad_refs(grads)
    lib = _lib.lib()
    nbytes = lib.dfc_grad_stats_scratch_bytes(_lib.ptr(refs), len(refs))
    with torch.cuda.device(dev):
        scratch = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=dev)
        out = torch.empty(max(len(refs), 1) * _lib.GRADSTATS_DTYPE.itemsize, dtype=torch.uint8,
                          device=dev)
        _lib.check("dfc_grad_stats", lib.dfc_grad_stats(
            _lib.ptr(refs), len(refs), out.data_ptr(), scratch.data_ptr(), nbytes, _stream(dev)))
    return out[: len(refs) * _lib.GRADSTATS_DTYPE.itemsize]


def stats_to_numpy(stats: torch.Tensor) -> np.ndarray:
    return stats.cpu().numpy().view(_lib.GRADSTATS_DTYPE)


def clip_coef(stats: torch.Tensor, n: int, max_norm: float) -> torch.Tensor:
    """Device tensor [coef, total_norm] from statistics records."""
    dev = _need_cuda(stats)
    with torch.cuda.device(dev):
        out = torch.empty(2, dtype=torch.float32, device=dev)
        _lib.check("dfc_clip_coef", _lib.lib().dfc_clip_coef(
            stats.data_ptr(), n, float(max_norm), out.data_ptr(), out.data_ptr() + 4, _stream(dev)))
    return out
