"""B200 drop-in for the reference's ``torch_fiber`` module (YellowJune/T3st,
remote/torch_fiber.py): ``DFCAdamW``, ``TorchSignFiberChannel``,
``local_fiber_capacity`` and the two bit masks, with the same names,
arguments, state layout and exceptions.

The step itself runs as one fused multi-tensor CUDA launch through the C ABI
of libdfc_b200.so (``dfc_mt_step``); there is no CPU path and no eager
fallback: CPU tensors or a missing library raise.

Additive options (defaults reproduce the reference):
  moment_format="packed"  keep each moment word as bf16-high + 16-bit
                          error-feedback residual-low (bit 31 of the second
                          moment still carries the payload bit);
  max_grad_norm=x         clip by the global gradient norm, computed on the
                          device (warp-shuffle statistics kernel), applied
                          inside the step kernel; no host synchronisation.
"""

from __future__ import annotations

import math
import operator
from collections import deque
from itertools import repeat
from typing import Iterable

import numpy as np
import torch
from torch.optim.optimizer import _global_optimizer_post_hooks, _global_optimizer_pre_hooks

from . import _lib

_profiler_enabled = torch._C._autograd._profiler_enabled

# optimizer attributes a native step plan depends on: if any of them is
# rebound, the plan no longer holds
_PLAN_WATCH = ("param_groups", "state", "enable_fiber", "moment_format", "max_grad_norm")

SIGN_MASK_I32 = -2147483648
MAGNITUDE_MASK_I32 = 2147483647

_FORMATS = ("fp32", "packed")

# parameter and gradient types the kernels read and write directly; other
# floating gradients are converted with .float() (remote/torch_fiber.py:83)
_PARAM_CODES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16,
                torch.float16: _lib.DTYPE_F16}


def _is_dense(t: torch.Tensor) -> bool:
    """True when t's elements occupy one gap-free block of memory in some
    dimension order (contiguous, channels_last, any permutation)."""
    if t.is_contiguous():
        return True
    dims = sorted((st, sz) for st, sz in zip(t.stride(), t.shape) if sz != 1)
    expect = 1
    for st, sz in dims:
        if st != expect:
            return False
        expect *= sz
    return True


def hyper_row(lr: float, betas, eps: float, weight_decay: float, step: int,
              grad_scale: float = 1.0) -> tuple:
    """FP32 scalars of one parameter's update (remote/torch_fiber.py:75-116).

    Every value is formed in double, as the reference does in Python, and is
    rounded once to f32 when stored -- which is what PyTorch does when a
    Python float meets an FP32 tensor: ``mul_(beta1)`` (:98),
    ``add_(alpha=1-beta1)`` (:98), ``mul_(beta2)``/``addcmul_(value=1-beta2)``
    (:99), ``div_(sqrt(bc2))`` and ``add_(eps)`` (:112), ``mul_(1-lr*wd)``
    only when wd != 0 (:114-115; multiplying by 1.0 is exact, so the skip is
    decay=1) and ``addcdiv_(value=-lr/bc1)`` (:116).
    """
    beta1, beta2 = float(betas[0]), float(betas[1])
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    decay = (1.0 - lr * weight_decay) if weight_decay else 1.0
    return (beta1, 1.0 - beta1, beta2, 1.0 - beta2, math.sqrt(bc2), eps, decay,
            -(lr / bc1), grad_scale, (0.0, 0.0, 0.0))


class DFCAdamW(torch.optim.Optimizer):
    """AdamW with one exact payload bit per FP32 second-moment coordinate.

    Same constructor, ``step``, ``state_dict``/``load_state_dict``,
    ``initialize_state``, ``second_moment_tensors`` and
    ``payload_bit_capacity`` as remote/torch_fiber.py:22-117.
    """

    def __init__(
        self,
        params: Iterable[torch.nn.Parameter],
        lr: float = 1e-3,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.0,
        enable_fiber: bool = True,
        *,
        moment_format: str = "fp32",
        max_grad_norm: float | None = None,
    ):
        if lr < 0 or eps < 0 or not 0 <= betas[0] < 1 or not 0 <= betas[1] < 1:
            raise ValueError("invalid AdamW hyperparameters")
        if moment_format not in _FORMATS:
            raise ValueError(f"moment_format must be one of {_FORMATS}")
        if max_grad_norm is not None and not max_grad_norm > 0:
            raise ValueError("max_grad_norm must be positive")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay)
        super().__init__(params, defaults)
        self.enable_fiber = bool(enable_fiber)
        self.moment_format = moment_format
        self.max_grad_norm = max_grad_norm
        self._plan_key = None
        self._plan = None
        self._fast = None
        self._native = None
        self.initialize_state()

    # ---- state (remote/torch_fiber.py:41-66) ----
    @torch.no_grad()
    def initialize_state(self) -> None:
        for group in self.param_groups:
            for parameter in group["params"]:
                if parameter.dtype not in (torch.float16, torch.bfloat16, torch.float32):
                    raise TypeError("DFCAdamW expects floating parameters")
                state = self.state[parameter]
                if not state:
                    state["step"] = 0
                    state["exp_avg"] = torch.zeros_like(
                        parameter, dtype=torch.float32, memory_format=torch.preserve_format)
                    state["exp_avg_sq"] = torch.zeros_like(
                        parameter, dtype=torch.float32, memory_format=torch.preserve_format)

    def second_moment_tensors(self) -> list[torch.Tensor]:
        return [self.state[p]["exp_avg_sq"] for group in self.param_groups for p in group["params"]]

    @property
    def payload_bit_capacity(self) -> int:
        return sum(t.numel() for t in self.second_moment_tensors()) if self.enable_fiber else 0

    @property
    def mode(self) -> int:
        if self.moment_format == "packed":
            return _lib.MODE_PACKED
        return _lib.MODE_SIGNFIBER if self.enable_fiber else _lib.MODE_PLAIN

    # torch.optim.Optimizer pickles defaults, state and param_groups only; the
    # moment format and options travel too, the step plans are rebuilt
    def __getstate__(self):
        st = super().__getstate__()
        st.update(enable_fiber=self.enable_fiber, moment_format=self.moment_format,
                  max_grad_norm=self.max_grad_norm)
        return st

    # load_state_dict goes through __setstate__ too, with state and
    # param_groups only: options missing from `state` keep their current values
    def __setstate__(self, state):
        state = dict(state)
        self.enable_fiber = bool(state.pop("enable_fiber", getattr(self, "enable_fiber", True)))
        self.moment_format = state.pop("moment_format", getattr(self, "moment_format", "fp32"))
        self.max_grad_norm = state.pop("max_grad_norm", getattr(self, "max_grad_norm", None))
        super().__setstate__(state)
        self._plan_key = self._plan = self._fast = self._native = None

    def add_param_group(self, param_group) -> None:
        super().add_param_group(param_group)
        self._plan_key = None
        self._fast = None
        self._native = None
        if hasattr(self, "enable_fiber"):
            self.initialize_state()

    def state_dict(self):
        sd = super().state_dict()
        sd["moment_format"] = self.moment_format
        return sd

    @torch.no_grad()
    def load_state_dict(self, state_dict) -> None:
        """Load a checkpoint of this class or of the reference; moment words
        are converted when the checkpoint's format differs from this
        optimizer's (reference checkpoints are FP32)."""
        saved_format = state_dict.get("moment_format", "fp32")
        if saved_format not in _FORMATS:
            raise ValueError(f"unknown moment_format {saved_format!r} in checkpoint")
        super().load_state_dict(state_dict)
        self._plan_key = None
        self._fast = None
        self._native = None
        if saved_format != self.moment_format:
            convert = (_lib.lib().dfc_pack_moments if self.moment_format == "packed"
                       else _lib.lib().dfc_unpack_moments)
            for group in self.param_groups:
                for p in group["params"]:
                    st = self.state[p]
                    for key, second in (("exp_avg", 0), ("exp_avg_sq", 1)):
                        if not st[key].is_cuda:
                            raise RuntimeError("DFCAdamW state must live on a CUDA device")
                        # load_state_dict may alias the checkpoint's tensors
                        # (same dtype and device): convert a private copy
                        t = st[key] = st[key].clone(memory_format=torch.preserve_format)
                        with torch.cuda.device(t.device):
                            _lib.check(convert.__name__, convert(
                                t.data_ptr(), t.numel(), second,
                                torch.cuda.current_stream(t.device).cuda_stream))

    # ---- the step (remote/torch_fiber.py:68-117) ----
    def step(self, closure=None):
        """One DFC-AdamW step over every parameter with a gradient.

        Steady state (no closure, no step hooks, no profiler): the native
        plan re-checks pointers, dtypes and step counters and launches the
        fused step (one C call).  Otherwise the step runs inside
        torch.optim.Optimizer's wrapper (profiler range, pre/post hooks)."""
        plan = self._native
        if (plan is not None and closure is None and not self._optimizer_step_pre_hooks
                and not self._optimizer_step_post_hooks and not _global_optimizer_pre_hooks
                and not _global_optimizer_post_hooks and not _profiler_enabled()):
            rc = plan.step()
            if rc == 1:
                return None
            self._native = None
            if rc < 0:
                _lib.check("dfc_mt_step", rc)
        return self._hooked_step(closure)

    # torch.optim.Optimizer wraps a subclass's step() in its profiler/hook
    # wrapper unless the function says it is already hooked; this step()
    # applies the same wrapper itself whenever hooks or a profiler are there
    step.hooked = True

    @torch.no_grad()
    def _step_impl(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        plan = self._native  # steps under hooks or a profiler keep the native plan
        if plan is not None:
            rc = plan.step()
            if rc == 1:
                return loss
            self._native = None
            if rc < 0:
                _lib.check("dfc_mt_step", rc)
        fast = self._fast
        if fast is not None and fast.try_step(self):
            return loss
        self._fast = None
        self._step_general()
        return loss

    _hooked_step = torch.optim.Optimizer.profile_hook_step(_step_impl)

    def _step_general(self) -> None:
        work = []  # (param, state, grad, group index)
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                g = p.grad
                if g is None:
                    continue
                if g.is_sparse:
                    raise RuntimeError("DFCAdamW does not support sparse gradients")
                work.append((p, self.state[p], g, gi))
        if not work:
            return

        key = tuple((id(p), id(g)) for p, _, g, _ in work)
        if key != self._plan_key:
            plan = self._build_plan(work)
            # a converted or re-laid-out gradient is a copy of this step's
            # values and cannot be reused next step
            self._plan, self._plan_key = plan, (key if plan[3] else None)
        segs, devices, keepalive, _, perm = self._plan
        if perm is not None:
            work = [work[i] for i in perm]

        # per-tensor step counters (:85-86) and one hyper set per (group, step)
        hyper_rows, hyper_index = [], {}
        hidx = segs["hyper"]
        for i, (p, state, _, gi) in enumerate(work):
            s = state["step"] + 1
            k = (gi, s)
            j = hyper_index.get(k)
            if j is None:
                group = self.param_groups[gi]
                j = hyper_index[k] = len(hyper_rows)
                hyper_rows.append(hyper_row(group["lr"], group["betas"], group["eps"],
                                            group["weight_decay"], s))
            hidx[i] = j
        hypers = np.array(hyper_rows, dtype=_lib.HYPER_DTYPE)

        lib = _lib.lib()
        for dev, sl in devices:
            with torch.cuda.device(dev):
                stream = torch.cuda.current_stream(dev).cuda_stream
                scale_ptr = None
                if self.max_grad_norm is not None:
                    scale_ptr = self._clip_scale(segs[sl], dev, stream)
                _lib.check("dfc_mt_step", lib.dfc_mt_step(
                    _lib.ptr(segs[sl]), sl.stop - sl.start, _lib.ptr(hypers), len(hypers),
                    self.mode, scale_ptr, stream))
        for _, state, _, _ in work:
            state["step"] += 1
        del keepalive
        n_params = sum(len(g["params"]) for g in self.param_groups)
        if len(work) == n_params and len(devices) == 1 and self._plan_key is not None:
            if self.max_grad_norm is None:
                self._native = _native_plan(self, work, segs, devices[0][0])
            if self._native is None:
                self._fast = _FastPlan(self, work, segs, devices[0][0])

    def _build_plan(self, work):
        """Validate every (param, grad, state) triple and lay out the segment
        descriptors, grouped by device (one launch per device).

        Returns (segments, [(device, slice)], tensors to keep alive,
        cacheable, permutation of ``work`` into device order or None)."""
        order = sorted(range(len(work)), key=lambda i: (work[i][0].device.index or 0, i))
        perm = None if order == list(range(len(work))) else order
        if perm is not None:
            work = [work[i] for i in perm]
        segs = np.zeros(len(work), dtype=_lib.SEGMENT_DTYPE)
        keep = []
        devices = []
        start = 0
        for i, (p, state, g, _) in enumerate(work):
            if not p.is_cuda:
                raise RuntimeError("DFCAdamW (t3st_b200) runs on CUDA tensors only; "
                                   "move the model to a CUDA device")
            pcode = _PARAM_CODES.get(p.dtype)
            if pcode is None:
                raise TypeError("DFCAdamW expects floating parameters")
            if g.device != p.device or g.shape != p.shape:
                raise RuntimeError("gradient must match its parameter's device and shape")
            m, v = state["exp_avg"], state["exp_avg_sq"]
            if not _is_dense(p):
                raise RuntimeError("DFCAdamW (t3st_b200) needs dense parameters")
            code = _PARAM_CODES.get(g.dtype)
            if code is None:
                g = g.float()  # remote/torch_fiber.py:83
                code = _lib.DTYPE_F32
            if g.stride() != p.stride():
                g = torch.empty_like(p, dtype=g.dtype).copy_(g)
            if m.stride() != p.stride() or v.stride() != p.stride():
                raise RuntimeError("optimizer state layout differs from its parameter")
            keep.append(g)
            segs[i] = (p.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr(), p.numel(), 0, code,
                       pcode)
            if i + 1 == len(work) or work[i + 1][0].device != p.device:
                devices.append((p.device, slice(start, i + 1)))
                start = i + 1
        if self.max_grad_norm is not None and len(devices) > 1:
            raise NotImplementedError("max_grad_norm needs all parameters on one device")
        cacheable = all(k is w[2] for k, w in zip(keep, work))
        return segs, devices, keep, cacheable, perm

    def _clip_scale(self, segs, dev, stream) -> int:
        lib = _lib.lib()
        refs = np.zeros(len(segs), dtype=_lib.GRADREF_DTYPE)
        refs["grad"] = segs["grad"]
        refs["numel"] = segs["numel"]
        refs["grad_dtype"] = segs["grad_dtype"]
        nbytes = lib.dfc_grad_stats_scratch_bytes(_lib.ptr(refs), len(refs))
        scratch = torch.empty(max(nbytes, 8), dtype=torch.uint8, device=dev)
        stats = torch.empty(len(refs) * _lib.GRADSTATS_DTYPE.itemsize, dtype=torch.uint8, device=dev)
        coef = torch.empty(2, dtype=torch.float32, device=dev)
        _lib.check("dfc_grad_stats", lib.dfc_grad_stats(
            _lib.ptr(refs), len(refs), stats.data_ptr(), scratch.data_ptr(), nbytes, stream))
        _lib.check("dfc_clip_coef", lib.dfc_clip_coef(
            stats.data_ptr(), len(refs), float(self.max_grad_norm), coef.data_ptr(),
            coef.data_ptr() + 4, stream))
        self._last_clip = coef  # coef[0] = clip coefficient, coef[1] = total norm
        return coef.data_ptr()

    @property
    def last_grad_norm(self) -> torch.Tensor | None:
        """Device tensor holding the global gradient norm of the last clipped step."""
        c = getattr(self, "_last_clip", None)
        return None if c is None else c[1]


_GRAD = operator.attrgetter("grad")
_DTYPE = operator.attrgetter("dtype")
_STEP = operator.itemgetter("step")
_IS_SPARSE = operator.attrgetter("is_sparse")
_DATA_PTR = torch.Tensor.data_ptr
_STRIDE = torch.Tensor.stride


def _native_plan(opt: "DFCAdamW", work, segs, device, launch=None):
    """The native steady-state plan (t3st_b200._dfc_host.StepPlan) for the
    descriptors of the step just taken, or None where it does not apply
    (parameters that are tensor subclasses).  ``launch`` is the address of a
    function with dfc_mt_step's signature (default: dfc_mt_step itself)."""
    host = _lib.host()
    segs = segs.copy()
    segs["hyper"] = [w[3] for w in work]
    hyp = np.zeros(len(opt.param_groups), dtype=_lib.HYPER_DTYPE)
    try:
        return host.StepPlan([w[0] for w in work], [w[1] for w in work], opt.param_groups, segs,
                             hyp, opt.mode, device.index or 0,
                             launch if launch is not None else _lib.mt_step_address(),
                             opt.__dict__, _PLAN_WATCH)
    except (TypeError, ValueError):
        return None


class _FastPlan:
    """Steady-state step with gradient clipping (max_grad_norm), or over
    parameters the native plan does not take: every parameter has a gradient, one device, one
    step count shared by all parameters, the same parameter and gradient
    storage as the step that built the plan.  Checking that costs a few
    C-level passes over the parameter list (pointers, dtypes, counters); any
    mismatch falls back to the general path, which re-validates everything."""

    def __init__(self, opt: "DFCAdamW", work, segs, device):
        self.params = [w[0] for w in work]
        self.states = [w[1] for w in work]
        self.grads = [w[2] for w in work]
        self.pptrs = list(map(_DATA_PTR, self.params))
        self.gptrs = list(map(_DATA_PTR, self.grads))
        self.gdtypes = list(map(_DTYPE, self.grads))
        self.gstrides = list(map(_STRIDE, self.grads))
        self.mode = opt.mode
        self.device = device
        self.segs = segs.copy()
        self.segs["hyper"] = [w[3] for w in work]
        self.hyp = np.zeros(len(opt.param_groups), dtype=_lib.HYPER_DTYPE)
        self.n_groups = len(opt.param_groups)
        self.segs_ptr = _lib.ptr(self.segs)  # both arrays live as long as the plan
        self.hyp_ptr = _lib.ptr(self.hyp)

    def try_step(self, opt: "DFCAdamW") -> bool:
        grads = list(map(_GRAD, self.params))
        try:
            gptrs = list(map(_DATA_PTR, grads))
        except TypeError:  # a parameter without gradient
            return False
        if list(map(_DATA_PTR, self.params)) != self.pptrs:
            return False
        if not all(map(operator.is_, grads, self.grads)):
            # new gradient tensors (zero_grad(set_to_none=True) then backward):
            # PyTorch keeps a .grad on its parameter's device with its shape and
            # dtype; the plan holds while the layout matches, with new pointers
            if (list(map(_DTYPE, grads)) != self.gdtypes
                    or list(map(_STRIDE, grads)) != self.gstrides
                    or any(map(_IS_SPARSE, grads))):
                return False
            if gptrs != self.gptrs:
                self.segs["grad"] = gptrs
                self.gptrs = gptrs
            self.grads = grads
        elif gptrs != self.gptrs:  # storage swapped under the same tensor
            return False
        steps = list(map(_STEP, self.states))
        s = steps[0]
        if steps.count(s) != len(steps) or opt.mode != self.mode or \
                len(opt.param_groups) != self.n_groups:
            return False
        s += 1
        for gi, group in enumerate(opt.param_groups):
            self.hyp[gi] = hyper_row(group["lr"], group["betas"], group["eps"],
                                     group["weight_decay"], s)
        dev = self.device
        lib = _lib.lib()
        if torch.cuda.current_device() != dev.index:
            with torch.cuda.device(dev):
                return self._launch(opt, lib, dev, s)
        return self._launch(opt, lib, dev, s)

    def _launch(self, opt, lib, dev, s) -> bool:
        stream = torch.cuda.current_stream(dev).cuda_stream
        scale_ptr = None
        if opt.max_grad_norm is not None:
            scale_ptr = opt._clip_scale(self.segs, dev, stream)
        _lib.check("dfc_mt_step", lib.dfc_mt_step(
            self.segs_ptr, len(self.segs), self.hyp_ptr, self.n_groups, self.mode, scale_ptr,
            stream))
        deque(map(operator.setitem, self.states, repeat("step"), repeat(s)), 0)
        return True


class TorchSignFiberChannel:
    """Byte-addressable sign fiber over a DFCAdamW state shard
    (remote/torch_fiber.py:120-185).  Reads and writes run as one device
    kernel each (``dfc_fiber_read``/``dfc_fiber_write``) with a single
    host<->device copy of the packed payload."""

    def __init__(self, optimizer: DFCAdamW):
        if not optimizer.enable_fiber:
            raise ValueError("optimizer fiber is disabled")
        self.optimizer = optimizer
        self.tensors = optimizer.second_moment_tensors()
        self.ends = np.cumsum([t.numel() for t in self.tensors], dtype=np.int64)
        devs = {t.device for t in self.tensors}
        if any(not d.type == "cuda" for d in devs) or len(devs) > 1:
            raise RuntimeError("TorchSignFiberChannel (t3st_b200) needs the state on one CUDA device")
        self.device = next(iter(devs)) if devs else None
        for t in self.tensors:
            if not t.is_contiguous() and not _is_dense(t):
                raise RuntimeError("second-moment tensors must be dense")
        self._ranges = np.zeros(len(self.tensors), dtype=_lib.WORDRANGE_DTYPE)
        for i, t in enumerate(self.tensors):
            self._ranges[i] = (t.data_ptr(), t.numel())

    @property
    def bit_capacity(self) -> int:
        return int(self.ends[-1]) if self.ends.size else 0

    @property
    def byte_capacity(self) -> int:
        return self.bit_capacity // 8

    def _check(self, start: int, count: int) -> None:
        if start < 0 or count < 0 or start + count > self.bit_capacity:
            raise IndexError("fiber range out of bounds")

    def _read_dev(self, start: int, count: int) -> torch.Tensor:
        out = torch.empty((count + 7) // 8, dtype=torch.uint8, device=self.device)
        if count:
            with torch.cuda.device(self.device):
                _lib.check("dfc_fiber_read", _lib.lib().dfc_fiber_read(
                    _lib.ptr(self._ranges), len(self._ranges), start, count, out.data_ptr(),
                    torch.cuda.current_stream(self.device).cuda_stream))
        return out

    def _write_dev(self, start: int, count: int, src: torch.Tensor) -> None:
        if count == 0:
            return
        with torch.cuda.device(self.device):
            src = src.to(device=self.device, dtype=torch.uint8).contiguous()
            _lib.check("dfc_fiber_write", _lib.lib().dfc_fiber_write(
                _lib.ptr(self._ranges), len(self._ranges), start, count, src.data_ptr(),
                torch.cuda.current_stream(self.device).cuda_stream))

    def _read_packed(self, start: int, count: int) -> np.ndarray:
        if count == 0:
            return np.empty(0, dtype=np.uint8)
        return self._read_dev(start, count).cpu().numpy()

    def _write_packed(self, start: int, count: int, packed: np.ndarray) -> None:
        if count == 0:
            return
        self._write_dev(start, count, torch.from_numpy(np.array(packed, dtype=np.uint8, copy=True)))

    @torch.no_grad()
    def read_bits(self, start: int, count: int) -> np.ndarray:
        self._check(start, count)
        packed = self._read_packed(int(start), int(count))
        return np.unpackbits(packed, bitorder="little")[:count] if count else packed

    @torch.no_grad()
    def write_bits(self, start: int, payload: np.ndarray) -> None:
        bits = np.ascontiguousarray(payload, dtype=np.uint8).reshape(-1)
        if np.any(bits > 1):
            raise ValueError("payload must be binary")
        self._check(start, bits.size)
        self._write_packed(int(start), bits.size, np.packbits(bits, bitorder="little"))

    def read_bytes(self, start: int, count: int) -> bytes:
        if start < 0 or count < 0 or start + count > self.byte_capacity:
            raise IndexError("fiber byte range out of bounds")
        return self._read_packed(int(start) * 8, int(count) * 8).tobytes()

    def write_bytes(self, start: int, payload: bytes | bytearray | memoryview) -> None:
        raw = bytes(payload)
        if start < 0 or start + len(raw) > self.byte_capacity:
            raise IndexError("fiber byte range out of bounds")
        self._write_packed(int(start) * 8, len(raw) * 8, np.frombuffer(raw, dtype=np.uint8))

    # device-resident byte I/O (no reference counterpart): the replay codec
    # moves records between the fiber and its kernels without a host copy
    @torch.no_grad()
    def read_device(self, start: int, count: int) -> torch.Tensor:
        """Bytes [start, start + count) as a uint8 tensor on the fiber's device."""
        if start < 0 or count < 0 or start + count > self.byte_capacity:
            raise IndexError("fiber byte range out of bounds")
        return self._read_dev(int(start) * 8, int(count) * 8)

    @torch.no_grad()
    def write_device(self, start: int, data: torch.Tensor) -> None:
        """Write the uint8 tensor ``data`` (any device) at byte ``start``."""
        if data.dtype != torch.uint8:
            raise TypeError("fiber bytes are uint8")
        n = data.numel()
        if start < 0 or start + n > self.byte_capacity:
            raise IndexError("fiber byte range out of bounds")
        self._write_dev(int(start) * 8, n * 8, data.reshape(-1))


def local_fiber_capacity(optimizer: DFCAdamW) -> dict[str, int]:
    """Report capacity for a single optimizer/DDP/FSDP shard (remote/torch_fiber.py:188-191)."""
    bits = optimizer.payload_bit_capacity
    return {"payload_bits": bits, "payload_bytes": bits // 8, "state_coordinates": bits}
