"""ZeRO-1 sharded DFC-AdamW across the GPUs of one node.

Every rank holds the full FP32 parameters and computes its own full
gradient (data parallel); the optimizer state is split into N contiguous
shards of the flattened parameter vector.  One step:

  1. compress the local gradient to bf16 with per-element error feedback
     (``dfc_compress_ef``; N > 1 only);
  2. NCCL reduce-scatter (sum) of the bf16 gradients -> this rank's shard;
  3. fused DFC-AdamW step on the shard (``dfc_mt_step``, bf16 gradients,
     grad_scale = 1/N to average), packed moment words by default;
  4. NCCL all-gather of the updated FP32 shard into every rank's parameters.

The parameters are re-homed into one flat FP32 buffer (each becomes a view
of it) and their ``.grad`` into one flat gradient buffer, so the collectives
run on contiguous memory with no packing copies.  Each parameter starts on a
16-element boundary and each shard on a 64-element boundary, so every segment
of the step is 16-byte aligned.  The reference has no distributed code; its
docstrings only say that FP32 state keeps the payload under DDP/FSDP local
shards (remote/torch_fiber.py:3-6, 188-191) -- here the sign fiber of a rank
is the payload bit of its own shard's second-moment words.
"""

from __future__ import annotations

import math
from typing import Iterable

import numpy as np
import torch
import torch.distributed as dist

from . import _lib, kernels
from .torch_fiber import _FORMATS, hyper_row

PARAM_ALIGN = 16   # elements (64 bytes)
SHARD_ALIGN = 64   # elements (256 bytes)


class CudaKernels:
    """The product backend: libdfc_b200.so kernels on CUDA tensors.  The
    step's descriptor array is built once (the buffers never move) and only
    its hyper-set column changes between steps."""

    def __init__(self):
        self._segs = None
        self._key = None

    def compress_ef(self, grad, comp, resid):
        kernels.compress_ef(grad, comp, resid)

    def step(self, segments, hyper_rows, hyper_index, mode, device):
        key = tuple((p.data_ptr(), g.data_ptr(), m.data_ptr(), p.numel()) for p, g, m, _ in segments)
        if key != self._key:
            ps, gs, ms, vs = zip(*segments) if segments else ((), (), (), ())
            self._segs = kernels.segments(ps, gs, ms, vs, hyper_index)
            self._key = key
        self._segs["hyper"] = hyper_index
        kernels.mt_step_raw(self._segs, kernels.hypers(hyper_rows), mode, device)

    def convert(self, words, pack: bool, second: bool):
        (kernels.pack_moments if pack else kernels.unpack_moments)(words, second)


class ShardedDFCAdamW(torch.optim.Optimizer):
    """ZeRO-1 DFC-AdamW.  Same hyperparameters as DFCAdamW; extra options:

    process_group   group to shard over (default: the world)
    moment_format   "packed" (default) or "fp32"
    compress_grads  bf16 + error-feedback compression before the
                    reduce-scatter (default: on when the group has > 1 rank)
    average_grads   divide the summed gradient by the group size (default on)
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-3,
                 betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, enable_fiber: bool = True, *,
                 moment_format: str = "packed", process_group=None,
                 compress_grads: bool | None = None, average_grads: bool = True,
                 backend=None):
        if lr < 0 or eps < 0 or not 0 <= betas[0] < 1 or not 0 <= betas[1] < 1:
            raise ValueError("invalid AdamW hyperparameters")
        if moment_format not in _FORMATS:
            raise ValueError(f"moment_format must be one of {_FORMATS}")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.enable_fiber = bool(enable_fiber)
        self.moment_format = moment_format
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.compress = (self.world > 1) if compress_grads is None else bool(compress_grads)
        self.average = bool(average_grads)
        self.kernels = backend if backend is not None else CudaKernels()
        self._layout()

    # ---- layout -----------------------------------------------------------
    @torch.no_grad()
    def _layout(self):
        self.params = [p for g in self.param_groups for p in g["params"]]
        self.group_of = [gi for gi, g in enumerate(self.param_groups) for _ in g["params"]]
        if not self.params:
            raise ValueError("no parameters")
        dev = self.params[0].device
        for p in self.params:
            if p.dtype != torch.float32:
                raise NotImplementedError("ShardedDFCAdamW updates FP32 parameters")
            if p.device != dev:
                raise RuntimeError("all parameters must live on one device")
        self.device = dev
        offs, o = [], 0
        for p in self.params:
            offs.append(o)
            o += -(-p.numel() // PARAM_ALIGN) * PARAM_ALIGN
        n = self.world
        self.shard = -(-o // (n * SHARD_ALIGN)) * SHARD_ALIGN
        self.padded = self.shard * n
        self.offsets = offs
        self.flat_param = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        self.flat_grad = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        for p, off in zip(self.params, offs):
            k = p.numel()
            self.flat_param[off:off + k].copy_(p.detach().reshape(-1))
            p.data = self.flat_param[off:off + k].view_as(p)
            p.grad = self.flat_grad[off:off + k].view_as(p)
        lo = self.rank * self.shard
        self.shard_range = (lo, lo + self.shard)
        if self.compress:
            self.comp = torch.zeros(self.padded, dtype=torch.int16, device=dev)
            self.resid = torch.zeros(self.padded, dtype=torch.int16, device=dev)
            self.shard_grad = torch.zeros(self.shard, dtype=torch.bfloat16, device=dev)
        elif n > 1:
            self.shard_grad = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        else:
            self.shard_grad = self.flat_grad
        self.exp_avg = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        # one segment per parameter slice that falls inside this shard
        self.segments, self.seg_param = [], []
        for i, (p, off) in enumerate(zip(self.params, offs)):
            a, b = max(off, lo), min(off + p.numel(), lo + self.shard)
            if a >= b:
                continue
            s = a - lo
            g = self.shard_grad[s:s + b - a] if self.shard_grad is not self.flat_grad \
                else self.flat_grad[a:b]
            self.segments.append((self.flat_param[a:b], g, self.exp_avg[s:s + b - a],
                                  self.exp_avg_sq[s:s + b - a]))
            self.seg_param.append(i)
        for p in self.params:
            self.state[p]["step"] = 0

    @property
    def mode(self) -> int:
        if self.moment_format == "packed":
            return _lib.MODE_PACKED
        return _lib.MODE_SIGNFIBER if self.enable_fiber else _lib.MODE_PLAIN

    def add_param_group(self, param_group):
        if hasattr(self, "params"):
            raise RuntimeError("ShardedDFCAdamW fixes its parameter set at construction")
        super().add_param_group(param_group)

    # ---- reference-compatible surface --------------------------------------
    def second_moment_tensors(self) -> list[torch.Tensor]:
        """Second-moment words of this rank's shard, one view per parameter
        slice (alignment padding excluded): this rank's sign fiber."""
        return [v for _, _, _, v in self.segments]

    @property
    def payload_bit_capacity(self) -> int:
        return sum(v.numel() for _, _, _, v in self.segments) if self.enable_fiber else 0

    @torch.no_grad()
    def zero_grad(self, set_to_none: bool = False):
        """Zero the flat gradient buffer; the .grad views stay in place."""
        self.flat_grad.zero_()

    # ---- the step ------------------------------------------------------------
    @torch.no_grad()
    def step(self, closure=None):
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._check_grads()
        n = self.world
        if self.compress:
            self.kernels.compress_ef(self.flat_grad, self.comp, self.resid)
            if n > 1:
                dist.reduce_scatter_tensor(self.shard_grad, self.comp.view(torch.bfloat16),
                                           op=dist.ReduceOp.SUM, group=self.group)
            else:
                self.shard_grad.copy_(self.comp.view(torch.bfloat16))
        elif n > 1:
            dist.reduce_scatter_tensor(self.shard_grad, self.flat_grad, op=dist.ReduceOp.SUM,
                                       group=self.group)
        scale = 1.0 / n if (self.average and n > 1) else 1.0
        rows, index, seen = [], [], {}
        steps = []
        for p, gi in zip(self.params, self.group_of):
            st = self.state[p]
            st["step"] += 1
            steps.append(st["step"])
        for pi in self.seg_param:
            k = (self.group_of[pi], steps[pi])
            j = seen.get(k)
            if j is None:
                g = self.param_groups[k[0]]
                j = seen[k] = len(rows)
                rows.append(hyper_row(g["lr"], g["betas"], g["eps"], g["weight_decay"], k[1],
                                      grad_scale=scale))
            index.append(j)
        if self.segments:
            self.kernels.step(self.segments, rows, index, self.mode, self.device)
        if n > 1:
            lo, hi = self.shard_range
            dist.all_gather_into_tensor(self.flat_param, self.flat_param[lo:hi], group=self.group)
        return loss

    def _check_grads(self):
        # the step reads the flat gradient buffer; a .grad rebound elsewhere
        # would be silently ignored, so refuse it
        for p, off in zip(self.params, self.offsets):
            g = p.grad
            if g is None or g.data_ptr() != self.flat_grad.data_ptr() + 4 * off:
                raise RuntimeError("ShardedDFCAdamW owns .grad of its parameters; use its "
                                   "zero_grad() (set_to_none is not supported)")

    # ---- checkpoints -------------------------------------------------------
    def state_dict(self):
        """This rank's shard (moment words, step counters, layout)."""
        return {
            "shard": {"exp_avg": self.exp_avg.clone(), "exp_avg_sq": self.exp_avg_sq.clone(),
                      "rank": self.rank, "world": self.world, "shard": self.shard},
            "steps": [self.state[p]["step"] for p in self.params],
            "param_groups": [{k: v for k, v in g.items() if k != "params"}
                             for g in self.param_groups],
            "moment_format": self.moment_format,
        }

    @torch.no_grad()
    def load_state_dict(self, state_dict):
        sh = state_dict["shard"]
        if sh["world"] != self.world or sh["shard"] != self.shard or sh["rank"] != self.rank:
            raise ValueError("shard layout differs; use load_consolidated_state_dict")
        self.exp_avg.copy_(sh["exp_avg"])
        self.exp_avg_sq.copy_(sh["exp_avg_sq"])
        for p, s in zip(self.params, state_dict["steps"]):
            self.state[p]["step"] = int(s)
        for g, saved in zip(self.param_groups, state_dict["param_groups"]):
            g.update(saved)
        self._convert_from(state_dict.get("moment_format", "fp32"))

    def _convert_from(self, fmt):
        if fmt not in _FORMATS:
            raise ValueError(f"unknown moment_format {fmt!r}")
        if fmt != self.moment_format:
            pack = self.moment_format == "packed"
            self.kernels.convert(self.exp_avg, pack, False)
            self.kernels.convert(self.exp_avg_sq, pack, True)

    @torch.no_grad()
    def consolidated_state_dict(self, to_rank: int | None = 0):
        """The whole optimizer state in DFCAdamW's per-parameter layout
        (``state[i] = {step, exp_avg, exp_avg_sq}``), gathered from every
        shard.  Collective: every rank must call it.  Returns the dict on
        ``to_rank`` (every rank when None), else None."""
        full_m = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        full_v = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        if self.world > 1:
            dist.all_gather_into_tensor(full_m, self.exp_avg, group=self.group)
            dist.all_gather_into_tensor(full_v, self.exp_avg_sq, group=self.group)
        else:
            full_m.copy_(self.exp_avg)
            full_v.copy_(self.exp_avg_sq)
        if to_rank is not None and self.rank != to_rank:
            return None
        state, groups, idx = {}, [], 0
        for g in self.param_groups:
            entry = {k: v for k, v in g.items() if k != "params"}
            entry["params"] = list(range(idx, idx + len(g["params"])))
            idx += len(g["params"])
            groups.append(entry)
        for i, (p, off) in enumerate(zip(self.params, self.offsets)):
            k = p.numel()
            state[i] = {"step": self.state[p]["step"],
                        "exp_avg": full_m[off:off + k].view_as(p).clone(),
                        "exp_avg_sq": full_v[off:off + k].view_as(p).clone()}
        return {"state": state, "param_groups": groups, "moment_format": self.moment_format}

    @torch.no_grad()
    def load_consolidated_state_dict(self, state_dict):
        """Load a per-parameter state dict (this class's consolidated form,
        DFCAdamW's, or the reference's) and keep this rank's shard."""
        st = state_dict["state"]
        lo, hi = self.shard_range
        flat_m = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        flat_v = torch.zeros(self.padded, dtype=torch.float32, device=self.device)
        for i, (p, off) in enumerate(zip(self.params, self.offsets)):
            s = st.get(i, st.get(str(i)))
            if s is None:
                continue
            k = p.numel()
            flat_m[off:off + k].copy_(s["exp_avg"].reshape(-1))
            flat_v[off:off + k].copy_(s["exp_avg_sq"].reshape(-1))
            self.state[p]["step"] = int(s["step"])
        self.exp_avg.copy_(flat_m[lo:hi])
        self.exp_avg_sq.copy_(flat_v[lo:hi])
        for g, saved in zip(self.param_groups, state_dict["param_groups"]):
            g.update({k: v for k, v in saved.items() if k != "params"})
        self._convert_from(state_dict.get("moment_format", "fp32"))
