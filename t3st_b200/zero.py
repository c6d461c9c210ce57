"""ZeRO-1 sharded DFC-AdamW across the GPUs of one node.

Every rank holds the full FP32 parameters and computes its own full
gradient (data parallel); the optimizer state is sharded.  The flattened
parameter vector is cut into buckets of ``bucket_elems`` elements and each
bucket into N equal pieces; rank r owns piece r of every bucket.  One step,
per bucket b, pipelined across buckets:

  C(b)   compress the local gradient to bf16 with per-element error
         feedback (``dfc_compress_ef``; when compressing);
  RS(b)  NCCL reduce-scatter (sum) of the bucket -> this rank's piece;
  S(b)   fused DFC-AdamW step on the piece (``dfc_mt_step``, bf16 gradients,
         grad_scale = 1/N to average), packed moment words by default;
  AG(b)  NCCL all-gather of the updated FP32 piece into every rank's bucket.

With transport="nccl" the host issues C(0) RS(0), then for each b: C(b+1)
RS(b+1), wait RS(b), S(b) AG(b); the collectives run in that order on
NCCL's stream and the kernels on the caller's stream.  With transport="peer"
(the fast path) RS, S and AG of a bucket are one kernel over NVLink peer
memory (dfc_zero_fused_step): it reads every rank's bf16 values of its
piece, sums them in FP32 in rank order, steps, and stores the new FP32
parameters into every rank's copy; a cross-GPU barrier before it (every
rank's C(b) done) and one at the end of the step (every rank's parameters
done) order the ranks, and C(b+1) on the caller's stream overlaps the fused
kernel of bucket b on a side stream (the compression grid is capped so that
the two kernels share the SMs).  transport="nvls" is the same kernel with
the reduction and the broadcast done by the NVSwitch.  With
fuse_compression, C(b+1) runs inside the grid of bucket b's fused kernel
(dfc_zero_fused_step_ef) rather than as a capped kernel on a second stream:
one stream, C(0), then a barrier and one kernel per bucket.  Either way the
step returns with the caller's stream ordered after all of it.

The parameters are re-homed into one flat FP32 buffer (each becomes a view
of it) and their ``.grad`` into one flat gradient buffer, so the collectives
run on contiguous memory with no packing copies.  Each parameter starts on a
16-element boundary and each piece on a 64-element boundary, so every
segment of the step is 16-byte aligned.  The reference has no distributed
code; its docstrings only say that FP32 state keeps the payload under
DDP/FSDP local shards (remote/torch_fiber.py:3-6, 188-191) -- here the sign
fiber of a rank is the payload bit of its own pieces' second-moment words.
"""

from __future__ import annotations

from typing import Iterable

import torch
import torch.distributed as dist

from . import _lib, kernels
from .torch_fiber import _FORMATS, hyper_row

PARAM_ALIGN = 16   # elements (64 bytes)
PIECE_ALIGN = 64   # elements (256 bytes)
DEFAULT_BUCKET = 1 << 26  # elements per bucket (256 MB of FP32 parameters)
# Grid caps of the peer/nvls pipeline (see __init__): the fused kernel one
# CTA per tile; the compression beside it 3 CTAs per SM at 2 ranks, 4 beyond
# (sweep on B200 over 2^30 elements, ms per step at 2 ranks for caps
# 2/3/4/5/6/uncapped: 6.18/5.53/5.69/6.00/6.21/6.51; at 4 ranks for 3/4/
# uncapped: 7.72/7.43/8.78)
FUSED_CTAS_PER_SM = 0
COMPRESS_CTAS_PER_SM = {2: 3}
COMPRESS_CTAS_DEFAULT = 4
# Rank counts where fuse_compression is the default: over 2^30 elements it
# measured 5.32-5.34 ms per step at 2 ranks against 5.59 for the capped
# compression on a second stream (the launch after the barrier made no
# difference: 5.321 with, 5.326 without), and 7.37 against 7.47 at 4 ranks;
# not measured at 8 ranks.
FUSE_COMPRESSION_WORLDS = (2, 4)


class CudaKernels:
    """The product backend: libdfc_b200.so kernels on CUDA tensors.  Each
    bucket's descriptor array is built once (the buffers never move) and
    only its hyper-set column changes between steps."""

    def __init__(self):
        self._segs = {}
        self.compress_ctas = 0  # CTAs per SM of the compression grid (0: the whole SM)

    def compress_ef(self, grad, comp, resid):
        kernels.compress_ef(grad, comp, resid, self.compress_ctas)

    def step(self, segments, hyper_rows, hyper_index, mode, device, key=0):
        segs = self._segs.get(key)
        if segs is None:
            ps, gs, ms, vs = zip(*segments)
            segs = self._segs[key] = kernels.segments(ps, gs, ms, vs, hyper_index)
        segs["hyper"] = hyper_index
        kernels.mt_step_raw(segs, kernels.hypers(hyper_rows), mode, device)

    def convert(self, words, pack: bool, second: bool):
        (kernels.pack_moments if pack else kernels.unpack_moments)(words, second)

    def fiber_read(self, ranges, start_bit: int, n_bits: int, out: torch.Tensor):
        """Bits [start_bit, start_bit + n_bits) of the word ranges (NULL words:
        holes, read as zero) packed into the uint8 tensor out."""
        with torch.cuda.device(out.device):
            _lib.check("dfc_fiber_read", _lib.lib().dfc_fiber_read(
                _lib.ptr(ranges), len(ranges), start_bit, n_bits, out.data_ptr(),
                torch.cuda.current_stream(out.device).cuda_stream))

    def fiber_write(self, ranges, start_bit: int, n_bits: int, src: torch.Tensor):
        """Write bits of the uint8 tensor src into the ranges (holes skipped)."""
        with torch.cuda.device(src.device):
            _lib.check("dfc_fiber_write", _lib.lib().dfc_fiber_write(
                _lib.ptr(ranges), len(ranges), start_bit, n_bits, src.data_ptr(),
                torch.cuda.current_stream(src.device).cuda_stream))


class ShardedDFCAdamW(torch.optim.Optimizer):
    """ZeRO-1 DFC-AdamW.  Same hyperparameters as DFCAdamW; extra options:

    process_group   group to shard over (default: the world)
    moment_format   "packed" (default) or "fp32"
    compress_grads  bf16 + error-feedback compression before the
                    reduce-scatter (default: on when the group has > 1 rank)
    average_grads   divide the summed gradient by the group size (default on)
    bucket_elems    elements per pipelined bucket (rounded to N*64)
    transport       "nccl": NCCL reduce-scatter + step + NCCL all-gather;
                    "peer": one fused kernel over NVLink peer memory
                    (dfc_zero_fused_step) between two cross-GPU barriers;
                    needs symmetric memory and compressed gradients;
                    "nvls": the same kernel with the reduction and the
                    parameter broadcast done by the NVSwitch (multimem);
                    needs NVLink multicast;
                    "auto" (default): the measured fastest -- on B200 over a
                    2^30-element vector, ms per step (peer / nvls / nccl):
                    2 ranks 5.5 / 9.1 / 10.5; 4 ranks 7.4 / 8.1 / 11.2;
                    8 ranks 9.0 / 8.0 / 11.2.  So peer up to 4 ranks, nvls
                    beyond where the node has NVLink multicast, else peer
    fused_ctas_per_sm, compress_ctas_per_sm
                    grid caps of the peer/nvls pipeline (defaults measured;
                    compress_ctas_per_sm=0: the uncapped tile compression;
                    with fuse_compression only the fused cap applies)
    side_stream_priority
                    CUDA priority of the stream that runs the barriers and the
                    fused kernel (lower is higher; PyTorch clamps to the
                    device's range)
    overlap_buckets peer/nvls: alternate the fused kernels of neighbouring
                    buckets between two streams, so bucket b's broadcast
                    overlaps bucket b+1's reduction (the barriers stay in
                    order on every rank)
    fuse_compression
                    peer/nvls: compress bucket b+1 inside the grid of bucket
                    b's fused kernel (dfc_zero_fused_step_ef) instead of in a
                    capped kernel on a second stream; one stream, one kernel
                    and one barrier per bucket (default: on at 2 and 4
                    ranks, where it was measured faster; off otherwise)
    overlap_barrier with fuse_compression: launch each bucket's kernel as the
                    programmatic dependent of the barrier before it, so its
                    compression tiles run while the barrier waits (default on)
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], lr: float = 1e-3,
                 betas: tuple[float, float] = (0.9, 0.999), eps: float = 1e-8,
                 weight_decay: float = 0.0, enable_fiber: bool = True, *,
                 moment_format: str = "packed", process_group=None,
                 compress_grads: bool | None = None, average_grads: bool = True,
                 bucket_elems: int = DEFAULT_BUCKET, transport: str = "auto",
                 barrier_timeout_s: float = 30.0, backend=None,
                 fused_ctas_per_sm: int | None = None, compress_ctas_per_sm: int | None = None,
                 side_stream_priority: int = 0, overlap_buckets: bool = False,
                 fuse_compression: bool | None = None, overlap_barrier: bool = True):
        if lr < 0 or eps < 0 or not 0 <= betas[0] < 1 or not 0 <= betas[1] < 1:
            raise ValueError("invalid AdamW hyperparameters")
        if moment_format not in _FORMATS:
            raise ValueError(f"moment_format must be one of {_FORMATS}")
        if bucket_elems <= 0:
            raise ValueError("bucket_elems must be positive")
        super().__init__(params, dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay))
        self.enable_fiber = bool(enable_fiber)
        self.moment_format = moment_format
        self.group = process_group
        self.world = dist.get_world_size(process_group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(process_group) if dist.is_initialized() else 0
        self.compress = (self.world > 1) if compress_grads is None else bool(compress_grads)
        self.average = bool(average_grads)
        self.kernels = backend if backend is not None else CudaKernels()
        if transport not in ("auto", "nccl", "peer", "nvls"):
            raise ValueError("transport must be 'auto', 'nccl', 'peer' or 'nvls'")
        if transport == "auto":
            transport = self._auto_transport(backend)
        self.transport = transport if self.world > 1 else "nccl"
        if self.transport in ("peer", "nvls") and not self.compress:
            raise ValueError("the peer and nvls transports reduce bf16 compressed gradients")
        self.barrier_timeout_ns = int(barrier_timeout_s * 1e9)
        self.side_stream_priority = int(side_stream_priority)
        self.overlap_buckets = bool(overlap_buckets)
        if fuse_compression is None:
            fuse_compression = self.world in FUSE_COMPRESSION_WORLDS and not self.overlap_buckets
        self.fuse_compression = bool(fuse_compression)
        self.overlap_barrier = bool(overlap_barrier)
        if self.fuse_compression and self.overlap_buckets:
            raise ValueError("fuse_compression runs every bucket on one stream; "
                             "overlap_buckets does not apply")
        # Peer and nvls transports: the fused kernel of bucket b and the
        # compression of bucket b+1 run on two streams.  The compression grid
        # is capped so that the fused kernel finds room on every SM beside it;
        # uncapped, its full-SM persistent grid makes the fused kernel wait,
        # and the two run one after the other.  The fused kernel keeps one CTA
        # per tile, so it takes the whole SM once the compression is done
        # (a persistent fused grid of 2 or 3 CTAs per SM measured slower).
        fk = FUSED_CTAS_PER_SM
        ck = COMPRESS_CTAS_PER_SM.get(self.world, COMPRESS_CTAS_DEFAULT)
        self.fused_ctas = fk if fused_ctas_per_sm is None else int(fused_ctas_per_sm)
        compress_ctas = ck if compress_ctas_per_sm is None else int(compress_ctas_per_sm)
        if self.transport in ("peer", "nvls") and isinstance(self.kernels, CudaKernels):
            self.kernels.compress_ctas = compress_ctas
        self._layout(bucket_elems)
        if self.transport in ("peer", "nvls"):
            self._setup_peer()

    def _auto_transport(self, backend) -> str:
        """The measured fastest on B200 over a 2^30-element vector: the
        peer-memory kernel up to 4 ranks; beyond, the NVSwitch-multicast
        kernel where the node has NVLink multicast, else the peer kernel;
        NCCL for one rank, uncompressed gradients, a custom backend or
        non-CUDA parameters."""
        params = [p for g in self.param_groups for p in g["params"]]
        if self.world < 2 or not self.compress or backend is not None or \
                not all(p.is_cuda for p in params):
            return "nccl"
        if self.world <= 4:
            return "peer"
        from torch._C._autograd import DeviceType
        from torch._C._distributed_c10d import _SymmetricMemory

        try:
            multicast = _SymmetricMemory.has_multicast_support(DeviceType.CUDA,
                                                               params[0].device.index)
        except RuntimeError:  # no CUDA driver to ask
            multicast = False
        return "nvls" if multicast else "peer"

    # ---- layout -----------------------------------------------------------
    @torch.no_grad()
    def _layout(self, bucket_elems: int):
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
        offs, total = [], 0
        for p in self.params:
            offs.append(total)
            total += -(-p.numel() // PARAM_ALIGN) * PARAM_ALIGN
        n = self.world
        unit = n * PIECE_ALIGN
        whole = -(-total // unit) * unit
        bucket = min(max(unit, bucket_elems // unit * unit), whole)
        self.bucket = bucket
        self.piece = bucket // n
        self.n_buckets = -(-total // bucket)
        self.padded = self.n_buckets * bucket
        self.offsets = offs
        self.flat_param = self._alloc(self.padded, torch.float32)
        self.flat_grad = torch.zeros(self.padded, dtype=torch.float32, device=dev)
        for p, off in zip(self.params, offs):
            k = p.numel()
            self.flat_param[off:off + k].copy_(p.detach().reshape(-1))
            p.data = self.flat_param[off:off + k].view_as(p)
            p.grad = self.flat_grad[off:off + k].view_as(p)
        local = self.n_buckets * self.piece
        if self.compress:
            self.comp = self._alloc(self.padded, torch.int16)
            self.resid = torch.zeros(self.padded, dtype=torch.int16, device=dev)
            # one rank: the step reads the compressed gradients where they are
            self.shard_grad = self.comp.view(torch.bfloat16) if n == 1 else \
                torch.zeros(local, dtype=torch.bfloat16, device=dev)
        elif n > 1:
            self.shard_grad = torch.zeros(local, dtype=torch.float32, device=dev)
        else:
            self.shard_grad = self.flat_grad
        self.exp_avg = torch.zeros(local, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros(local, dtype=torch.float32, device=dev)
        # per bucket: the parameter slices that fall in this rank's piece
        self.bucket_segments, self.bucket_params = [], []
        for b in range(self.n_buckets):
            lo = b * bucket + self.rank * self.piece   # flat range this rank owns
            base = b * self.piece                      # where it lives locally
            segs, pidx = [], []
            for i, (p, off) in enumerate(zip(self.params, offs)):
                a, e = max(off, lo), min(off + p.numel(), lo + self.piece)
                if a >= e:
                    continue
                s = base + a - lo
                g = self.flat_grad[a:e] if self.shard_grad is self.flat_grad \
                    else self.shard_grad[s:s + e - a]
                segs.append((self.flat_param[a:e], g, self.exp_avg[s:s + e - a],
                             self.exp_avg_sq[s:s + e - a]))
                pidx.append(i)
            self.bucket_segments.append(segs)
            self.bucket_params.append(pidx)
        for p in self.params:
            self.state[p]["step"] = 0

    def _alloc(self, n: int, dtype) -> torch.Tensor:
        """Zeroed buffer; in symmetric (peer-mapped) memory for the peer transport."""
        if self.transport in ("peer", "nvls"):
            import torch.distributed._symmetric_memory as symm_mem

            t = symm_mem.empty(n, dtype=dtype, device=self.device)
            return t.zero_()
        return torch.zeros(n, dtype=dtype, device=self.device)

    @torch.no_grad()
    def _setup_peer(self):
        """Exchange the peer addresses of the parameters, compressed
        gradients and barrier slots (collective), and lay out this rank's
        pieces as fused-kernel segments."""
        import numpy as np
        import torch.distributed._symmetric_memory as symm_mem

        group = self.group if self.group is not None else dist.group.WORLD
        n = self.world

        def peers(t):
            h = symm_mem.rendezvous(t, group)
            ptrs = [int(p) for p in h.buffer_ptrs]
            off = t.data_ptr() - ptrs[self.rank]
            nbytes = t.numel() * t.element_size()
            # the tensor must lie inside this rank's buffer at the handle's
            # offset, so the same offset addresses every peer's copy
            if len(ptrs) != n or off < 0 or off + nbytes > int(h.buffer_size) or \
                    (hasattr(h, "offset") and int(h.offset) != off):
                raise RuntimeError("symmetric-memory layout is not the expected one")
            mc = None
            if self.transport == "nvls":
                from torch._C._distributed_c10d import _SymmetricMemory

                if not _SymmetricMemory.has_multicast_support(
                        torch._C._autograd.DeviceType.CUDA, self.device.index) or \
                        not int(h.multicast_ptr):
                    raise RuntimeError("NVLink multicast is not available on this node")
                mc = int(h.multicast_ptr) + off
            return [p + off for p in ptrs], h, mc

        self.slots = symm_mem.empty(n, dtype=torch.int32, device=self.device).zero_()
        self._param_peers, self._h_param, self._param_mc = peers(self.flat_param)
        self._comp_peers, self._h_comp, self._comp_mc = peers(self.comp)
        self._slot_peers, self._h_slots, _ = peers(self.slots)
        self.peer_error = torch.zeros(1, dtype=torch.int32, device=self.device)
        # the flag as of the end of the last step, copied to the host on the
        # side stream; read by the next step() without waiting
        self._peer_error_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._peer_error_copied = None
        self._epoch = 0
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._comp_arr = np.array(self._comp_peers, dtype=np.uint64)
        self._param_arr = np.array(self._param_peers, dtype=np.uint64)
        self._slot_arr = np.array(self._slot_peers, dtype=np.uint64)
        self._peer_segs = []
        for group_segs in self.bucket_segments:
            segs = [((p.data_ptr() - self.flat_param.data_ptr()) // 4, p.numel(), m.data_ptr(),
                     v.data_ptr(), 0, 0) for p, _, m, v in group_segs]
            self._peer_segs.append(np.array(segs, dtype=_lib.PEERSEG_DTYPE))
        self._side = torch.cuda.Stream(self.device, priority=self.side_stream_priority)
        self._sides = [self._side]
        # fuse_compression: bucket b's kernel compresses bucket b+1 (none after the last)
        self._next_comp = []
        for b in range(self.n_buckets):
            r = np.zeros(1, dtype=_lib.COMPRESSRANGE_DTYPE)
            if b + 1 < self.n_buckets:
                r[0] = (self._bucket(self.flat_grad, b + 1).data_ptr(),
                        self._bucket(self.comp, b + 1).data_ptr(),
                        self._bucket(self.resid, b + 1).data_ptr(), self.bucket)
            self._next_comp.append(r)
        if self.overlap_buckets:
            self._sides.append(torch.cuda.Stream(self.device, priority=self.side_stream_priority))

    def _barrier(self, stream):
        self._epoch += 1
        _lib.check("dfc_peer_barrier", _lib.lib().dfc_peer_barrier(
            _lib.ptr(self._slot_arr), self.world, self.rank, self._epoch & 0xFFFFFFFF,
            self.peer_error.data_ptr(), self.barrier_timeout_ns, stream))

    def _check_peer_error(self):
        """Raise if a barrier of an earlier step gave up.  The flag's copy
        of the last step is read only if it has already landed (no wait); a
        later step() or peer_status() sees a copy still in flight."""
        ev = self._peer_error_copied
        if ev is not None and ev.query():
            self._peer_error_copied = None
            code = int(self._peer_error_host[0])
            if code:
                raise RuntimeError(
                    f"ShardedDFCAdamW: a cross-GPU barrier gave up waiting for rank {code - 1} "
                    f"after {self.barrier_timeout_ns / 1e9:g} s; the steps since then did not "
                    f"update parameters or moments (restore a checkpoint)")

    def _step_peer(self, rows, index):
        """Bucket b: compress on the caller's stream; then, on a side stream
        that waits for it, a barrier (every rank's bucket-b gradients are
        complete) and the fused step of bucket b -- which runs while the
        caller's stream compresses bucket b+1.  A last barrier (every rank's
        parameters are complete) ends the step; the caller's stream waits
        for it.  A barrier that gives up sets peer_error; from then on every
        fused kernel and barrier of this rank returns at once, touching no
        memory, and the next step() raises."""
        self._check_peer_error()
        main = torch.cuda.current_stream(self.device)
        sides = self._sides
        hyp = kernels.hypers(rows)
        lib = _lib.lib()
        for side in sides:
            side.wait_stream(main)
        barrier_done = None  # with two side streams, each barrier waits for the previous one
        with torch.cuda.device(self.device):
            for b in range(self.n_buckets):
                self.kernels.compress_ef(self._bucket(self.flat_grad, b), self._bucket(self.comp, b),
                                         self._bucket(self.resid, b))
                side = sides[b % len(sides)]
                side.wait_stream(main)
                if barrier_done is not None:
                    side.wait_event(barrier_done)
                self._barrier(side.cuda_stream)
                if len(sides) > 1:
                    barrier_done = side.record_event()
                segs = self._peer_segs[b]
                if len(segs):
                    segs["hyper"] = index[b]
                    _lib.check("dfc_zero_fused_step", lib.dfc_zero_fused_step(
                        _lib.ptr(self._comp_arr), _lib.ptr(self._param_arr), self._comp_mc,
                        self._param_mc, self.world, self.rank, _lib.ptr(segs), len(segs),
                        _lib.ptr(hyp), len(rows), self.mode, None, self.peer_error.data_ptr(),
                        self.fused_ctas, side.cuda_stream))
            last = sides[0]
            for side in sides[1:]:
                last.wait_stream(side)
            self._barrier(last.cuda_stream)
            with torch.cuda.stream(last):
                self._peer_error_host.copy_(self.peer_error, non_blocking=True)
                self._peer_error_copied = last.record_event()
        main.wait_stream(last)

    def _step_peer_fused_compression(self, rows, index):
        """One stream: C(0) alone (full grid); then for every bucket b a
        barrier (every rank's C(b) done) and one kernel that steps bucket b
        and compresses bucket b+1 in the same grid (with overlap_barrier its
        compression tiles start while the barrier waits); a last barrier ends
        the step.  Error handling as in _step_peer (the compression tiles run
        regardless: they touch only this rank's gradient buffers)."""
        self._check_peer_error()
        main = torch.cuda.current_stream(self.device)
        side = self._sides[0]
        side.wait_stream(main)
        hyp = kernels.hypers(rows)
        lib = _lib.lib()
        with torch.cuda.device(self.device), torch.cuda.stream(side):
            kernels.compress_ef(self._bucket(self.flat_grad, 0), self._bucket(self.comp, 0),
                                self._bucket(self.resid, 0), 0)
            for b in range(self.n_buckets):
                self._barrier(side.cuda_stream)
                segs = self._peer_segs[b]
                if len(segs):
                    segs["hyper"] = index[b]
                _lib.check("dfc_zero_fused_step_ef", lib.dfc_zero_fused_step_ef(
                    _lib.ptr(self._comp_arr), _lib.ptr(self._param_arr), self._comp_mc,
                    self._param_mc, self.world, self.rank, _lib.ptr(segs) if len(segs) else None,
                    len(segs), _lib.ptr(hyp), len(rows), self.mode, None,
                    self.peer_error.data_ptr(), _lib.ptr(self._next_comp[b]),
                    _lib.FUSED_AFTER_BARRIER if self.overlap_barrier else 0, self.fused_ctas,
                    side.cuda_stream))
            self._barrier(side.cuda_stream)
            self._peer_error_host.copy_(self.peer_error, non_blocking=True)
            self._peer_error_copied = side.record_event()
        main.wait_stream(side)

    def peer_status(self) -> int:
        """0, or 1 + the rank a barrier gave up waiting for (synchronises)."""
        return int(self.peer_error.item()) if self.transport in ("peer", "nvls") else 0

    def _bucket(self, t: torch.Tensor, b: int) -> torch.Tensor:
        return t[b * self.bucket:(b + 1) * self.bucket]

    def _piece(self, t: torch.Tensor, b: int) -> torch.Tensor:
        """This rank's piece of bucket b inside a full-length flat tensor."""
        lo = b * self.bucket + self.rank * self.piece
        return t[lo:lo + self.piece]

    def _local(self, t: torch.Tensor, b: int) -> torch.Tensor:
        """Bucket b's slot in a local (per-rank) tensor."""
        return t[b * self.piece:(b + 1) * self.piece]

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
        """Second-moment words of this rank's pieces, one view per parameter
        slice (alignment padding excluded): this rank's sign fiber."""
        return [v for segs in self.bucket_segments for _, _, _, v in segs]

    @property
    def payload_bit_capacity(self) -> int:
        return sum(v.numel() for v in self.second_moment_tensors()) if self.enable_fiber else 0

    # ---- the global sign fiber across every rank's pieces --------------------
    # Global bit k is bit 31 of the second moment of element k of the
    # parameters taken in order (param_groups order, each parameter's elements
    # in order, alignment padding excluded): the bit the reference's channel
    # would address on one process holding every parameter
    # (remote/torch_fiber.py:120-185).  Under ZeRO-1 the bit lives on the rank
    # whose piece holds that element.
    def fiber_runs(self) -> list[tuple[int, int, int, int]]:
        """Every run of the global fiber, in global order: (first global bit,
        length, owning rank, index of the run's first word in the owner's
        exp_avg_sq).  A run is one parameter's slice inside one piece; the
        table is the same on every rank (it follows from the layout)."""
        runs, g = [], 0
        for p, off in zip(self.params, self.offsets):
            n, e = p.numel(), 0
            while e < n:
                b, pos = divmod(off + e, self.bucket)
                q, inside = divmod(pos, self.piece)
                take = min(n - e, self.piece - inside)
                runs.append((g + e, take, q, b * self.piece + inside))
                e += take
            g += n
        return runs

    def fiber_owner(self, bit: int) -> tuple[int, int]:
        """(rank, word index in that rank's exp_avg_sq) of global fiber bit."""
        import bisect

        runs = self._fiber_runs_cached()
        starts = [r[0] for r in runs]
        total = runs[-1][0] + runs[-1][1] if runs else 0
        if not 0 <= bit < total:
            raise IndexError("fiber bit out of bounds")
        g, _, q, w = runs[bisect.bisect_right(starts, bit) - 1]
        return q, w + (bit - g)

    def _fiber_runs_cached(self):
        runs = getattr(self, "_fiber_runs", None)
        if runs is None:
            runs = self._fiber_runs = self.fiber_runs()
        return runs

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
        scale = 1.0 / n if (self.average and n > 1) else 1.0
        steps = []
        for p in self.params:
            st = self.state[p]
            st["step"] += 1
            steps.append(st["step"])
        rows, seen = [], {}
        index = []
        for pidx in self.bucket_params:
            idx = []
            for pi in pidx:
                k = (self.group_of[pi], steps[pi])
                j = seen.get(k)
                if j is None:
                    g = self.param_groups[k[0]]
                    j = seen[k] = len(rows)
                    rows.append(hyper_row(g["lr"], g["betas"], g["eps"], g["weight_decay"], k[1],
                                          grad_scale=scale))
                idx.append(j)
            index.append(idx)

        if self.transport in ("peer", "nvls"):
            if self.fuse_compression:
                self._step_peer_fused_compression(rows, index)
            else:
                self._step_peer(rows, index)
            return loss

        def reduce(b):
            if self.compress:
                self.kernels.compress_ef(self._bucket(self.flat_grad, b),
                                         self._bucket(self.comp, b), self._bucket(self.resid, b))
                if n == 1:  # shard_grad is comp itself
                    return None
                src = self._bucket(self.comp, b).view(torch.bfloat16)
            elif n > 1:
                src = self._bucket(self.flat_grad, b)
            else:
                return None
            return dist.reduce_scatter_tensor(self._local(self.shard_grad, b), src,
                                              op=dist.ReduceOp.SUM, group=self.group, async_op=True)

        gathers = []
        pending = reduce(0)
        for b in range(self.n_buckets):
            nxt = reduce(b + 1) if b + 1 < self.n_buckets else None
            if pending is not None:
                pending.wait()
            if self.bucket_segments[b]:
                self.kernels.step(self.bucket_segments[b], rows, index[b], self.mode, self.device,
                                  key=b)
            if n > 1:
                gathers.append(dist.all_gather_into_tensor(
                    self._bucket(self.flat_param, b), self._piece(self.flat_param, b),
                    group=self.group, async_op=True))
            pending = nxt
        for w in gathers:
            w.wait()
        return loss

    def _check_grads(self):
        # the step reads the flat gradient buffer; a .grad rebound elsewhere
        # would be silently ignored, so refuse it
        for p, off in zip(self.params, self.offsets):
            g = p.grad
            if g is None or g.data_ptr() != self.flat_grad.data_ptr() + 4 * off:
                raise RuntimeError("ShardedDFCAdamW owns .grad of its parameters; use its "
                                   "zero_grad() (set_to_none is not supported)")

    @torch.no_grad()
    def full_reduced_grad(self) -> torch.Tensor:
        """The gradient the last step used, in flat order on every rank
        (collective; for checking and debugging)."""
        if self.transport == "nvls":
            # the switch's sums, read through the multicast address; the barrier
            # keeps every rank's gradients in place until all have read them
            out = torch.empty(self.padded, dtype=torch.float32, device=self.device)
            _lib.check("dfc_multicast_sum_bf16", _lib.lib().dfc_multicast_sum_bf16(
                self._comp_mc, out.data_ptr(), self.padded,
                torch.cuda.current_stream(self.device).cuda_stream))
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            return out
        if self.transport == "peer":
            # the fused kernel sums every rank's bf16 values in FP32, rank order
            allc = torch.empty(self.world * self.padded, dtype=torch.bfloat16, device=self.device)
            dist.all_gather_into_tensor(allc, self.comp.view(torch.bfloat16), group=self.group)
            parts = allc.view(self.world, self.padded).float()
            total = parts[0].clone()
            for q in range(1, self.world):
                total += parts[q]
            return total
        out = torch.empty(self.padded, dtype=self.shard_grad.dtype, device=self.device)
        if self.world == 1:
            return out.copy_(self.shard_grad[:self.padded])
        for b in range(self.n_buckets):
            dist.all_gather_into_tensor(self._bucket(out, b), self._local(self.shard_grad, b),
                                        group=self.group)
        return out

    # ---- checkpoints -------------------------------------------------------
    def _layout_info(self):
        return {"rank": self.rank, "world": self.world, "bucket": self.bucket,
                "padded": self.padded}

    def state_dict(self):
        """This rank's pieces (moment words, step counters, layout)."""
        return {
            "shard": {"exp_avg": self.exp_avg.clone(), "exp_avg_sq": self.exp_avg_sq.clone(),
                      **self._layout_info()},
            "steps": [self.state[p]["step"] for p in self.params],
            "param_groups": [{k: v for k, v in g.items() if k != "params"}
                             for g in self.param_groups],
            "moment_format": self.moment_format,
        }

    @torch.no_grad()
    def load_state_dict(self, state_dict):
        sh = state_dict["shard"]
        if any(sh[k] != v for k, v in self._layout_info().items()):
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
        rank.  Collective: every rank must call it.  Returns the dict on
        ``to_rank`` (every rank when None), else None."""
        full_m = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        full_v = torch.empty(self.padded, dtype=torch.float32, device=self.device)
        for b in range(self.n_buckets):
            if self.world > 1:
                dist.all_gather_into_tensor(self._bucket(full_m, b), self._local(self.exp_avg, b),
                                            group=self.group)
                dist.all_gather_into_tensor(self._bucket(full_v, b),
                                            self._local(self.exp_avg_sq, b), group=self.group)
            else:
                self._bucket(full_m, b).copy_(self._local(self.exp_avg, b))
                self._bucket(full_v, b).copy_(self._local(self.exp_avg_sq, b))
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
        DFCAdamW's, or the reference's) and keep this rank's pieces."""
        st = state_dict["state"]
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
        for b in range(self.n_buckets):
            self._local(self.exp_avg, b).copy_(self._piece(flat_m, b))
            self._local(self.exp_avg_sq, b).copy_(self._piece(flat_v, b))
        for g, saved in zip(self.param_groups, state_dict["param_groups"]):
            g.update({k: v for k, v in saved.items() if k != "params"})
        self._convert_from(state_dict.get("moment_format", "fp32"))


class ShardedSignFiberChannel:
    """The sign fiber of a ShardedDFCAdamW as ONE channel over the whole
    parameter set, with the interface of TorchSignFiberChannel
    (remote/torch_fiber.py:120-185): global bit k is the payload bit of
    element k of the parameters in order (see ShardedDFCAdamW.fiber_runs),
    whichever rank holds it.

    Every call is collective: every rank of the optimizer's group calls it
    with the same arguments (and, for writes, the same payload).  A read runs
    the fiber kernel once per rank over the global window -- the other ranks'
    runs are holes that read as zero -- and a byte-wise sum over the ranks
    (each bit comes from exactly one rank, so the sum is their OR) gives every
    rank the same bytes.  A write runs the kernel once per rank, each storing
    only its own bits.  For the rank's own bits alone, without a collective,
    use TorchSignFiberChannel on the optimizer (its local fiber)."""

    def __init__(self, optimizer):
        if not optimizer.enable_fiber:
            raise ValueError("optimizer fiber is disabled")
        import numpy as np

        self.optimizer = optimizer
        runs = optimizer._fiber_runs_cached()
        self._ranges = np.zeros(len(runs), dtype=_lib.WORDRANGE_DTYPE)
        base = optimizer.exp_avg_sq.data_ptr()
        for i, (_, n, q, w) in enumerate(runs):
            self._ranges[i] = (base + 4 * w if q == optimizer.rank else 0, n)
        self._bits = sum(n for _, n, _, _ in runs)
        self.device = optimizer.exp_avg_sq.device

    @property
    def bit_capacity(self) -> int:
        return self._bits

    @property
    def byte_capacity(self) -> int:
        return self._bits // 8

    def owner(self, bit: int) -> tuple[int, int]:
        """(rank, word index in that rank's second-moment shard) of a global bit."""
        return self.optimizer.fiber_owner(bit)

    def _check(self, start: int, count: int) -> None:
        if start < 0 or count < 0 or start + count > self._bits:
            raise IndexError("fiber range out of bounds")

    def _read_dev(self, start: int, count: int) -> torch.Tensor:
        out = torch.zeros((count + 7) // 8, dtype=torch.uint8, device=self.device)
        if count:
            self.optimizer.kernels.fiber_read(self._ranges, start, count, out)
        if self.optimizer.world > 1:
            dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.optimizer.group)
        return out

    def _write_dev(self, start: int, count: int, src: torch.Tensor) -> None:
        if count:
            src = src.to(device=self.device, dtype=torch.uint8).contiguous()
            self.optimizer.kernels.fiber_write(self._ranges, start, count, src)

    @torch.no_grad()
    def read_bits(self, start: int, count: int):
        import numpy as np

        self._check(start, count)
        packed = self._read_dev(int(start), int(count)).cpu().numpy()
        return np.unpackbits(packed, bitorder="little")[:count] if count else packed

    @torch.no_grad()
    def write_bits(self, start: int, payload) -> None:
        import numpy as np

        bits = np.ascontiguousarray(payload, dtype=np.uint8).reshape(-1)
        if np.any(bits > 1):
            raise ValueError("payload must be binary")
        self._check(start, bits.size)
        self._write_dev(int(start), bits.size,
                        torch.from_numpy(np.packbits(bits, bitorder="little")))

    def read_bytes(self, start: int, count: int) -> bytes:
        if start < 0 or count < 0 or start + count > self.byte_capacity:
            raise IndexError("fiber byte range out of bounds")
        return self._read_dev(int(start) * 8, int(count) * 8).cpu().numpy().tobytes()

    def write_bytes(self, start: int, payload) -> None:
        import numpy as np

        raw = bytes(payload)
        if start < 0 or start + len(raw) > self.byte_capacity:
            raise IndexError("fiber byte range out of bounds")
        self._write_dev(int(start) * 8, len(raw) * 8,
                        torch.from_numpy(np.frombuffer(raw, dtype=np.uint8).copy()))

