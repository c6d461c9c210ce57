"""ZeRO-1 host logic on CPU gloo ranks (world 2, 4 and 8): flat layout, shard
segments, compression + reduce-scatter + step + all-gather wiring, hyper
sets, consolidated checkpoints, the per-rank sign fiber, and failure
behaviour.  The CUDA kernels are replaced by an oracle-backed backend (test
infrastructure; the product has no CPU path)."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


class OracleBackend:
    """Stand-in for t3st_b200.zero.CudaKernels on CPU tensors."""

    def compress_ef(self, g, c, q):
        O.compress_ef(g.numpy(), c.numpy().view(np.uint16), q.numpy().view(np.uint16))

    def step(self, segments, rows, index, mode, device, key=0):
        for (p, g, m, v), j in zip(segments, index):
            h = O.Hyper(*rows[j][:9])
            gg = g.view(torch.int16).numpy().view(np.uint16) if g.dtype == torch.bfloat16 else g.numpy()
            O.step(mode, h, p.numpy(), gg, m.numpy().view(np.uint32), v.numpy().view(np.uint32))

    # the fiber kernels' contract (include/dfc_b200.h): the concatenated
    # ranges' bit 31, NULL words = a hole (zero on a read, left alone on a write)
    @staticmethod
    def _words(ptr, n):
        import ctypes

        return np.ctypeslib.as_array((ctypes.c_uint32 * n).from_address(int(ptr)))

    def fiber_read(self, ranges, start, count, out):
        bits = np.concatenate([(self._words(w, n) >> 31).astype(np.uint8) if w else
                               np.zeros(n, np.uint8) for w, n in ranges])
        out.numpy()[:] = np.packbits(bits[start:start + count], bitorder="little")

    def fiber_write(self, ranges, start, count, src):
        bits = np.unpackbits(src.numpy(), bitorder="little")[:count].astype(np.uint32)
        pos = 0
        for w, n in ranges:
            lo, hi = max(pos, start), min(pos + n, start + count)
            if w and lo < hi:
                words = self._words(w, n)
                sl = slice(lo - pos, hi - pos)
                words[sl] = (words[sl] & 0x7FFFFFFF) | (bits[lo - start:hi - start] << 31)
            pos += n

    def convert(self, words, pack, second):
        w = words.numpy().view(np.uint32)
        if second:
            w[:] = O.pack_second(w) if pack else O.unpack_second(w)
        else:
            w[:] = O.pack_first(w.view(np.float32)) if pack else O.unpack_first(w).view(np.uint32)


SHAPES = [(33, 17), (17,), (1000,), (5,), (3, 3, 3)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _grads(rank, step, sizes):
    rng = np.random.default_rng(1000 * step + rank)
    return [(rng.standard_normal(n) * 1e-3).astype(np.float32) for n in sizes]


def _worker(rank, world, port, fmt, result_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from t3st_b200.zero import ShardedDFCAdamW

        torch.manual_seed(0)
        params = [torch.nn.Parameter(torch.randn(s) * 0.02) for s in SHAPES]
        p0 = [p.detach().numpy().reshape(-1).copy() for p in params]
        groups = [{"params": params[:3]}, {"params": params[3:], "lr": 3e-4, "weight_decay": 0.0}]
        opt = ShardedDFCAdamW(groups, lr=1e-3, weight_decay=0.01, moment_format=fmt,
                              backend=OracleBackend(), bucket_elems=256)
        assert opt.n_buckets >= 4
        sizes = [p.numel() for p in params]
        # payload in this rank's fiber (the shard's real coordinates)
        prng = np.random.default_rng(rank)
        payload = []
        for w in opt.second_moment_tensors():
            bits = torch.from_numpy(prng.integers(0, 2, w.numel()).astype(np.int32))
            wi = w.view(torch.int32)
            wi.copy_((wi & 0x7FFFFFFF) | (bits << 31))
            payload.append(bits)
        assert opt.payload_bit_capacity == sum(b.numel() for b in payload)

        # simulation state (every rank simulates the whole job)
        sim_p = [x.copy() for x in p0]
        sim_m = [np.zeros(n, np.uint32) for n in sizes]
        sim_v = [np.zeros(n, np.uint32) for n in sizes]
        ef_c = [np.zeros(opt.padded, np.uint16) for _ in range(world)]
        ef_q = [np.zeros(opt.padded, np.uint16) for _ in range(world)]
        mode = O.MODE_PACKED if fmt == "packed" else O.MODE_SIGNFIBER
        for step in range(1, 5):
            opt.zero_grad()
            for p, g in zip(params, _grads(rank, step, sizes)):
                p.grad.copy_(torch.from_numpy(g).view_as(p))
            opt.step()
            # gather the reduced gradient the step used, from every shard
            red = opt.full_reduced_grad()
            red16 = red.view(torch.int16).numpy().view(np.uint16).copy()
            exact = np.zeros(opt.padded, np.float64)
            mag = np.zeros(opt.padded, np.float64)
            for r in range(world):
                flat = np.zeros(opt.padded, np.float32)
                for off, g in zip(opt.offsets, _grads(r, step, sizes)):
                    flat[off:off + g.size] = g
                O.compress_ef(flat, ef_c[r], ef_q[r])
                cr = (ef_c[r].astype(np.uint32) << 16).view(np.float32).astype(np.float64)
                exact += cr
                mag += np.abs(cr)
            got = (red16.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
            # the collective sums in bf16: each of the world-1 additions rounds
            assert np.all(np.abs(got - exact) <= mag * 2.0 ** -8 * world + 1e-30)
            for i, off in enumerate(opt.offsets):
                gi = 0 if i < 3 else 1
                lr, wd = (1e-3, 0.01) if gi == 0 else (3e-4, 0.0)
                h = O.reference_hyper(lr, (0.9, 0.999), 1e-8, wd, step, grad_scale=1.0 / world)
                O.step(mode, h, sim_p[i], red16[off:off + sizes[i]].copy(), sim_m[i], sim_v[i])
            for i, p in enumerate(params):
                np.testing.assert_array_equal(p.detach().numpy().reshape(-1).view(np.uint32),
                                              sim_p[i].view(np.uint32))
        # payload kept
        for w, bits in zip(opt.second_moment_tensors(), payload):
            assert torch.equal((w.view(torch.int32) >> 31) & 1, bits)
        # consolidated moments equal the simulation (payload bits aside)
        full = opt.consolidated_state_dict(to_rank=None)
        for i in range(len(params)):
            st = full["state"][i]
            assert st["step"] == 4
            np.testing.assert_array_equal(st["exp_avg"].numpy().reshape(-1).view(np.uint32), sim_m[i])
            got_v = st["exp_avg_sq"].numpy().reshape(-1).view(np.uint32)
            np.testing.assert_array_equal(got_v & 0x7FFFFFFF, sim_v[i] & 0x7FFFFFFF)
        # round trip through a fresh optimizer, including a format change
        params2 = [torch.nn.Parameter(p.detach().clone()) for p in params]
        other = "fp32" if fmt == "packed" else "packed"
        opt2 = ShardedDFCAdamW(params2, moment_format=other, backend=OracleBackend(),
                               bucket_elems=4096)
        opt2.load_consolidated_state_dict(full)
        back = opt2.consolidated_state_dict(to_rank=None)
        opt3 = ShardedDFCAdamW([torch.nn.Parameter(p.detach().clone()) for p in params],
                               moment_format=fmt, backend=OracleBackend(), bucket_elems=256)
        opt3.load_consolidated_state_dict(back)
        assert torch.equal(opt3.exp_avg.view(torch.int32), opt.exp_avg.view(torch.int32))
        assert torch.equal(opt3.exp_avg_sq.view(torch.int32), opt.exp_avg_sq.view(torch.int32))
        # shard-local checkpoint
        opt3.load_state_dict(opt.state_dict())
        # .grad rebinding is refused
        params[0].grad = torch.zeros_like(params[0])
        with pytest.raises(RuntimeError, match="owns .grad"):
            opt.step()
        dist.barrier()
        dist.destroy_process_group()
        result_q.put((rank, "ok"))
    except BaseException:
        result_q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world,fmt", [(2, "packed"), (2, "fp32"), (4, "packed"), (8, "packed")])
def test_zero1_matches_simulation(world, fmt):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fmt, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert results[r] == "ok", results[r]


def _dying_worker(rank, world, port, result_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=3))
        from t3st_b200.zero import ShardedDFCAdamW

        params = [torch.nn.Parameter(torch.zeros(100))]
        opt = ShardedDFCAdamW(params, backend=OracleBackend())
        if rank == 1:
            result_q.put((rank, "left"))
            result_q.close()
            result_q.join_thread()
            os._exit(0)  # leaves between steps, no collective in flight
        try:
            opt.step()
            result_q.put((rank, "no error"))
        except RuntimeError as e:
            result_q.put((rank, "error: " + str(e)[:60]))
    except BaseException:
        result_q.put((rank, traceback.format_exc()))


def _fiber_worker(rank, world, port, result_q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime

        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        from t3st_b200.zero import ShardedDFCAdamW, ShardedSignFiberChannel

        torch.manual_seed(0)
        params = [torch.nn.Parameter(torch.randn(s) * 0.02) for s in SHAPES]
        opt = ShardedDFCAdamW(params, lr=1e-3, backend=OracleBackend(), bucket_elems=256)
        sizes = [p.numel() for p in params]
        total = sum(sizes)
        # the run table against a per-element walk of the layout
        runs = opt.fiber_runs()
        assert runs[0][0] == 0 and sum(r[1] for r in runs) == total
        assert all(a[0] + a[1] == b[0] for a, b in zip(runs, runs[1:]))
        g = 0
        for p, off in zip(params, opt.offsets):
            for e in range(0, p.numel(), 7):
                flat = off + e
                b, pos = divmod(flat, opt.bucket)
                want = (pos // opt.piece, b * opt.piece + pos % opt.piece)
                assert opt.fiber_owner(g + e) == want, (g + e, want)
            g += p.numel()
        local = opt.exp_avg_sq.numel()
        assert all(0 <= w and w + n <= local for _, n, q, w in runs if q == rank)
        # collective write, then collective reads, through the global channel
        ch = ShardedSignFiberChannel(opt)
        assert ch.bit_capacity == total
        rng = np.random.default_rng(5)  # the same payload on every rank
        bits = rng.integers(0, 2, total).astype(np.uint8)
        ch.write_bits(0, bits)
        mine = opt.exp_avg_sq.view(torch.int32).numpy().view(np.uint32) >> 31
        for gk, n, q, w in runs:
            if q == rank:
                np.testing.assert_array_equal(mine[w:w + n], bits[gk:gk + n])
        np.testing.assert_array_equal(ch.read_bits(0, total), bits)
        np.testing.assert_array_equal(ch.read_bits(13, 1001), bits[13:1014])
        payload = rng.bytes(ch.byte_capacity - 3)
        ch.write_bytes(3, payload)
        assert ch.read_bytes(3, len(payload)) == payload
        with pytest.raises(IndexError):
            ch.read_bits(total - 2, 3)
        dist.barrier()
        dist.destroy_process_group()
        result_q.put((rank, "ok"))
    except BaseException:
        result_q.put((rank, traceback.format_exc()))


@pytest.mark.parametrize("world", [2, 4])
def test_global_fiber_across_shards(world):
    """Global fiber bit -> (rank, word) mapping and the collective channel
    over every rank's pieces, on gloo ranks with the oracle backend."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fiber_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=180) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert res[r] == "ok", res[r]


def test_lost_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error"), results[0]


def test_auto_transport_choice():
    """The automatic transport: NCCL for one rank, uncompressed gradients,
    a custom backend or CPU tensors; the peer kernel up to 4 ranks; beyond,
    the multicast kernel only where the node reports NVLink multicast (never
    on a machine without a CUDA driver), else the peer kernel."""
    import types

    from t3st_b200.zero import ShardedDFCAdamW

    class FakeParam:
        is_cuda = True
        device = types.SimpleNamespace(index=0)

    def choose(world, compress=True, backend=None, cuda=True):
        stub = types.SimpleNamespace(world=world, compress=compress,
                                     param_groups=[{"params": [FakeParam() if cuda else
                                                               torch.zeros(1)]}])
        return ShardedDFCAdamW._auto_transport(stub, backend)

    assert choose(1) == "nccl"
    assert choose(2) == "peer"
    assert choose(4) == "peer"
    assert choose(2, compress=False) == "nccl"
    assert choose(2, backend=object()) == "nccl"
    assert choose(4, cuda=False) == "nccl"
    if not torch.cuda.is_available():
        assert choose(8) == "peer"


def test_fused_compression_excludes_bucket_overlap():
    """fuse_compression runs every bucket on one stream, so asking for the
    two-stream bucket overlap as well is refused at construction."""
    from t3st_b200.zero import ShardedDFCAdamW

    with pytest.raises(ValueError, match="overlap_buckets"):
        ShardedDFCAdamW([torch.nn.Parameter(torch.zeros(8))], fuse_compression=True,
                        overlap_buckets=True)
    opt = ShardedDFCAdamW([torch.nn.Parameter(torch.zeros(8))], fuse_compression=True)
    assert opt.fuse_compression and opt.transport == "nccl"  # one rank: nothing to fuse into
    assert not ShardedDFCAdamW([torch.nn.Parameter(torch.zeros(8))]).fuse_compression
