"""A cross-GPU barrier that gives up, and what the fused ZeRO-1 step does then.

dfc_peer_barrier waits for every peer's epoch for at most its time limit;
on time-out it sets an error flag.  From then on dfc_zero_fused_step (given
the flag) and every later barrier return at once, touching no memory, so a
stalled or departed peer's gradients are never read and its parameter copy
is never written, and this rank's parameters and moments stay as they were.

The one-GPU test makes the wait run out on purpose: the barrier's second
"rank" is a signal array in this GPU's own memory that nothing writes, with
a 2 ms limit; every buffer is local, every access in bounds.  The two-GPU
test lets rank 0 step alone through ShardedDFCAdamW and checks that its next
step() raises and that no parameter changed on either rank.
"""

import ctypes
import os
import socket
import time
import traceback

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

N = 6144 + 5  # three 2048-element tiles and a ragged tail


def _ptrs(*ts):
    return (ctypes.c_uint64 * len(ts))(*[t.data_ptr() for t in ts])


def _fused(lib, comps, params, m, v, hyp, error, stream):
    from t3st_b200 import _lib

    segs = np.zeros(1, dtype=_lib.PEERSEG_DTYPE)
    segs[0] = (0, N, m.data_ptr(), v.data_ptr(), 0, 0)
    _lib.check("dfc_zero_fused_step", lib.dfc_zero_fused_step(
        _ptrs(*comps), _ptrs(*params), None, None, 2, 0, _lib.ptr(segs), 1, _lib.ptr(hyp), 1,
        _lib.MODE_PACKED, None, None if error is None else error.data_ptr(), 0, stream))


def test_barrier_timeout_stops_the_fused_step(cuda):
    from t3st_b200 import _lib, kernels
    from t3st_b200.torch_fiber import hyper_row

    lib = _lib.lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    g = torch.Generator(device=cuda).manual_seed(7)
    comps = [(torch.randn(N, generator=g, device=cuda) * 1e-3).to(torch.bfloat16).view(torch.int16)
             for _ in range(2)]
    p0 = torch.randn(N, generator=g, device=cuda) * 0.02
    params = [p0.clone(), p0.clone()]
    m = torch.zeros(N, dtype=torch.int32, device=cuda)
    v = torch.zeros(N, dtype=torch.int32, device=cuda)
    hyp = kernels.hypers([hyper_row(1e-3, (0.9, 0.999), 1e-8, 0.01, 1, grad_scale=0.5)])

    # rank 0 of two; "rank 1"'s signal array is local memory nothing writes
    mine = torch.zeros(2, dtype=torch.int32, device=cuda)
    phantom = torch.zeros(2, dtype=torch.int32, device=cuda)
    error = torch.zeros(1, dtype=torch.int32, device=cuda)
    t0 = time.perf_counter()
    _lib.check("dfc_peer_barrier", lib.dfc_peer_barrier(
        _ptrs(mine, phantom), 2, 0, 1, error.data_ptr(), 2_000_000, stream))
    _fused(lib, comps, params, m, v, hyp, error, stream)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 5.0
    assert int(error.item()) == 2                    # gave up waiting for rank 1
    assert int(phantom[0].item()) == 1               # its own epoch reached the peer's array
    for p in params:                                 # nothing read, nothing written
        assert torch.equal(p.view(torch.int32), p0.view(torch.int32))
    assert int(m.abs().sum()) == 0 and int(v.abs().sum()) == 0

    # a later barrier with the flag set signals nobody and waits for nothing
    t0 = time.perf_counter()
    _lib.check("dfc_peer_barrier", lib.dfc_peer_barrier(
        _ptrs(mine, phantom), 2, 0, 2, error.data_ptr(), 10_000_000_000, stream))
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 1.0
    assert int(phantom[0].item()) == 1 and int(error.item()) == 2

    # control: with a clear flag the same call steps, bit-exact against the
    # oracle given g = comp_0 + comp_1 (FP32, rank order), into both copies
    clear = torch.zeros(1, dtype=torch.int32, device=cuda)
    _fused(lib, comps, params, m, v, hyp, clear, stream)
    torch.cuda.synchronize()
    c = [x.view(torch.bfloat16).float().cpu().numpy() for x in comps]
    gsum = (c[0] + c[1]).astype(np.float32)
    sim_p = p0.cpu().numpy().copy()
    sim_m = np.zeros(N, np.uint32)
    sim_v = np.zeros(N, np.uint32)
    O.step(O.MODE_PACKED, O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.01, 1, grad_scale=0.5),
           sim_p, gsum, sim_m, sim_v)
    for p in params:
        np.testing.assert_array_equal(p.cpu().numpy().view(np.uint32), sim_p.view(np.uint32))
    np.testing.assert_array_equal(m.cpu().numpy().view(np.uint32), sim_m)
    np.testing.assert_array_equal(v.cpu().numpy().view(np.uint32), sim_v)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _lonely_worker(rank, world, port, q):
    """Both ranks step once; then rank 0 steps alone (rank 1 sleeps between
    steps, none of its kernels in flight)."""
    try:
        import datetime

        import torch.distributed as dist

        from t3st_b200.zero import ShardedDFCAdamW

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        torch.manual_seed(0)
        params = [torch.nn.Parameter((torch.randn(s) * 0.02).to(dev)) for s in [(4099,), (257, 31)]]
        opt = ShardedDFCAdamW(params, lr=1e-3, moment_format="packed", bucket_elems=4096,
                              transport="peer", barrier_timeout_s=2.0)
        for p in params:
            p.grad.normal_(0.0, 1e-3)
        opt.step()
        torch.cuda.synchronize()
        assert opt.peer_status() == 0
        before = [p.detach().clone() for p in params]
        m0, v0 = opt.exp_avg.clone(), opt.exp_avg_sq.clone()
        dist.barrier()
        if rank == 0:
            opt.step()                       # rank 1 never arrives
            torch.cuda.synchronize()
            assert opt.peer_status() == 2
            with pytest.raises(RuntimeError, match="gave up waiting for rank 1"):
                opt.step()
        else:
            time.sleep(6.0)
        torch.cuda.synchronize()
        for p, b in zip(params, before):
            assert torch.equal(p.detach().view(torch.int32), b.view(torch.int32))
        assert torch.equal(opt.exp_avg.view(torch.int32), m0.view(torch.int32))
        assert torch.equal(opt.exp_avg_sq.view(torch.int32), v0.view(torch.int32))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException:
        q.put((rank, traceback.format_exc()))


def test_sharded_step_raises_after_a_peer_times_out():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lonely_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert results[r] == "ok", results[r]
