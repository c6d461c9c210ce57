"""ZeRO-1 ShardedDFCAdamW on CUDA: one GPU (no collective), and two GPUs
over NCCL, NVLink peer memory or NVSwitch multicast when the machine has
them (the reduced gradient is read back from every shard and the step is
checked bit for bit against the oracle given that reduced gradient)."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

SHAPES = [(257, 31), (31,), (4099,), (3, 3, 3), (1 << 16,)]
# a piece of ~1M elements per rank at two ranks: 513 tiles of 2048, so with
# one fused CTA per SM each CTA walks several tiles
SHAPES_LARGE = [(1 << 21,), (3001,), (257, 31)]


def _grads(rank, step, sizes):
    rng = np.random.default_rng(1000 * step + rank)
    return [(rng.standard_normal(n) * 1e-3).astype(np.float32) for n in sizes]


def _bf16_bracket(x):
    """The two bf16 values next to each float64 x (equal when x is one)."""
    _, e = np.frexp(x)
    ulp = np.ldexp(1.0, np.maximum(e, -125) - 8)
    lo = np.floor(x / ulp) * ulp
    return lo, np.where(lo == x, lo, lo + ulp)


def _check_switch_sums(opt, red, world):
    """The switch's sums are a faithful bf16 rounding of the exact sum of
    every rank's bf16 values (the neighbour below or above it)."""
    import torch.distributed as dist

    allc = torch.empty(world * opt.padded, dtype=torch.bfloat16, device=opt.device)
    dist.all_gather_into_tensor(allc, opt.comp.view(torch.bfloat16))
    exact = allc.view(world, opt.padded).double().sum(0).cpu().numpy()
    lo, hi = _bf16_bracket(exact)
    got = red.double().cpu().numpy()
    bad = np.flatnonzero((got != lo) & (got != hi))
    assert bad.size == 0, (bad[:8], got[bad[:8]], exact[bad[:8]])


def _run(rank, world, device, compress, transport="nccl", shapes=SHAPES, bucket=8192,
         fused_ctas=None, overlap=False, fuse=None):
    from t3st_b200.zero import ShardedDFCAdamW

    torch.manual_seed(0)
    params = [torch.nn.Parameter((torch.randn(s) * 0.02).to(device)) for s in shapes]
    sizes = [p.numel() for p in params]
    p0 = [p.detach().cpu().numpy().reshape(-1).copy() for p in params]
    opt = ShardedDFCAdamW(params, lr=1e-3, weight_decay=0.01, moment_format="packed",
                          compress_grads=compress, bucket_elems=bucket, transport=transport,
                          fused_ctas_per_sm=fused_ctas, overlap_buckets=overlap,
                          fuse_compression=fuse)
    sim_p = [x.copy() for x in p0]
    sim_m = [np.zeros(n, np.uint32) for n in sizes]
    sim_v = [np.zeros(n, np.uint32) for n in sizes]
    ef_c = [np.zeros(opt.padded, np.uint16) for _ in range(world)]
    ef_q = [np.zeros(opt.padded, np.uint16) for _ in range(world)]
    for step in range(1, 6):
        opt.zero_grad()
        for p, g in zip(params, _grads(rank, step, sizes)):
            p.grad.copy_(torch.from_numpy(g).view_as(p))
        opt.step()
        torch.cuda.synchronize()
        if world > 1:
            red = opt.full_reduced_grad()
            if transport == "nvls":
                _check_switch_sums(opt, red, world)
            if red.dtype == torch.bfloat16:  # NCCL's bf16 sum
                red = red.view(torch.int16).cpu().numpy().view(np.uint16)
            else:  # the fused kernel's FP32 sum in rank order (nvls: rounded to bf16)
                red = red.cpu().numpy()
            gsrc = [red[off:off + n].copy() for off, n in zip(opt.offsets, sizes)]
            scale = 1.0 / world
        elif compress:
            flat = np.zeros(opt.padded, np.float32)
            for off, g in zip(opt.offsets, _grads(rank, step, sizes)):
                flat[off:off + g.size] = g
            O.compress_ef(flat, ef_c[0], ef_q[0])
            gsrc = [ef_c[0][off:off + n].copy() for off, n in zip(opt.offsets, sizes)]
            scale = 1.0
        else:
            gsrc = _grads(rank, step, sizes)
            scale = 1.0
        h = O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.01, step, grad_scale=scale)
        for i in range(len(sizes)):
            O.step(O.MODE_PACKED, h, sim_p[i], gsrc[i], sim_m[i], sim_v[i])
        for i, p in enumerate(params):
            np.testing.assert_array_equal(p.detach().cpu().numpy().reshape(-1).view(np.uint32),
                                          sim_p[i].view(np.uint32))
    assert opt.peer_status() == 0
    full = opt.consolidated_state_dict(to_rank=None)
    for i in range(len(sizes)):
        np.testing.assert_array_equal(full["state"][i]["exp_avg"].cpu().numpy().reshape(-1).view(np.uint32), sim_m[i])
        np.testing.assert_array_equal(full["state"][i]["exp_avg_sq"].cpu().numpy().reshape(-1).view(np.uint32), sim_v[i])
    return opt, params


@pytest.mark.parametrize("compress", [False, True])
def test_sharded_on_one_gpu_matches_oracle(cuda, compress):
    opt, params = _run(0, 1, cuda, compress)
    # the consolidated state loads into the single-GPU DFCAdamW
    from t3st_b200 import DFCAdamW

    single = DFCAdamW(params, lr=1e-3, weight_decay=0.01, moment_format="packed")
    single.load_state_dict(opt.consolidated_state_dict())
    for i, p in enumerate(params):
        assert single.state[p]["step"] == 5
        full = opt.consolidated_state_dict()["state"][i]["exp_avg"]
        assert torch.equal(single.state[p]["exp_avg"].view(torch.int32), full.view(torch.int32))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _fiber_check(rank, world, device):
    """The global sign fiber across the ranks' shards (real kernels, NCCL
    sum of the ranks' reads): a payload written by every rank lands in the
    owning ranks' words and reads back whole on every rank."""
    from t3st_b200.zero import ShardedDFCAdamW, ShardedSignFiberChannel

    torch.manual_seed(0)
    params = [torch.nn.Parameter((torch.randn(s) * 0.02).to(device)) for s in SHAPES]
    opt = ShardedDFCAdamW(params, lr=1e-3, moment_format="packed", bucket_elems=8192,
                          transport="nccl")
    ch = ShardedSignFiberChannel(opt)
    total = sum(p.numel() for p in params)
    assert ch.bit_capacity == total
    rng = np.random.default_rng(9)
    bits = rng.integers(0, 2, total).astype(np.uint8)
    ch.write_bits(0, bits)
    torch.cuda.synchronize()
    mine = opt.exp_avg_sq.view(torch.int32).cpu().numpy().view(np.uint32) >> 31
    for g, n, q, w in opt.fiber_runs():
        if q == rank:
            np.testing.assert_array_equal(mine[w:w + n], bits[g:g + n])
    np.testing.assert_array_equal(ch.read_bits(0, total), bits)
    payload = rng.bytes(ch.byte_capacity - 11)
    ch.write_bytes(11, payload)
    assert ch.read_bytes(11, len(payload)) == payload
    # the payload survives a step (bit 31 of the second moment is kept)
    for p in params:
        p.grad.normal_(0.0, 1e-3)
    opt.step()
    assert ch.read_bytes(11, len(payload)) == payload


def _worker(rank, world, port, transport, q, kw):
    try:
        import datetime

        import torch.distributed as dist

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        if transport == "fiber":
            _fiber_check(rank, world, dev)
        else:
            _run(rank, world, dev, True, transport, **kw)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except BaseException:
        q.put((rank, traceback.format_exc()))


def _multicast_ok() -> bool:
    from torch._C._autograd import DeviceType
    from torch._C._distributed_c10d import _SymmetricMemory

    return _SymmetricMemory.has_multicast_support(DeviceType.CUDA, 0)


def _spawn(world, transport, **kw):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, transport, q, kw))
             for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert results[r] == "ok", results[r]


@pytest.mark.parametrize("transport", ["nccl", "peer", "nvls"])
def test_sharded_on_two_gpus(transport):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if transport == "nvls" and not _multicast_ok():
        pytest.skip("no NVLink multicast on this node")
    _spawn(2, transport)


def test_global_fiber_one_rank(cuda):
    """ShardedSignFiberChannel at one rank (real kernels): global bit k is
    element k of the parameters in order, padding between parameters
    excluded, so it agrees with the local channel over the shard's views and
    survives a step."""
    from t3st_b200 import TorchSignFiberChannel
    from t3st_b200.zero import ShardedDFCAdamW, ShardedSignFiberChannel

    torch.manual_seed(0)
    params = [torch.nn.Parameter((torch.randn(s) * 0.02).to(cuda)) for s in SHAPES]
    opt = ShardedDFCAdamW(params, lr=1e-3, moment_format="packed", compress_grads=True,
                          bucket_elems=8192)
    ch = ShardedSignFiberChannel(opt)
    local = TorchSignFiberChannel(opt)
    total = sum(p.numel() for p in params)
    assert ch.bit_capacity == total == local.bit_capacity
    rng = np.random.default_rng(2)
    bits = rng.integers(0, 2, total).astype(np.uint8)
    ch.write_bits(0, bits)
    np.testing.assert_array_equal(local.read_bits(0, total), bits)
    np.testing.assert_array_equal(ch.read_bits(5, total - 9), bits[5:total - 4])
    assert ch.owner(total - 1)[0] == 0
    for p in params:
        p.grad.normal_(0.0, 1e-3)
    opt.step()
    np.testing.assert_array_equal(ch.read_bits(0, total), bits)


@pytest.mark.parametrize("world", [2, 4])
def test_global_fiber_on_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _spawn(world, "fiber")


@pytest.mark.parametrize("transport", ["peer", "nvls"])
def test_fused_kernel_walks_tiles_on_two_gpus(transport):
    """One fused CTA per SM over ~1M-element pieces, with the compression in
    its own capped kernel on the caller's stream: every CTA of the persistent
    grid steps several tiles; bit-exact as above."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if transport == "nvls" and not _multicast_ok():
        pytest.skip("no NVLink multicast on this node")
    _spawn(2, transport, shapes=SHAPES_LARGE, bucket=1 << 20, fused_ctas=1, fuse=False)


@pytest.mark.parametrize("transport", ["peer", "nvls"])
def test_overlapped_buckets_on_two_gpus(transport):
    """Fused kernels of neighbouring buckets on two streams (barriers kept in
    order): still bit-exact, over several buckets."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if transport == "nvls" and not _multicast_ok():
        pytest.skip("no NVLink multicast on this node")
    _spawn(2, transport, overlap=True)


@pytest.mark.parametrize("transport", ["peer", "nvls"])
def test_fused_compression_on_two_gpus(transport):
    """Bucket b+1's compression inside the grid of bucket b's fused kernel
    (fuse_compression): bit-exact as above over several buckets, with one
    CTA per tile, and with a capped grid whose CTAs walk step and
    compression tiles."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    if transport == "nvls" and not _multicast_ok():
        pytest.skip("no NVLink multicast on this node")
    _spawn(2, transport, fuse=True)
    _spawn(2, transport, fuse=True, shapes=SHAPES_LARGE, bucket=1 << 20, fused_ctas=1)


@pytest.mark.parametrize("world", [4, 8])
def test_fused_compression_on_more_gpus(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    transport = "nvls" if world > 4 and _multicast_ok() else "peer"
    _spawn(world, transport, fuse=True)


@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("transport", ["nccl", "peer", "nvls"])
def test_sharded_on_more_gpus(transport, world):
    """The same check with 4 and 8 ranks (the switch then sums 4 or 8 values
    per element, and the fused kernel reads and writes 3 or 7 peers)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    if transport == "nvls" and not _multicast_ok():
        pytest.skip("no NVLink multicast on this node")
    _spawn(world, transport)
