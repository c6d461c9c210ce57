"""End-to-end training parity (the C3 configuration): ResNet-18 (3x3 stem,
no max-pool, 10 classes), batches of 256 N(0,1) 3x32x32 images with uniform
int64 labels, bf16 autocast forward/backward, cross-entropy, deterministic
algorithms.

The reference optimizer is the reference's FP32 DFCAdamW step
(remote/torch_fiber.py:68-117, fiber on) run by the oracle on the host each
step (the reference's CPU arithmetic, with an IEEE square root): gradients
go to the host, the oracle updates p, m, v there, p comes back.

  * DFCAdamW with packed moment words and FP32 gradients reproduces the
    reference's loss curve exactly, every step of 100 (fixed batch, so the
    loss falls and the run is sensitive to any difference).
  * ShardedDFCAdamW with bf16 error-feedback compressed gradients, 200 steps
    with a fresh seeded batch each, as the C3 configuration runs:
      - exactly the loss curve of the reference's step fed the same
        compressed gradients (the oracle compresses each step's gradient
        with its own error-feedback state, then steps with it);
      - against the reference run on uncompressed FP32 gradients, the loss
        curves do NOT agree within the north star's 1e-3 relative over 100
        steps: they agree within 1e-3 over the first 10 steps, and over
        100 steps (and over all 200) deviate by up to 7.5e-3, mean ~2e-3
        (measured on B200).  The gap is the compression itself amplified by
        training:
        an FP32 run whose only difference is rounding (the reference step
        restated as PyTorch CUDA ops) deviates from the reference by as
        much (7.9e-3), so the test asserts no more than 1.5x that noise
        floor.
  * Two ranks over NVLink peer memory (when two GPUs are present), each on
    its own batch stream: every step's parameters and both ranks' losses
    equal a one-process simulation of the same data-parallel run whose
    optimizer is the reference's step fed the average of both ranks'
    compressed gradients (FP32 sum in rank order, then 1/2).
"""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from oracle import torch_port

pytestmark = pytest.mark.gpu

LR, BETAS, EPS, WD = 1e-3, (0.9, 0.999), 1e-8, 0.01


@pytest.fixture
def deterministic():
    prev = torch.are_deterministic_algorithms_enabled()
    prev_cudnn = (torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark)
    torch.use_deterministic_algorithms(True)
    torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark = True, False
    yield
    torch.use_deterministic_algorithms(prev)
    torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark = prev_cudnn


def _model(device):
    tv = pytest.importorskip("torchvision")
    torch.manual_seed(0)
    m = tv.models.resnet18(num_classes=10)
    m.conv1 = torch.nn.Conv2d(3, 64, 3, 1, 1, bias=False)
    m.maxpool = torch.nn.Identity()
    return m.to(device)


def _batches(device, fresh):
    g = torch.Generator().manual_seed(1)
    while True:
        x = torch.randn(256, 3, 32, 32, generator=g).to(device)
        y = torch.randint(0, 10, (256,), generator=g).to(device)
        while True:
            yield x, y
            if fresh:
                break


def _loss(model, x, y):
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model(x)
    return torch.nn.functional.cross_entropy(out.float(), y)


class _HostReference:
    """The reference's FP32 step (fiber on) on host copies of the parameters,
    run by the oracle, one thread per tensor.  compress=True first passes
    each gradient through the oracle's bf16 error-feedback compression (its
    own residual state per tensor and per rank) and steps with the bf16
    values; several ranks' compressed gradients are summed in FP32 in rank
    order and scaled by 1/ranks (the fused ZeRO-1 kernel's reduction)."""

    def __init__(self, params, compress=False, ranks=1):
        from concurrent.futures import ThreadPoolExecutor

        self.host = [dict(p=p.detach().cpu().numpy().reshape(-1).copy(),
                          m=np.zeros(p.numel(), np.uint32), v=np.zeros(p.numel(), np.uint32))
                     for p in params]
        self.compress, self.ranks, self.t = compress, ranks, 0
        self.ef = [[(np.zeros(p.numel(), np.uint16), np.zeros(p.numel(), np.uint16))
                    for p in params] for _ in range(ranks)]
        self.pool = ThreadPoolExecutor(max_workers=16)

    def _one(self, i, grads_by_rank):
        if self.compress:
            g = None
            for r, grads in enumerate(grads_by_rank):
                c, q = self.ef[r][i]
                O.compress_ef(np.ascontiguousarray(grads[i], dtype=np.float32), c, q)
                gr = (c.astype(np.uint32) << 16).view(np.float32)
                g = gr.copy() if g is None else (g + gr).astype(np.float32)
        else:
            g = np.ascontiguousarray(grads_by_rank[0][i])
        h = O.reference_hyper(LR, BETAS, EPS, WD, self.t, grad_scale=1.0 / self.ranks)
        t = self.host[i]
        O.step(O.MODE_SIGNFIBER, h, t["p"], g, t["m"], t["v"])

    def step(self, params, grads_by_rank):
        self.t += 1
        list(self.pool.map(lambda i: self._one(i, grads_by_rank), range(len(self.host))))
        with torch.no_grad():
            for p, h in zip(params, self.host):
                p.copy_(torch.from_numpy(h["p"]).view_as(p))


def _train(kind, device, init, steps, fresh):
    model = _model(device)
    model.load_state_dict(init)
    params = list(model.parameters())
    data = _batches(device, fresh)
    losses = []
    if kind in ("reference", "reference_compressed"):
        ref = _HostReference(params, compress=kind == "reference_compressed")
        for _ in range(steps):
            x, y = next(data)
            for p in params:
                p.grad = None
            loss = _loss(model, x, y)
            loss.backward()
            losses.append(loss.item())
            ref.step(params, [[p.grad.detach().cpu().numpy().reshape(-1) for p in params]])
        return np.array(losses)
    if kind == "torch_cuda":
        state = [(torch.zeros_like(p), torch.zeros_like(p)) for p in params]
        for t in range(1, steps + 1):
            x, y = next(data)
            for p in params:
                p.grad = None
            loss = _loss(model, x, y)
            loss.backward()
            losses.append(loss.item())
            with torch.no_grad():
                for p, (m, v) in zip(params, state):
                    torch_port.step_fp32(p.data, p.grad, m, v, LR, BETAS, EPS, WD, t, fiber=True)
        return np.array(losses)
    if kind == "packed":
        from t3st_b200 import DFCAdamW

        opt = DFCAdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD,
                       moment_format="packed")
    else:
        from t3st_b200.zero import ShardedDFCAdamW

        opt = ShardedDFCAdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD,
                              moment_format="packed", compress_grads=True)
    for _ in range(steps):
        x, y = next(data)
        opt.zero_grad()
        loss = _loss(model, x, y)
        loss.backward()
        losses.append(loss.item())
        opt.step()
    return np.array(losses)


def test_packed_step_reproduces_reference_loss_curve_exactly(cuda, deterministic):
    init = {k: v.clone() for k, v in _model(cuda).state_dict().items()}
    ref = _train("reference", cuda, init, 100, fresh=False)
    assert ref[-1] < 0.5 * ref[0]  # the fixed batch is being learned
    got = _train("packed", cuda, init, 100, fresh=False)
    np.testing.assert_array_equal(got, ref)


def test_compressed_grads_loss_curve(cuda, deterministic):
    steps = 200  # the C3 configuration
    init = {k: v.clone() for k, v in _model(cuda).state_dict().items()}
    got = _train("compressed", cuda, init, steps, fresh=True)
    same_grads = _train("reference_compressed", cuda, init, steps, fresh=True)
    # the reference's step fed the same compressed gradients: the same curve
    np.testing.assert_array_equal(got, same_grads)
    # against the reference on uncompressed FP32 gradients (secondary): the
    # effect of compression, bounded by the rounding-noise floor of this run
    ref = _train("reference", cuda, init, steps, fresh=True)
    floor = _train("torch_cuda", cuda, init, steps, fresh=True)
    rel = np.abs(got - ref) / np.abs(ref)
    noise = np.abs(floor - ref) / np.abs(ref)
    print(f"compressed vs FP32-gradient reference: max rel {rel[:100].max():.2e} over 100 "
          f"steps, {rel.max():.2e} over {steps}; rounding-noise floor {noise[:100].max():.2e} "
          f"/ {noise.max():.2e}")
    assert rel[:10].max() <= 1e-3, (float(rel[:10].max()), int(rel[:10].argmax()))
    assert rel.max() <= 1.5 * noise.max(), (float(rel.max()), float(noise.max()))
    assert rel.mean() <= 1.5 * noise.mean(), (float(rel.mean()), float(noise.mean()))


def _rank_batches(device, rank, steps):
    g = torch.Generator().manual_seed(1000 + rank)
    for _ in range(steps):
        x = torch.randn(256, 3, 32, 32, generator=g).to(device)
        y = torch.randint(0, 10, (256,), generator=g).to(device)
        yield x, y


E2E_RANK_STEPS = 30


def _e2e_rank(rank, world, port, q, init, outdir):
    import datetime
    import os
    import traceback

    try:
        import torch.distributed as dist

        from t3st_b200.zero import ShardedDFCAdamW

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        torch.use_deterministic_algorithms(True)
        torch.backends.cudnn.deterministic, torch.backends.cudnn.benchmark = True, False
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=dev)
        model = _model(dev)
        model.load_state_dict({k: v.to(dev) for k, v in init.items()})
        params = list(model.parameters())
        opt = ShardedDFCAdamW(params, lr=LR, betas=BETAS, eps=EPS, weight_decay=WD,
                              moment_format="packed", compress_grads=True, transport="peer")
        losses = []
        for t, (x, y) in enumerate(_rank_batches(dev, rank, E2E_RANK_STEPS)):
            opt.zero_grad()
            loss = _loss(model, x, y)
            loss.backward()
            losses.append(loss.item())
            opt.step()
            if rank == 0:  # every step's parameters, for the comparison
                np.save(os.path.join(outdir, f"p{t}.npy"),
                        opt.flat_param.detach().cpu().numpy().view(np.uint32))
        torch.cuda.synchronize()
        assert opt.peer_status() == 0
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok", losses, list(opt.offsets)))
    except BaseException:
        q.put((rank, traceback.format_exc(), None, None))


def test_two_rank_compressed_training_matches_reference(cuda, deterministic, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import socket

    import torch.multiprocessing as mp

    init = {k: v.detach().cpu().clone() for k, v in _model(cuda).state_dict().items()}
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_e2e_rank, args=(r, 2, port, q, init, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    res = {r: (status, losses, offs) for r, status, losses, offs in
           (q.get(timeout=900) for _ in range(2))}
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert res[r][0] == "ok", res[r][0]
    offsets = res[0][2]

    # one-process simulation on cuda:0: both ranks' forward/backward with the
    # same parameters, the reference step fed their averaged compressed grads
    model = _model(cuda)
    model.load_state_dict(init)
    params = list(model.parameters())
    ref = _HostReference(params, compress=True, ranks=2)
    streams = [_rank_batches(cuda, r, E2E_RANK_STEPS) for r in range(2)]
    for t in range(E2E_RANK_STEPS):
        grads_by_rank = []
        for r in range(2):
            x, y = next(streams[r])
            for p in params:
                p.grad = None
            loss = _loss(model, x, y)
            loss.backward()
            assert loss.item() == res[r][1][t], (r, t, loss.item(), res[r][1][t])
            grads_by_rank.append([p.grad.detach().cpu().numpy().reshape(-1) for p in params])
        ref.step(params, grads_by_rank)
        snap = np.load(tmp_path / f"p{t}.npy")
        for i, (h, off) in enumerate(zip(ref.host, offsets)):
            np.testing.assert_array_equal(snap[off:off + h["p"].size], h["p"].view(np.uint32),
                                          err_msg=f"step {t + 1}, parameter {i}")
