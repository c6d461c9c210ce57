"""End-to-end training parity: ResNet-18 (3x3 stem, no max-pool, 10
classes), batches of 256 N(0,1) 3x32x32 images with uniform int64 labels,
bf16 autocast forward/backward, cross-entropy, deterministic algorithms.

The reference optimizer is the reference's FP32 DFCAdamW step
(remote/torch_fiber.py:68-117, fiber on) run by the oracle on the host each
step (the reference's CPU arithmetic, with an IEEE square root): gradients
go to the host, the oracle updates p, m, v there, p comes back.

  * t3st_b200 DFCAdamW with packed moment words and FP32 gradients must
    reproduce the reference's loss curve exactly, every step (fixed batch,
    so the loss falls and the run is sensitive to any difference).
  * ShardedDFCAdamW on one GPU with bf16 error-feedback gradients (a fresh
    seeded batch every step): within 1e-3 relative of the reference's loss
    over the first 10 steps, and over 100 steps no further from it than an
    FP32 run whose only difference is rounding -- the reference's step
    restated as PyTorch CUDA ops.  This training run amplifies any last-bit
    difference to ~0.5% of the loss within ~20 steps (measured: the FP32
    PyTorch-CUDA restatement itself deviates by up to ~8e-3), so a 1e-3 bound
    over 100 steps holds only for bit-identical arithmetic, which the packed
    step above meets.
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


def _train(kind, device, init, steps, fresh):
    model = _model(device)
    model.load_state_dict(init)
    params = list(model.parameters())
    data = _batches(device, fresh)
    losses = []
    if kind == "reference":
        host = [dict(p=p.detach().cpu().numpy().reshape(-1).copy(),
                     m=np.zeros(p.numel(), np.uint32), v=np.zeros(p.numel(), np.uint32))
                for p in params]
        counters = [0] * len(params)
        group = dict(lr=LR, betas=BETAS, eps=EPS, weight_decay=WD)
        for _ in range(steps):
            x, y = next(data)
            for p in params:
                p.grad = None
            loss = _loss(model, x, y)
            loss.backward()
            losses.append(loss.item())
            grads = [p.grad.detach().cpu().numpy().reshape(-1) for p in params]
            O.multi_tensor_step(O.MODE_SIGNFIBER, host, grads, group, counters)
            with torch.no_grad():
                for p, h in zip(params, host):
                    p.copy_(torch.from_numpy(h["p"]).view_as(p))
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
    init = {k: v.clone() for k, v in _model(cuda).state_dict().items()}
    ref = _train("reference", cuda, init, 100, fresh=True)
    got = _train("compressed", cuda, init, 100, fresh=True)
    floor = _train("torch_cuda", cuda, init, 100, fresh=True)
    rel = np.abs(got - ref) / np.abs(ref)
    noise = np.abs(floor - ref) / np.abs(ref)
    assert rel[:10].max() <= 1e-3, (float(rel[:10].max()), int(rel[:10].argmax()))
    assert rel.max() <= 1.5 * noise.max(), (float(rel.max()), float(noise.max()))
    assert rel.mean() <= 1.5 * noise.mean(), (float(rel.mean()), float(noise.mean()))
