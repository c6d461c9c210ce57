"""End-to-end training parity: ResNet-18 (3x3 stem, no max-pool, 10
classes) on a fixed synthetic batch of 256 N(0,1) 3x32x32 images with
uniform int64 labels, bf16 autocast forward/backward, cross-entropy.

Three runs from the same initial weights, 200 steps each:
  reference   the reference's FP32 DFCAdamW step (remote/torch_fiber.py:
              68-117, fiber on) restated as eager PyTorch ops on the GPU
  packed      t3st_b200 DFCAdamW, packed moment words, FP32 gradients
  compressed  t3st_b200 ShardedDFCAdamW on one GPU: bf16 gradients with
              per-element error feedback, packed moments
The loss curves must agree with the reference's to 1e-3 relative over the
first 100 steps."""

import numpy as np
import pytest
import torch

from oracle import torch_port

pytestmark = pytest.mark.gpu

STEPS = 200
CHECK = 100
LR, BETAS, EPS, WD = 1e-3, (0.9, 0.999), 1e-8, 0.01


def _model(device):
    tv = pytest.importorskip("torchvision")
    torch.manual_seed(0)
    m = tv.models.resnet18(num_classes=10)
    m.conv1 = torch.nn.Conv2d(3, 64, 3, 1, 1, bias=False)
    m.maxpool = torch.nn.Identity()
    return m.to(device)


def _batch(device):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(256, 3, 32, 32, generator=g).to(device)
    y = torch.randint(0, 10, (256,), generator=g).to(device)
    return x, y


def _loss(model, x, y):
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = model(x)
    return torch.nn.functional.cross_entropy(out.float(), y)


def _train(kind, device, init, x, y):
    model = _model(device)
    model.load_state_dict(init)
    params = list(model.parameters())
    losses = []
    if kind == "reference":
        state = [(torch.zeros_like(p), torch.zeros_like(p)) for p in params]
        for t in range(1, STEPS + 1):
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
    for _ in range(STEPS):
        opt.zero_grad()
        loss = _loss(model, x, y)
        loss.backward()
        losses.append(loss.item())
        opt.step()
    return np.array(losses)


def test_resnet18_loss_curves_match_reference(cuda):
    torch.backends.cudnn.deterministic = True
    torch.backends.cudnn.benchmark = False
    init = {k: v.clone() for k, v in _model(cuda).state_dict().items()}
    x, y = _batch(cuda)
    ref = _train("reference", cuda, init, x, y)
    assert ref[CHECK - 1] < 0.9 * ref[0]  # the run actually trains
    for kind in ("packed", "compressed"):
        got = _train(kind, cuda, init, x, y)
        rel = np.abs(got[:CHECK] - ref[:CHECK]) / np.abs(ref[:CHECK])
        assert rel.max() <= 1e-3, (kind, float(rel.max()), int(rel.argmax()))
