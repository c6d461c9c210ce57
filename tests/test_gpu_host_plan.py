"""DFCAdamW's native steady-state plan on the GPU: several steps over FP32,
bf16 and fp16 parameters in one optimizer, in all three moment modes, with
gradients re-created every step (as backward does after
zero_grad(set_to_none=True)), a learning-rate change between steps (as a
scheduler makes) and one step taken under a step hook (the torch.optim
wrapper path).  After every step, parameters, moment words (payload bits
included) and step counters are compared bit for bit with the oracle
(remote/torch_fiber.py:68-117 restated)."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from t3st_b200 import DFCAdamW

pytestmark = pytest.mark.gpu

SHAPES = [(257, 31), (31,), (4099,), (3, 3, 3), (1000,), (64, 3, 3, 3)]
DTYPES = [torch.float32, torch.bfloat16, torch.float16, torch.float32, torch.bfloat16,
          torch.float16]
NAMES = {torch.float32: "f32", torch.bfloat16: "bf16", torch.float16: "f16"}


def _bits(t):
    t = t.detach().reshape(-1).cpu()
    if t.dtype == torch.float32:
        return t.numpy().copy()
    return t.view(torch.int16).numpy().view(np.uint16).copy()


@pytest.mark.parametrize("fmt,fiber,mode", [("fp32", True, O.MODE_SIGNFIBER),
                                            ("fp32", False, O.MODE_PLAIN),
                                            ("packed", True, O.MODE_PACKED)])
def test_native_plan_steps_match_oracle(cuda, fmt, fiber, mode):
    gen = torch.Generator().manual_seed(3)
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(dt).to(cuda))
              for s, dt in zip(SHAPES, DTYPES)]
    lr, betas, eps, wd = 1e-3, (0.9, 0.999), 1e-8, 0.01
    opt = DFCAdamW(params, lr=lr, betas=betas, eps=eps, weight_decay=wd, enable_fiber=fiber,
                   moment_format=fmt)
    rng = np.random.default_rng(4)
    sim = []
    for p in params:
        v = opt.state[p]["exp_avg_sq"].view(torch.int32)
        if fiber:  # payload bits in bit 31 of the second moment
            bits = torch.from_numpy(rng.integers(0, 2, p.numel()).astype(np.int32)).to(cuda)
            v.view(-1).copy_(bits << 31)
        sim.append([_bits(p), np.zeros(p.numel(), np.uint32),
                    v.reshape(-1).cpu().numpy().view(np.uint32).copy()])
    seen = []
    for step in range(1, 7):
        if step == 4:
            lr = 5e-4
            opt.param_groups[0]["lr"] = lr
        grads = [(torch.randn(s, generator=gen) * 1e-3).to(dt) for s, dt in zip(SHAPES, DTYPES)]
        for p, g in zip(params, grads):
            p.grad = g.to(cuda)  # a new gradient tensor every step
        plan_before = opt._native
        handle = opt.register_step_pre_hook(lambda o, a, k: seen.append(step)) if step == 5 else None
        opt.step()
        if handle is not None:
            handle.remove()
        if step >= 2:  # the same plan every step, the hooked step (5) included
            assert plan_before is not None and opt._native is plan_before, \
                f"step {step} left the native plan"
        torch.cuda.synchronize()
        h = O.reference_hyper(lr, betas, eps, wd, step)
        for i, (p, g) in enumerate(zip(params, grads)):
            name = NAMES[p.dtype]
            O.step(mode, h, sim[i][0], _bits(g), sim[i][1], sim[i][2], name, name)
            np.testing.assert_array_equal(_bits(p).view(np.uint32 if name == "f32" else np.uint16),
                                          sim[i][0].view(np.uint32 if name == "f32" else np.uint16),
                                          err_msg=f"step {step}, tensor {i}")
            np.testing.assert_array_equal(
                opt.state[p]["exp_avg"].reshape(-1).cpu().numpy().view(np.uint32), sim[i][1])
            np.testing.assert_array_equal(
                opt.state[p]["exp_avg_sq"].reshape(-1).cpu().numpy().view(np.uint32), sim[i][2])
            assert opt.state[p]["step"] == step
    assert seen == [5]
