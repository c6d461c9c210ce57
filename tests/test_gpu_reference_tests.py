"""The reference's own unit tests (remote/test_torch_fiber.py:11-48),
re-pointed at the B200 DFCAdamW on CUDA, in both moment formats."""

import io

import numpy as np
import pytest
import torch

import golden_io as G
from t3st_b200 import DFCAdamW, TorchSignFiberChannel, local_fiber_capacity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fmt", ["fp32", "packed"])
def test_reference_and_payload_trajectory_are_bitwise_equal(cuda, fmt):
    """remote/test_torch_fiber.py:11-31: a full payload does not perturb the
    trajectory, and the step does not corrupt the payload."""
    torch.manual_seed(17)
    reference = torch.nn.Linear(257, 31).to(cuda)
    lifted = torch.nn.Linear(257, 31).to(cuda)
    lifted.load_state_dict(reference.state_dict())
    opt_ref = DFCAdamW(reference.parameters(), lr=3e-4, weight_decay=0.01, enable_fiber=False,
                       moment_format=fmt)
    opt_dfc = DFCAdamW(lifted.parameters(), lr=3e-4, weight_decay=0.01, enable_fiber=True,
                       moment_format=fmt)
    channel = TorchSignFiberChannel(opt_dfc)
    rng = np.random.default_rng(19)
    payload = rng.bytes(channel.byte_capacity)
    channel.write_bytes(0, payload)
    for _ in range(50):
        x = torch.randn(23, 257).to(cuda)
        y = torch.randn(23, 31).to(cuda)
        for model, optimizer in ((reference, opt_ref), (lifted, opt_dfc)):
            optimizer.zero_grad()
            torch.nn.functional.mse_loss(model(x), y).backward()
            optimizer.step()
    for a, b in zip(reference.parameters(), lifted.parameters()):
        assert torch.equal(a, b)
    assert channel.read_bytes(0, len(payload)) == payload


def test_trajectory_close_to_reference_cpu_run(cuda):
    """Same 50-step trajectory as the golden run of the reference on CPU.
    Gradients come from cuBLAS instead of MKL here, so agreement is to
    rounding noise, not bits."""
    d = G.load("unit_linear")
    model = torch.nn.Linear(257, 31).to(cuda)
    with torch.no_grad():
        model.weight.copy_(torch.from_numpy(d["w0"]))
        model.bias.copy_(torch.from_numpy(d["b0"]))
    opt = DFCAdamW(model.parameters(), lr=3e-4, weight_decay=0.01, enable_fiber=True)
    ch = TorchSignFiberChannel(opt)
    ch.write_bytes(0, d["payload"].tobytes())
    x = torch.from_numpy(d["x"]).to(cuda)
    y = torch.from_numpy(d["y"]).to(cuda)
    for s in range(x.shape[0]):
        opt.zero_grad()
        torch.nn.functional.mse_loss(model(x[s]), y[s]).backward()
        opt.step()
    np.testing.assert_allclose(model.weight.detach().cpu().numpy(), d["w"], rtol=0, atol=2e-6)
    np.testing.assert_allclose(model.bias.detach().cpu().numpy(), d["b"], rtol=0, atol=2e-6)
    assert ch.read_bytes(0, len(d["payload"])) == d["payload"].tobytes()


@pytest.mark.parametrize("fmt", ["fp32", "packed"])
def test_checkpoint_preserves_payload(cuda, fmt):
    """remote/test_torch_fiber.py:33-48."""
    model = torch.nn.Linear(128, 64).to(cuda)
    optimizer = DFCAdamW(model.parameters(), enable_fiber=True, moment_format=fmt)
    channel = TorchSignFiberChannel(optimizer)
    payload = bytes((index * 37) % 256 for index in range(channel.byte_capacity))
    channel.write_bytes(0, payload)
    file = io.BytesIO()
    torch.save({"model": model.state_dict(), "optimizer": optimizer.state_dict()}, file)
    file.seek(0)
    restored_model = torch.nn.Linear(128, 64).to(cuda)
    restored_optimizer = DFCAdamW(restored_model.parameters(), enable_fiber=True, moment_format=fmt)
    checkpoint = torch.load(file, weights_only=True)
    restored_model.load_state_dict(checkpoint["model"])
    restored_optimizer.load_state_dict(checkpoint["optimizer"])
    restored = TorchSignFiberChannel(restored_optimizer)
    assert restored.read_bytes(0, len(payload)) == payload


def test_checkpoint_format_conversion(cuda):
    """An FP32 (reference-format) checkpoint loads into a packed optimizer
    and back, payload and moments intact."""
    torch.manual_seed(3)
    model = torch.nn.Linear(64, 33).to(cuda)
    opt = DFCAdamW(model.parameters(), weight_decay=0.1)
    ch = TorchSignFiberChannel(opt)
    ch.write_bytes(0, bytes(range(256)) * (ch.byte_capacity // 256) + bytes(ch.byte_capacity % 256))
    for _ in range(3):
        opt.zero_grad()
        model(torch.randn(8, 64, device=cuda)).square().mean().backward()
        opt.step()
    sd = opt.state_dict()
    packed = DFCAdamW(model.parameters(), weight_decay=0.1, moment_format="packed")
    packed.load_state_dict(sd)
    back = DFCAdamW(model.parameters(), weight_decay=0.1)
    back.load_state_dict(packed.state_dict())
    for p in model.parameters():
        for k in ("exp_avg", "exp_avg_sq"):
            a = opt.state[p][k].view(torch.int32)
            b = back.state[p][k].view(torch.int32)
            assert torch.equal(a, b)
            w = packed.state[p][k].view(torch.int32)
            # the packed words differ wherever bit 15 rounded the high half up,
            # and keep bit 31 (sign / payload) everywhere
            assert torch.equal(w < 0, a < 0)
            assert torch.equal(w != a, (a & 0x8000) != 0)
    assert packed.state_dict()["moment_format"] == "packed"


def test_capacity_and_errors(cuda):
    model = torch.nn.Linear(10, 3).to(cuda)
    opt = DFCAdamW(model.parameters())
    assert local_fiber_capacity(opt) == {"payload_bits": 33, "payload_bytes": 4,
                                         "state_coordinates": 33}
    ch = TorchSignFiberChannel(opt)
    with pytest.raises(IndexError):
        ch.read_bytes(0, 5)
    with pytest.raises(IndexError):
        ch.read_bits(30, 4)
    with pytest.raises(ValueError):
        ch.write_bits(0, np.array([0, 2], np.uint8))
    with pytest.raises(ValueError):
        TorchSignFiberChannel(DFCAdamW(model.parameters(), enable_fiber=False))
    model.weight.grad = torch.zeros_like(model.weight).to_sparse()
    with pytest.raises(RuntimeError, match="sparse"):
        opt.step()
