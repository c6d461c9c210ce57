"""The device replay codec (dfc_replay_encode / dfc_replay_decode) and the
reservoir mirror on the GPU, against the reference's records
(tests/golden/replay.npz) and the oracle: bit-exact records, pixels, labels
and errors; the reservoir's channel bytes and samples; records routed
through the optimizer's sign fiber; and a large batch through the round
trip decode(encode(x)) == quantize(x) / 15 with every CRC checked."""

import os

import numpy as np
import pytest
import torch

from oracle import replay as R

pytestmark = pytest.mark.gpu

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "replay.npz"))


def _codec():
    from t3st_b200.replay import CIFAR4BitCodec

    return CIFAR4BitCodec


def test_encode_batch_matches_reference_records(cuda):
    x = torch.from_numpy(G["images"]).to(cuda)
    rec = _codec().encode_batch(x, torch.from_numpy(G["labels"]), torch.from_numpy(G["tasks"]))
    np.testing.assert_array_equal(rec.cpu().numpy(), G["records"])


def test_decode_batch_matches_reference(cuda):
    rec = torch.from_numpy(G["records"]).to(cuda)
    x, y, t = _codec().decode_batch(rec)
    np.testing.assert_array_equal(x.reshape(len(rec), -1).cpu().numpy().view(np.uint32),
                                  G["decoded"].view(np.uint32))
    np.testing.assert_array_equal(y.cpu().numpy(), G["dec_labels"])
    np.testing.assert_array_equal(t.cpu().numpy(), G["dec_tasks"])


def test_single_record_api_matches_reference(cuda):
    codec = _codec()
    for i in (0, 1, 3, 6):
        raw = codec.encode(torch.from_numpy(G["images"][i]), int(G["labels"][i]), int(G["tasks"][i]))
        assert raw == G["records"][i].tobytes()
        x, y, t = codec.decode(raw)
        assert x.shape == (3, 32, 32) and x.device.type == "cpu"
        np.testing.assert_array_equal(x.numpy().reshape(-1), G["decoded"][i])
        assert (y, t) == (int(G["dec_labels"][i]), int(G["dec_tasks"][i]))


def test_bad_records_raise_the_reference_errors(cuda):
    codec = _codec()
    for raw, err in zip(G["bad_records"], G["bad_errors"]):
        with pytest.raises(RuntimeError, match=str(err)):
            codec.decode(raw.tobytes())
    _, _, _, status = codec.decode_batch(torch.from_numpy(G["bad_records"]).to(cuda), check=False)
    np.testing.assert_array_equal(status.cpu().numpy(), [R.status(r.tobytes()) for r in G["bad_records"]])
    # first bad record in order decides the error of a batch
    mixed = torch.from_numpy(np.stack([G["records"][0], G["bad_records"][2], G["bad_records"][0]])).to(cuda)
    with pytest.raises(RuntimeError, match="invalid CIFAR replay record"):
        codec.decode_batch(mixed)


def test_label_range_and_dtype_errors(cuda):
    codec = _codec()
    x = torch.zeros(3, 32, 32)
    with pytest.raises(OverflowError):
        codec.encode(x, 65536, 0)
    with pytest.raises(OverflowError):
        codec.encode(x, 0, -1)
    with pytest.raises(OverflowError):
        codec.encode_batch(x.reshape(1, -1).to(cuda), torch.tensor([70000]), torch.tensor([0]))
    with pytest.raises(TypeError):
        codec.encode(x.double(), 0, 0)
    assert codec.encode_batch(torch.zeros(0, 3072, device=cuda), [], []).shape == (0, 1552)


def test_reservoir_over_host_channel_matches_reference(cuda):
    from t3st_b200.replay import ArrayChannel, FiberReservoir

    ch = ArrayChannel(len(G["channel"]))
    res = FiberReservoir(ch)
    rng = np.random.default_rng(int(G["res_rng_seed"]))
    for i in range(int(G["res_adds"])):
        res.add(torch.from_numpy(G["images"][i]), int(G["labels"][i]), int(G["tasks"][i]), rng)
    assert bytes(ch.storage) == G["channel"].tobytes()
    sx, sy = res.sample(6, rng)
    assert sx.device.type == "cpu" and sy.dtype == torch.int64
    np.testing.assert_array_equal(sx.numpy(), G["sample_x"])
    np.testing.assert_array_equal(sy.numpy(), G["sample_y"])


def _oracle_channel(cap_bytes, images, labels, tasks, seed, n_sample):
    rng = np.random.default_rng(seed)
    capacity = max(0, (cap_bytes - 16) // R.RECORD_BYTES)
    slots, size, seen = R.reservoir_slots(capacity, 0, 0, len(images), rng)
    chan = bytearray(cap_bytes)
    for i, s in enumerate(slots):
        if s >= 0:
            off = 16 + s * R.RECORD_BYTES
            chan[off:off + R.RECORD_BYTES] = R.encode(images[i], int(labels[i]), int(tasks[i]))
    chan[:16] = R.reservoir_header(size, seen)
    idx = rng.integers(0, size, size=n_sample)
    return bytes(chan), idx


@pytest.mark.parametrize("batched", [False, True])
def test_reservoir_through_the_sign_fiber(cuda, batched):
    """The benchmark's layout: the optimizer's sign fiber first, then an
    external array (here in device memory), records encoded and decoded on
    the GPU without a host copy."""
    from t3st_b200 import DFCAdamW, TorchSignFiberChannel
    from t3st_b200.replay import CompositeChannel, DeviceArrayChannel, FiberReservoir

    torch.manual_seed(0)
    params = [torch.nn.Parameter(torch.randn(n, device=cuda)) for n in (4099, 31 * 257, 15000)]
    opt = DFCAdamW(params, lr=1e-3)
    fiber = TorchSignFiberChannel(opt)
    ext = DeviceArrayChannel(3 * 1552 + 40, device=cuda)
    ch = CompositeChannel([fiber, ext])
    res = FiberReservoir(ch)
    rng = np.random.default_rng(21)
    imgs = np.random.default_rng(2).random((40, 3, 32, 32), dtype=np.float32)
    labels = np.arange(40) % 100
    tasks = labels // 10
    if batched:
        res.add_batch(torch.from_numpy(imgs).to(cuda), torch.from_numpy(labels),
                      torch.from_numpy(tasks), rng)
    else:
        for i in range(40):
            res.add(torch.from_numpy(imgs[i]).to(cuda), int(labels[i]), int(tasks[i]), rng)
    want, idx = _oracle_channel(ch.byte_capacity, imgs, labels, tasks, 21, 9)
    assert ch.read_bytes(0, ch.byte_capacity) == want
    sx, sy = res.sample(9, rng, device=cuda)
    assert sx.is_cuda
    exp = [R.decode(want[16 + int(i) * 1552:16 + (int(i) + 1) * 1552]) for i in idx]
    np.testing.assert_array_equal(sx.reshape(9, -1).cpu().numpy(), np.stack([e[0] for e in exp]))
    np.testing.assert_array_equal(sy.cpu().numpy(), [e[1] for e in exp])
    # the records survive an optimizer step: only bit 31 of v carries them
    for p in params:
        p.grad = torch.randn_like(p) * 1e-3
    opt.step()
    assert ch.read_bytes(0, ch.byte_capacity) == want


def test_large_batch_round_trip(cuda):
    """65,536 records (805 MB of images): every record's CRC matches the
    oracle's on a sample, every record decodes to quantize(x) / 15."""
    n = 65536
    g = torch.Generator(device=cuda).manual_seed(9)
    x = torch.rand((n, 3072), generator=g, device=cuda) * 1.2 - 0.1
    y = torch.randint(0, 65536, (n,), generator=g, device=cuda)
    t = torch.randint(0, 65536, (n,), generator=g, device=cuda)
    codec = _codec()
    rec = codec.encode_batch(x, y, t)
    xd, yd, td, status = codec.decode_batch(rec, check=False)
    assert int(status.abs().sum()) == 0
    assert torch.equal(yd, y) and torch.equal(td, t)
    q = torch.clamp(torch.round(x * 15.0), 0, 15).long()
    lut = torch.from_numpy(np.arange(16, dtype=np.float32) / np.float32(15.0)).to(cuda)
    assert torch.equal(xd.reshape(n, -1), lut[q])
    pick = torch.randint(0, n, (64,), generator=g, device=cuda).cpu().numpy()
    xs, rs = x[pick].cpu().numpy(), rec[pick].cpu().numpy()
    for i, k in enumerate(pick):
        assert rs[i].tobytes() == R.encode(xs[i], int(y[k]), int(t[k]))
