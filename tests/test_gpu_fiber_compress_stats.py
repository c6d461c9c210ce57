"""Device sign-fiber I/O, bf16 compression with error feedback and the
gradient statistics kernels, against the oracle / host bit arithmetic."""

import numpy as np
import pytest
import torch

from oracle import oracle as O
from t3st_b200 import DFCAdamW, TorchSignFiberChannel, _lib, kernels

pytestmark = pytest.mark.gpu


def _fiber_bits(tensors):
    return np.concatenate([(t.reshape(-1).view(torch.int32).cpu().numpy().view(np.uint32) >> 31)
                           .astype(np.uint8) for t in tensors])


def test_fiber_bits_and_bytes_over_many_ranges(cuda):
    rng = np.random.default_rng(7)
    sizes = [int(s) for s in rng.integers(1, 300, 1500)] + [1, 7, 9, 4099]
    params = [torch.nn.Parameter(torch.zeros(s, device=cuda)) for s in sizes]
    opt = DFCAdamW(params)
    ch = TorchSignFiberChannel(opt)
    total = ch.bit_capacity
    bits = rng.integers(0, 2, total, dtype=np.uint8)
    ch.write_bits(0, bits)
    np.testing.assert_array_equal(_fiber_bits(opt.second_moment_tensors()), bits)
    for start, count in [(0, total), (3, 1), (5, 1000), (total - 13, 13), (8 * 77 + 3, 4001)]:
        np.testing.assert_array_equal(ch.read_bits(start, count), bits[start:start + count])
    # byte form, unaligned start bit inside tensors
    payload = rng.bytes(ch.byte_capacity - 5)
    ch.write_bytes(5, payload)
    assert ch.read_bytes(5, len(payload)) == payload
    got = _fiber_bits(opt.second_moment_tensors())[40:40 + 8 * len(payload)]
    np.testing.assert_array_equal(np.packbits(got, bitorder="little").tobytes(), payload)
    # partial write leaves neighbours alone
    before = _fiber_bits(opt.second_moment_tensors())
    ch.write_bits(1001, np.array([1, 0, 1], np.uint8))
    after = _fiber_bits(opt.second_moment_tensors())
    before[1001:1004] = [1, 0, 1]
    np.testing.assert_array_equal(after, before)
    # magnitudes untouched by payload writes
    for t in opt.second_moment_tensors():
        assert torch.count_nonzero(t.view(torch.int32) & 0x7FFFFFFF) == 0


@pytest.mark.parametrize("n,offset", [(1, 0), (4, 0), (4099, 0), (1 << 20, 0), (1000003, 1),
                                      (77777, 3)])
def test_compress_matches_oracle_over_steps(cuda, n, offset):
    rng = np.random.default_rng(n)
    gbuf = torch.zeros(n + offset, device=cuda)
    cbuf = torch.zeros(n + offset, dtype=torch.int16, device=cuda)
    qbuf = torch.zeros(n + offset, dtype=torch.int16, device=cuda)
    g, c, q = gbuf[offset:], cbuf[offset:], qbuf[offset:]
    hc = np.zeros(n, np.uint16)
    hq = np.zeros(n, np.uint16)
    for step in range(4):
        x = (rng.standard_t(3, n) * 1e-3).astype(np.float32)
        if step == 2 and n > 8:
            x[:3] = [np.inf, np.nan, 1e-40]
        g.copy_(torch.from_numpy(x))
        kernels.compress_ef(g, c, q)
        O.compress_ef(x, hc, hq)
        np.testing.assert_array_equal(c.cpu().numpy().view(np.uint16), hc)
        np.testing.assert_array_equal(q.cpu().numpy().view(np.uint16), hq)


@pytest.mark.parametrize("ctas_per_sm", [1, 3])
def test_compress_capped_grid_matches_oracle(cuda, ctas_per_sm):
    """The grid capped as the ZeRO-1 pipeline caps it: every thread walks
    several grid strides, two quads per iteration (odd quad counts leave one
    thread a single quad), plus a scalar tail."""
    n = (1 << 21) + 4 * 129 + 3
    rng = np.random.default_rng(ctas_per_sm)
    g = torch.zeros(n, device=cuda)
    c = torch.zeros(n, dtype=torch.int16, device=cuda)
    q = torch.zeros(n, dtype=torch.int16, device=cuda)
    hc = np.zeros(n, np.uint16)
    hq = np.zeros(n, np.uint16)
    for _ in range(3):
        x = (rng.standard_t(3, n) * 1e-3).astype(np.float32)
        g.copy_(torch.from_numpy(x))
        kernels.compress_ef(g, c, q, ctas_per_sm)
        O.compress_ef(x, hc, hq)
        np.testing.assert_array_equal(c.cpu().numpy().view(np.uint16), hc)
        np.testing.assert_array_equal(q.cpu().numpy().view(np.uint16), hq)


def test_grad_stats_match_oracle(cuda):
    rng = np.random.default_rng(8)
    sizes = [0, 1, 5, 8192, 8193, 100003, 1 << 20]
    grads = []
    for i, n in enumerate(sizes):
        x = (rng.standard_normal(n) * 1e-2).astype(np.float32)
        if i == 4:
            x[[3, 77]] = [np.inf, np.nan]
        grads.append(x)
    tg = [torch.from_numpy(x).to(cuda) for x in grads]
    tg.append(torch.from_numpy(grads[5]).to(cuda).bfloat16())
    stats = kernels.stats_to_numpy(kernels.grad_stats(tg))
    for i, x in enumerate(grads + [None]):
        if x is None:
            x = tg[-1].float().cpu().numpy()
        s, a, bad = O.grad_stats(x)
        assert stats[i]["nonfinite"] == bad
        assert stats[i]["amax"] == np.float32(a)
        if np.isnan(s):
            assert np.isnan(stats[i]["sumsq"])
        else:
            assert stats[i]["sumsq"] == pytest.approx(s, rel=1e-12, abs=0)
    # deterministic: the same input gives the same bits
    again = kernels.stats_to_numpy(kernels.grad_stats(tg))
    assert again.tobytes() == stats.tobytes()


def test_grad_stats_large_buffers_match_oracle(cuda):
    """Buffers of 1,101 and 611 tiles (8,192 elements each) with a ragged
    tail: every CTA of the statistics pass walks several tiles (the next
    tile's loads in flight during the block reduction), and the final fold
    of the 1,101-tile buffer loops over batches of records."""
    rng = np.random.default_rng(21)
    xs = [(rng.standard_t(3, 8192 * 1100 + 5) * 1e-2).astype(np.float32),
          (rng.standard_normal(8192 * 611) * 1e-3).astype(np.float32), np.ones(3, np.float32)]
    xs[0][[17, 8192 * 700 + 1]] = [np.inf, -np.inf]
    tg = [torch.from_numpy(x).to(cuda) for x in xs]
    stats = kernels.stats_to_numpy(kernels.grad_stats(tg))
    for i, x in enumerate(xs):
        s, a, bad = O.grad_stats(x)
        assert stats[i]["nonfinite"] == bad
        assert stats[i]["amax"] == np.float32(a)
        if np.isnan(s) or np.isinf(s):
            assert stats[i]["sumsq"] == s or (np.isnan(s) and np.isnan(stats[i]["sumsq"]))
        else:
            assert stats[i]["sumsq"] == pytest.approx(s, rel=1e-12, abs=0)
    again = kernels.stats_to_numpy(kernels.grad_stats(tg))
    assert again.tobytes() == stats.tobytes()


def test_fiber_large_ranges_round_trip(cuda):
    """Ranges of millions of words: every warp of the fiber kernels walks
    several groups of 256 words, including across range boundaries."""
    rng = np.random.default_rng(22)
    sizes = [3_000_001, 5, 2_500_000, 777_777]
    params = [torch.nn.Parameter(torch.zeros(s, device=cuda)) for s in sizes]
    opt = DFCAdamW(params)
    ch = TorchSignFiberChannel(opt)
    payload = rng.integers(0, 256, ch.byte_capacity, dtype=np.uint8)
    ch.write_device(0, torch.from_numpy(payload).to(cuda))
    bits = _fiber_bits(opt.second_moment_tensors())
    np.testing.assert_array_equal(np.packbits(bits[:8 * payload.size], bitorder="little"), payload)
    np.testing.assert_array_equal(ch.read_device(0, payload.size).cpu().numpy(), payload)
    # an unaligned window that starts inside the first range and ends in the last
    start, count = 3 * 8 + 1, ch.bit_capacity - 40
    np.testing.assert_array_equal(ch.read_bits(start, count), bits[start:start + count])


@pytest.mark.parametrize("word_off", [0, 1, 4])   # first word 16-byte aligned, not, aligned
@pytest.mark.parametrize("pay_off", [0, 1])       # payload pointer 4-byte aligned, not
@pytest.mark.parametrize("start", [0, 512, 13])
def test_fiber_vector_and_word_paths(cuda, word_off, pay_off, start):
    """One range of ~1M words through the C ABI: 512-bit spans take the
    16-byte path when the words and the payload pointer allow it, the
    per-word path otherwise; both give the reference's bit order."""
    rng = np.random.default_rng(100 * word_off + 10 * pay_off + start)
    n = (1 << 20) + 37
    base = torch.from_numpy(rng.integers(0, 2 ** 32, n, dtype=np.uint64).astype(np.uint32)
                            .view(np.int32)).to(cuda)
    w = base[word_off:]
    before = w.cpu().numpy().view(np.uint32).copy()
    ranges = np.zeros(1, dtype=_lib.WORDRANGE_DTYPE)
    ranges[0] = (w.data_ptr(), w.numel())
    count = w.numel() - start - 7
    nbytes = (count + 7) // 8
    buf = torch.full((nbytes + 8,), 0x5A, dtype=torch.uint8, device=cuda)
    out = buf[pay_off:pay_off + nbytes]
    lib = _lib.lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    _lib.check("dfc_fiber_read", lib.dfc_fiber_read(_lib.ptr(ranges), 1, start, count,
                                                    out.data_ptr(), stream))
    want = np.packbits((before[start:start + count] >> 31).astype(np.uint8), bitorder="little")
    np.testing.assert_array_equal(out.cpu().numpy(), want)
    assert int((buf[pay_off + nbytes:] != 0x5A).sum()) == 0 and (pay_off == 0 or int(buf[0]) == 0x5A)
    payload = rng.integers(0, 256, nbytes, dtype=np.uint8)
    out.copy_(torch.from_numpy(payload))
    _lib.check("dfc_fiber_write", lib.dfc_fiber_write(_lib.ptr(ranges), 1, start, count,
                                                      out.data_ptr(), stream))
    after = w.cpu().numpy().view(np.uint32)
    bits = np.unpackbits(payload, bitorder="little")[:count].astype(np.uint32)
    expect = before.copy()
    expect[start:start + count] = (before[start:start + count] & 0x7FFFFFFF) | (bits << 31)
    np.testing.assert_array_equal(after, expect)


def test_fiber_holes(cuda):
    """Ranges with NULL words are holes: zero bits on a read, untouched on a
    write (how a ZeRO-1 rank addresses its own bits of the global fiber).
    Holes of a few bits and of several whole 512-bit spans, between ranges
    that take the 16-byte and the per-word paths."""
    rng = np.random.default_rng(3)
    layout = [("w", 1000, 0), ("h", 777, 0), ("w", 5000, 3), ("h", 3 * 4096 + 5, 0),
              ("w", 70000, 0), ("h", 9, 0), ("w", 4096, 1)]
    ranges = np.zeros(len(layout), dtype=_lib.WORDRANGE_DTYPE)
    bufs, truth = [], []
    for i, (kind, n, off) in enumerate(layout):
        if kind == "w":
            b = torch.from_numpy(rng.integers(0, 2 ** 32, n + off, dtype=np.uint64)
                                 .astype(np.uint32).view(np.int32)).to(cuda)
            bufs.append((b, off, n))
            ranges[i] = (b.data_ptr() + 4 * off, n)
            truth.append((b[off:].cpu().numpy().view(np.uint32) >> 31).astype(np.uint8))
        else:
            ranges[i] = (0, n)
            truth.append(np.zeros(n, np.uint8))
    bits = np.concatenate(truth)
    total = bits.size
    lib = _lib.lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for start, count in [(0, total), (1003, total - 2000), (512 * 30, 4096 * 2)]:
        out = torch.full(((count + 7) // 8,), 0xFF, dtype=torch.uint8, device=cuda)
        _lib.check("dfc_fiber_read", lib.dfc_fiber_read(_lib.ptr(ranges), len(ranges), start,
                                                        count, out.data_ptr(), stream))
        want = np.packbits(bits[start:start + count], bitorder="little")
        np.testing.assert_array_equal(out.cpu().numpy(), want)
    before = [b.cpu().numpy().view(np.uint32).copy() for b, _, _ in bufs]
    payload = rng.integers(0, 256, (total + 7) // 8, dtype=np.uint8)
    src = torch.from_numpy(payload).to(cuda)
    _lib.check("dfc_fiber_write", lib.dfc_fiber_write(_lib.ptr(ranges), len(ranges), 0, total,
                                                      src.data_ptr(), stream))
    pbits = np.unpackbits(payload, bitorder="little")[:total].astype(np.uint32)
    pos = 0
    k = 0
    for kind, n, off in layout:
        if kind == "w":
            b, _, _ = bufs[k]
            want = before[k].copy()
            want[off:] = (want[off:] & 0x7FFFFFFF) | (pbits[pos:pos + n] << 31)
            np.testing.assert_array_equal(b.cpu().numpy().view(np.uint32), want)
            k += 1
        pos += n


def test_clip_coef_and_clipped_step(cuda):
    torch.manual_seed(0)
    shapes = [(300, 77), (1000,), (5,)]
    params = [torch.nn.Parameter(torch.randn(s, device=cuda) * 0.02) for s in shapes]
    grads = [torch.randn(s, device=cuda) for s in shapes]
    p0 = [p.detach().cpu().numpy().copy() for p in params]
    opt = DFCAdamW(params, lr=1e-3, weight_decay=0.01, max_grad_norm=1.0)
    for p, g in zip(params, grads):
        p.grad = g
    opt.step()
    torch.cuda.synchronize()
    coef, norm = opt._last_clip.cpu().numpy()
    total = np.sqrt(sum(float(np.sum(g.double().cpu().numpy() ** 2)) for g in grads))
    assert norm == pytest.approx(total, rel=1e-6)
    assert coef == np.float32(np.float32(1.0) / (np.float32(norm) + np.float32(1e-6)))
    h = O.reference_hyper(1e-3, (0.9, 0.999), 1e-8, 0.01, 1, grad_scale=float(coef))
    for p, p_init, g in zip(params, p0, grads):
        p_ref = p_init.reshape(-1).copy()
        m = np.zeros(p_ref.size, np.uint32)
        v = np.zeros(p_ref.size, np.uint32)
        O.step(O.MODE_SIGNFIBER, h, p_ref, g.cpu().numpy().reshape(-1).copy(), m, v)
        np.testing.assert_array_equal(p.detach().cpu().numpy().reshape(-1).view(np.uint32),
                                      p_ref.view(np.uint32))
