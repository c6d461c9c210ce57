"""The replay-record oracle against records made by the reference's own
CIFAR4BitCodec and FiberReservoir (tests/golden/replay.npz), the split CRC
the device uses against zlib, and the host side of the reservoir mirror.
CPU only."""

import os
import zlib

import numpy as np
import pytest

from oracle import replay as R

G = np.load(os.path.join(os.path.dirname(__file__), "golden", "replay.npz"))


def test_encode_matches_reference_records():
    for i in range(len(G["images"])):
        rec = R.encode(G["images"][i], int(G["labels"][i]), int(G["tasks"][i]))
        assert rec == G["records"][i].tobytes(), i


def test_decode_matches_reference():
    for i in range(len(G["records"])):
        x, y, t = R.decode(G["records"][i].tobytes())
        np.testing.assert_array_equal(x.view(np.uint32), G["decoded"][i].view(np.uint32))
        assert (y, t) == (int(G["dec_labels"][i]), int(G["dec_tasks"][i]))


def test_bad_records_raise_the_reference_errors():
    for raw, err in zip(G["bad_records"], G["bad_errors"]):
        with pytest.raises(RuntimeError, match=str(err)):
            R.decode(raw.tobytes())
        assert R.status(raw.tobytes()) == (1 if "invalid" in str(err) else 2)
    with pytest.raises(RuntimeError, match="invalid"):
        R.decode(G["records"][0].tobytes()[:-1])


def test_quantisation_edges():
    x = np.array([np.nan, np.inf, -np.inf, -0.0, 0.5 / 15, 1.5 / 15, 2.5 / 15, 1.0, -0.3, 2.0],
                 np.float32)
    np.testing.assert_array_equal(R.quantize(x), [0, 15, 0, 0, 0, 2, 2, 15, 0, 15])


@pytest.mark.parametrize("n", [0, 1, 3, 4, 5, 64, 1544, 4099])
def test_split_crc_equals_zlib(n):
    rng = np.random.default_rng(n)
    data = bytes(rng.integers(0, 256, n, dtype=np.uint8))
    cuts = sorted(set([0, n] + list(rng.integers(0, n + 1, 5))))
    runs = list(zip(cuts[:-1], cuts[1:])) or [(0, 0)]
    assert R.crc32_split(data, runs) == zlib.crc32(data)


def test_device_runs_tile_a_record():
    runs = R.device_runs()
    assert runs[0][0] == 0 and runs[-1][1] == R.CRC_BYTES
    assert all(a[1] == b[0] for a, b in zip(runs[:-1], runs[1:]))
    rec = G["records"][0].tobytes()
    assert R.crc32_split(rec[:R.CRC_BYTES], runs) == int.from_bytes(rec[1544:1548], "little")


def test_reservoir_oracle_reproduces_reference_channel():
    cap = int(G["res_capacity"])
    rng = np.random.default_rng(int(G["res_rng_seed"]))
    slots, size, seen = R.reservoir_slots(cap, 0, 0, int(G["res_adds"]), rng)
    assert (size, seen) == (int(G["res_size"]), int(G["res_seen"]))
    chan = bytearray(len(G["channel"]))
    for i, s in enumerate(slots):
        if s >= 0:
            off = R.RESERVOIR_HEADER + s * R.RECORD_BYTES
            chan[off:off + R.RECORD_BYTES] = R.encode(G["images"][i], int(G["labels"][i]),
                                                      int(G["tasks"][i]))
    chan[:16] = R.reservoir_header(size, seen)
    assert bytes(chan) == G["channel"].tobytes()
    idx = rng.integers(0, size, size=6)  # the sample's draws
    got = [R.decode(bytes(chan[16 + int(i) * 1552:16 + (int(i) + 1) * 1552])) for i in idx]
    np.testing.assert_array_equal(np.stack([g[0] for g in got]),
                                  G["sample_x"].reshape(6, -1))
    np.testing.assert_array_equal([g[1] for g in got], G["sample_y"])


def test_mirror_reservoir_slots_and_header_on_cpu():
    """The mirror's slot choice and header I/O need no GPU; they draw from the
    rng exactly as the oracle (and the reference) does."""
    from t3st_b200.replay import ArrayChannel, FiberReservoir

    ch = ArrayChannel(16 + 3 * 1552 + 7)
    res = FiberReservoir(ch)
    assert res.capacity == 3 and ch.read_bytes(0, 4) == b"CVR2"
    r1, r2 = np.random.default_rng(4), np.random.default_rng(4)
    got = [res._slot(r1) for _ in range(40)]
    want, size, seen = R.reservoir_slots(3, 0, 0, 40, r2)
    assert got == want and (res.size, res.seen) == (size, seen)
    res._header()
    again = FiberReservoir(ch)
    assert (again.size, again.seen) == (size, seen)
    assert r1.integers(0, 1 << 30) == r2.integers(0, 1 << 30)


def test_mirror_composite_channel_bounds():
    from t3st_b200.replay import ArrayChannel, CompositeChannel

    c = CompositeChannel([ArrayChannel(5), ArrayChannel(7)])
    c.write_bytes(3, b"abcdef")
    assert c.read_bytes(0, 12) == b"\0\0\0abcdef\0\0\0"
    with pytest.raises(IndexError):
        c.read_bytes(10, 3)


def test_composite_channel_matches_one_flat_store():
    """Random reads and writes through a composite with zero-capacity members
    (first, middle and last) behave as one flat byte store of the summed
    capacity; zero-capacity members are never called; ranges outside it
    raise the benchmark's IndexError (vision_benchmark.py:41-71)."""
    from t3st_b200.replay import ArrayChannel, CompositeChannel

    class Counted(ArrayChannel):
        def __init__(self, n):
            super().__init__(n)
            self.calls = 0

        def read_bytes(self, start, count):
            self.calls += 1
            assert 0 <= start and start + count <= self.byte_capacity and count > 0
            return super().read_bytes(start, count)

        def write_bytes(self, start, payload):
            self.calls += 1
            assert isinstance(payload, bytes) and 0 < len(payload)
            assert start + len(payload) <= self.byte_capacity
            super().write_bytes(start, payload)

    sizes = [0, 3, 0, 0, 11, 1, 0, 6, 0]
    parts = [Counted(n) for n in sizes]
    c = CompositeChannel(parts)
    flat = bytearray(sum(sizes))
    assert c.byte_capacity == len(flat) == 21
    rng = np.random.default_rng(9)
    for _ in range(400):
        a = int(rng.integers(0, len(flat) + 1))
        n = int(rng.integers(0, len(flat) - a + 1))
        if rng.integers(0, 2):
            data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
            c.write_bytes(a, data)
            flat[a:a + n] = data
        else:
            assert c.read_bytes(a, n) == bytes(flat[a:a + n])
    assert c.read_bytes(0, len(flat)) == bytes(flat)
    assert all(p.calls == 0 for p, n in zip(parts, sizes) if n == 0)
    for a, n in [(-1, 1), (0, -1), (21, 1), (20, 2), (0, 22)]:
        with pytest.raises(IndexError, match="channel range out of bounds"):
            c.read_bytes(a, n)
    with pytest.raises(IndexError, match="channel range out of bounds"):
        c.write_bytes(19, b"abc")
    assert CompositeChannel([]).byte_capacity == 0
    assert CompositeChannel([]).read_bytes(0, 0) == b""


def _rn32(x):
    """A Fraction rounded to the nearest FP32 value, ties to even."""
    from fractions import Fraction

    f = np.float32(float(x))
    cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
    return min(cands, key=lambda c: (abs(Fraction(float(c)) - x),
                                     int(np.array(c).view(np.uint32)) & 1))


def test_decode_nibble_division_is_correctly_rounded():
    """The decode kernel forms q / 15 as y = q * RN(1/15), e = fma(-15, y, q),
    fma(e, RN(1/15), y).  For every 4-bit q this equals the correctly
    rounded q / 15 that the reference's q.astype(float32) / 15 produces
    (remote/vision_benchmark.py:92-100); checked here in exact arithmetic."""
    from fractions import Fraction

    F = lambda v: Fraction(float(v))  # noqa: E731
    r = _rn32(Fraction(1, 15))
    assert np.array(r).view(np.uint32) == 0x3D888889
    for q in range(16):
        y = _rn32(q * F(r))
        e = _rn32(q - 15 * F(y))          # fma: one rounding of the exact value
        got = _rn32(F(e) * F(r) + F(y))   # fma
        want = np.float32(q) / np.float32(15)
        assert got == want and _rn32(Fraction(q, 15)) == want, q
