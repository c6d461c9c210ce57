"""CPU restatement of the replay-record codec and reservoir of the sign-fiber
benchmark (remote/vision_benchmark.py:74-151).

Test infrastructure only: the tests, the smoke check and the bench's CPU
baseline compare the device codec (libdfc_b200.so, dfc_replay_encode /
dfc_replay_decode) against this module.  Nothing in the product imports it.
Pinned against records made by the reference's own CIFAR4BitCodec and
FiberReservoir (tests/golden/replay.npz).
"""

from __future__ import annotations

import zlib

import numpy as np

MAGIC = b"CF4B"          # vision_benchmark.py:75
RECORD_BYTES = 1552      # vision_benchmark.py:76
PIXELS = 3072
CRC_BYTES = 1544         # the CRC covers bytes [0, 1544) (vision_benchmark.py:86)
RESERVOIR_MAGIC = b"CVR2"  # vision_benchmark.py:105
RESERVOIR_HEADER = 16      # vision_benchmark.py:104


def quantize(x: np.ndarray) -> np.ndarray:
    """clamp(round(x * 15), 0, 15) as uint8 (vision_benchmark.py:80): the
    product in FP32, round half to even, NaN to 0 (what the reference's
    float->uint8 cast gives on x86)."""
    x = np.asarray(x, dtype=np.float32).reshape(-1)
    r = np.rint(x * np.float32(15.0))
    q = np.where(r >= 15, 15, np.where(r > 0, r, 0))
    return np.nan_to_num(q, nan=0.0).astype(np.uint8)


def encode(x: np.ndarray, y: int, task: int) -> bytes:
    """One record (vision_benchmark.py:78-88)."""
    q = quantize(x)
    if q.size != PIXELS:
        raise ValueError("a record holds 3072 pixels")
    packed = q[0::2] | (q[1::2] << np.uint8(4))
    raw = bytearray(RECORD_BYTES)
    raw[:4] = MAGIC
    raw[4:6] = int(y).to_bytes(2, "little")
    raw[6:8] = int(task).to_bytes(2, "little")
    raw[8:CRC_BYTES] = packed.tobytes()
    raw[CRC_BYTES:CRC_BYTES + 4] = (zlib.crc32(raw[:CRC_BYTES]) & 0xFFFFFFFF).to_bytes(4, "little")
    return bytes(raw)


def decode(raw: bytes) -> tuple[np.ndarray, int, int]:
    """One record -> (3072 FP32 pixels, label, task), raising the reference's
    RuntimeErrors (vision_benchmark.py:90-100)."""
    if len(raw) != RECORD_BYTES or raw[:4] != MAGIC:
        raise RuntimeError("invalid CIFAR replay record")
    if zlib.crc32(raw[:CRC_BYTES]) & 0xFFFFFFFF != int.from_bytes(raw[CRC_BYTES:CRC_BYTES + 4], "little"):
        raise RuntimeError("CIFAR replay checksum mismatch")
    packed = np.frombuffer(raw[8:CRC_BYTES], dtype=np.uint8)
    q = np.empty(PIXELS, dtype=np.uint8)
    q[0::2], q[1::2] = packed & 15, packed >> 4
    return (q.astype(np.float32) / np.float32(15.0), int.from_bytes(raw[4:6], "little"),
            int.from_bytes(raw[6:8], "little"))


def status(raw: bytes) -> int:
    """0 valid, 1 bad length or magic, 2 checksum mismatch (the order in
    which the reference checks, vision_benchmark.py:92-95)."""
    if len(raw) != RECORD_BYTES or raw[:4] != MAGIC:
        return 1
    stored = int.from_bytes(raw[CRC_BYTES:CRC_BYTES + 4], "little")
    return 0 if zlib.crc32(raw[:CRC_BYTES]) & 0xFFFFFFFF == stored else 2


# ---- the device's split CRC, restated --------------------------------------
POLY = 0xEDB88320   # reflected 0x04C11DB7
ONE = 0x80000000    # x^0 in the reflected representation


def gf2_mulmod(a: int, b: int) -> int:
    """a * b mod P with bit 31 holding x^0."""
    p = 0
    for i in range(32):
        if a & (ONE >> i):
            p ^= b
        b = (b >> 1) ^ (POLY if b & 1 else 0)
    return p


def x_pow_8n(n: int) -> int:
    result, base = ONE, ONE >> 8
    while n:
        if n & 1:
            result = gf2_mulmod(result, base)
        base = gf2_mulmod(base, base)
        n >>= 1
    return result


def _remainder(data: bytes, c: int) -> int:
    for byte in data:
        c ^= byte
        for _ in range(8):
            c = (c >> 1) ^ (POLY if c & 1 else 0)
    return c


def crc32_split(data: bytes, runs: list[tuple[int, int]]) -> int:
    """CRC-32 of data from independent runs [start, end) that tile it: each
    run's remainder (the first from 0xFFFFFFFF, the rest from 0) times
    x^(8 * bytes after the run), XORed, then inverted -- the device scheme."""
    total = 0
    for k, (a, b) in enumerate(runs):
        r = _remainder(data[a:b], 0xFFFFFFFF if k == 0 else 0)
        total ^= gf2_mulmod(r, x_pow_8n(len(data) - b))
    return total ^ 0xFFFFFFFF


def device_runs() -> list[tuple[int, int]]:
    """The 32 lane runs of a record: lane 0 [0, 56), lane k [8+48k, 56+48k)."""
    return [(0 if k == 0 else 8 + 48 * k, 8 + 48 * (k + 1)) for k in range(32)]


# ---- reservoir --------------------------------------------------------------
def reservoir_slots(capacity: int, size: int, seen: int, n_items: int, rng: np.random.Generator):
    """Slots chosen by n_items successive FiberReservoir.add calls
    (vision_benchmark.py:125-139): -1 where an item is dropped.  Returns
    (slots, size, seen) and draws from rng exactly as the reference does."""
    slots = []
    for _ in range(n_items):
        if capacity == 0:
            slots.append(-1)
            continue
        seen += 1
        if size < capacity:
            slots.append(size)
            size += 1
        else:
            index = int(rng.integers(0, seen))
            slots.append(index if index < capacity else -1)
    return slots, size, seen


def reservoir_header(size: int, seen: int) -> bytes:
    """vision_benchmark.py:121-124."""
    return RESERVOIR_MAGIC + size.to_bytes(4, "little") + seen.to_bytes(8, "little")
