"""Replay records of the sign-fiber continual-learning benchmark, on the GPU
(remote/vision_benchmark.py:25-151).

``CIFAR4BitCodec`` keeps the reference's record format and its
``encode``/``decode`` API.  ``encode_batch``/``decode_batch`` run a whole
batch as one kernel each way (``dfc_replay_encode``/``dfc_replay_decode``: 4-bit
quantisation, packing and the zlib CRC-32 on the device, one warp per record).
``FiberReservoir``, ``ArrayChannel`` and ``CompositeChannel`` mirror the
benchmark's classes.  When a channel can move device bytes
(``TorchSignFiberChannel``, ``DeviceArrayChannel``, or a ``CompositeChannel``
of them), records go between the codec and the optimizer's sign fiber
without a host round trip.
"""

from __future__ import annotations

import bisect
import struct

import numpy as np
import torch

from . import _lib

RECORD_BYTES = _lib.REPLAY_RECORD_BYTES
PIXELS = _lib.REPLAY_PIXELS
# reservoir header: magic, records held (uint32), records offered (uint64)
_RESERVOIR_HEADER = struct.Struct("<4sIQ")


def _device_of(t: torch.Tensor | None) -> torch.device:
    if t is not None and t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("the replay codec runs on a CUDA device (libdfc_b200.so)")
    return torch.device("cuda", torch.cuda.current_device())


def _check_u16(values) -> None:
    """Raise what the reference's int.to_bytes(2, "little") raises for a
    label or task outside [0, 65535] (vision_benchmark.py:83-84)."""
    for v in values:
        int(v).to_bytes(2, "little")


def _u16_tensor(v, n: int, device: torch.device) -> torch.Tensor:
    t = torch.as_tensor(v).reshape(-1)
    if t.numel() == 1 and n != 1:
        t = t.expand(n)
    if t.numel() != n:
        raise ValueError("one label and one task per record")
    if n == 0:
        return torch.empty(0, dtype=torch.int32, device=device)
    if t.dtype.is_floating_point or t.dtype == torch.bool:
        raise TypeError("labels and tasks must be integers")
    if n:
        lo, hi = int(t.min()), int(t.max())
        if lo < 0 or hi > 0xFFFF:
            _check_u16([lo, hi])
    return t.to(device=device, dtype=torch.int32).contiguous()


class CIFAR4BitCodec:
    """remote/vision_benchmark.py:74-100, on the device."""

    MAGIC = b"CF4B"
    RECORD_BYTES = RECORD_BYTES

    @classmethod
    def encode_batch(cls, x: torch.Tensor, y, task) -> torch.Tensor:
        """x: (n, 3, 32, 32) or (n, 3072) FP32 images -> (n, 1552) uint8
        records on the images' CUDA device (the current one for CPU images)."""
        if x.dtype != torch.float32:
            raise TypeError("replay images must be float32 (as ToTensor makes them)")
        n = x.shape[0] if x.dim() > 1 else 1
        if x.numel() != n * PIXELS:
            raise ValueError("a record holds 3 x 32 x 32 = 3072 pixels")
        dev = _device_of(x)
        images = x.detach().reshape(n, PIXELS).to(dev).contiguous()
        labels = _u16_tensor(y, n, dev)
        tasks = _u16_tensor(task, n, dev)
        out = torch.empty((n, RECORD_BYTES), dtype=torch.uint8, device=dev)
        if n:
            with torch.cuda.device(dev):
                _lib.check("dfc_replay_encode", _lib.lib().dfc_replay_encode(
                    images.data_ptr(), PIXELS, labels.data_ptr(), tasks.data_ptr(), n,
                    out.data_ptr(), RECORD_BYTES, torch.cuda.current_stream(dev).cuda_stream))
        return out

    @classmethod
    def decode_batch(cls, records: torch.Tensor, check: bool = True):
        """(n, 1552) uint8 records -> (images (n, 3, 32, 32) FP32, labels
        int64, tasks int64) on the records' CUDA device.  With check, the
        first bad record (in order) raises the reference's RuntimeError;
        without, a fourth tensor holds each record's status
        (0 ok, 1 bad magic, 2 checksum mismatch)."""
        if records.dtype != torch.uint8 or records.dim() != 2 or records.shape[1] != RECORD_BYTES:
            raise RuntimeError("invalid CIFAR replay record")
        dev = _device_of(records)
        n = records.shape[0]
        recs = records.to(dev).contiguous()
        images = torch.empty((n, 3, 32, 32), dtype=torch.float32, device=dev)
        meta = torch.empty((3, n), dtype=torch.int32, device=dev)
        if n:
            with torch.cuda.device(dev):
                _lib.check("dfc_replay_decode", _lib.lib().dfc_replay_decode(
                    recs.data_ptr(), RECORD_BYTES, n, images.data_ptr(), meta[0].data_ptr(),
                    meta[1].data_ptr(), meta[2].data_ptr(),
                    torch.cuda.current_stream(dev).cuda_stream))
        labels, tasks, status = meta[0].long(), meta[1].long(), meta[2]
        if not check:
            return images, labels, tasks, status
        if n:
            bad = torch.nonzero(status).reshape(-1)
            if bad.numel():
                code = int(status[bad[0]])
                if code == _lib.RECORD_BAD_MAGIC:
                    raise RuntimeError("invalid CIFAR replay record")
                raise RuntimeError("CIFAR replay checksum mismatch")
        return images, labels, tasks

    @classmethod
    def encode(cls, x: torch.Tensor, y: int, task: int) -> bytes:
        """One record as bytes (vision_benchmark.py:78-88)."""
        _check_u16([y, task])
        rec = cls.encode_batch(x.detach().reshape(1, -1), [int(y)], [int(task)])
        return rec.cpu().numpy().tobytes()

    @classmethod
    def decode(cls, raw: bytes) -> tuple[torch.Tensor, int, int]:
        """One record -> (CPU image (3, 32, 32), label, task)
        (vision_benchmark.py:90-100)."""
        raw = bytes(raw)
        if len(raw) != RECORD_BYTES or raw[:4] != cls.MAGIC:
            raise RuntimeError("invalid CIFAR replay record")
        dev = _device_of(None)
        rec = torch.frombuffer(bytearray(raw), dtype=torch.uint8).reshape(1, -1).to(dev)
        x, y, t = cls.decode_batch(rec)
        return x[0].cpu(), int(y[0]), int(t[0])


# ---- channels -----------------------------------------------------------------
class ArrayChannel:
    """Host byte store (vision_benchmark.py:25-38)."""

    def __init__(self, capacity: int):
        self.storage = bytearray(max(0, int(capacity)))

    @property
    def byte_capacity(self) -> int:
        return len(self.storage)

    def read_bytes(self, start: int, count: int) -> bytes:
        return bytes(self.storage[start:start + count])

    def write_bytes(self, start: int, payload) -> None:
        raw = bytes(payload)
        self.storage[start:start + len(raw)] = raw


class DeviceArrayChannel:
    """ArrayChannel whose bytes live in device memory (no reference
    counterpart): the external replay memory next to the fiber on the GPU."""

    def __init__(self, capacity: int, device=None):
        dev = torch.device(device) if device is not None else _device_of(None)
        self.storage = torch.zeros(max(0, int(capacity)), dtype=torch.uint8, device=dev)
        self.device = dev

    @property
    def byte_capacity(self) -> int:
        return self.storage.numel()

    def read_device(self, start: int, count: int) -> torch.Tensor:
        return self.storage[start:start + count].clone()

    def write_device(self, start: int, data: torch.Tensor) -> None:
        self.storage[start:start + data.numel()].copy_(data.reshape(-1))

    def read_bytes(self, start: int, count: int) -> bytes:
        return self.storage[start:start + count].cpu().numpy().tobytes()

    def write_bytes(self, start: int, payload) -> None:
        raw = bytes(payload)
        src = torch.frombuffer(bytearray(raw), dtype=torch.uint8) if raw else \
            torch.empty(0, dtype=torch.uint8)
        self.storage[start:start + len(raw)].copy_(src)


def _has_device_io(channel) -> bool:
    return hasattr(channel, "read_device") and hasattr(channel, "write_device")


class CompositeChannel:
    """Channels joined end to end into one byte space (the benchmark's
    CompositeChannel, vision_benchmark.py:41-71: same capacity, same
    ``IndexError("channel range out of bounds")``, channels of zero capacity
    never addressed).  A byte range is cut into per-channel pieces by a
    binary search over the channels' start offsets; the device forms move
    each piece with the channel's own device I/O where it has one."""

    def __init__(self, channels):
        self.channels = tuple(channels)
        sizes = [int(c.byte_capacity) for c in self.channels]
        self._starts = [0] * len(sizes)
        for i in range(1, len(sizes)):
            self._starts[i] = self._starts[i - 1] + sizes[i - 1]
        self._stops = [a + n for a, n in zip(self._starts, sizes)]
        self._total = self._stops[-1] if sizes else 0

    @property
    def byte_capacity(self) -> int:
        return self._total

    def _pieces(self, start: int, count: int) -> list:
        """[(channel, offset in it, length)] covering [start, start + count)."""
        start, count = int(start), int(count)
        stop = start + count
        if start < 0 or count < 0 or stop > self._total:
            raise IndexError("channel range out of bounds")
        pieces = []
        # the last channel that begins at or before ``start``: a zero-capacity
        # channel sharing that offset comes earlier and is passed over
        i = bisect.bisect_right(self._starts, start) - 1
        while start < stop:
            if self._stops[i] > start:
                n = min(stop, self._stops[i]) - start
                pieces.append((self.channels[i], start - self._starts[i], n))
                start += n
            i += 1
        return pieces

    def read_bytes(self, start: int, count: int) -> bytes:
        return b"".join(c.read_bytes(at, n) for c, at, n in self._pieces(start, count))

    def write_bytes(self, start: int, payload) -> None:
        data = bytes(payload)
        done = 0
        for c, at, n in self._pieces(start, len(data)):
            c.write_bytes(at, data[done:done + n])
            done += n

    @property
    def device_io(self) -> bool:
        return all(_has_device_io(c) for c in self.channels)

    def read_device(self, start: int, count: int, device=None) -> torch.Tensor:
        dev = torch.device(device) if device is not None else _device_of(None)
        parts = []
        for c, at, n in self._pieces(start, count):
            if _has_device_io(c):
                parts.append(c.read_device(at, n).to(dev))
            else:
                parts.append(torch.frombuffer(bytearray(c.read_bytes(at, n)),
                                              dtype=torch.uint8).to(dev))
        if len(parts) == 1:
            return parts[0]
        return torch.cat(parts) if parts else torch.empty(0, dtype=torch.uint8, device=dev)

    def write_device(self, start: int, data: torch.Tensor) -> None:
        flat = data.reshape(-1)
        done = 0
        for c, at, n in self._pieces(start, flat.numel()):
            if _has_device_io(c):
                c.write_device(at, flat[done:done + n])
            else:
                c.write_bytes(at, flat[done:done + n].cpu().numpy().tobytes())
            done += n


# ---- reservoir ----------------------------------------------------------------
class FiberReservoir:
    """Reservoir of replay records in a byte channel
    (vision_benchmark.py:103-151): a 16-byte header ("CVR2", size uint32,
    seen uint64, little-endian) and then fixed 1552-byte slots.  Same slot
    choice and the same draws from ``rng`` as the reference, so the channel
    ends up holding the same bytes."""

    HEADER_BYTES = _RESERVOIR_HEADER.size
    MAGIC = b"CVR2"

    def __init__(self, channel):
        self.channel = channel
        room = channel.byte_capacity
        self.capacity = max(0, (room - self.HEADER_BYTES) // RECORD_BYTES)
        self.size = self.seen = 0
        head = channel.read_bytes(0, min(self.HEADER_BYTES, room))
        if len(head) == self.HEADER_BYTES and head[:4] == self.MAGIC:
            _, self.size, self.seen = _RESERVOIR_HEADER.unpack(head)  # resume
        elif room >= self.HEADER_BYTES:
            self._header()  # a fresh reservoir stamps its empty header

    def _header(self) -> None:
        self.channel.write_bytes(0, _RESERVOIR_HEADER.pack(self.MAGIC, self.size, self.seen))

    def _offset(self, index: int) -> int:
        return self.HEADER_BYTES + index * RECORD_BYTES

    def _write_record(self, index: int, record: torch.Tensor) -> None:
        if _has_device_io(self.channel) and getattr(self.channel, "device_io", True):
            self.channel.write_device(self._offset(index), record)
        else:
            self.channel.write_bytes(self._offset(index), record.cpu().numpy().tobytes())

    def _slot(self, rng: np.random.Generator) -> int:
        self.seen += 1
        if self.size < self.capacity:
            index = self.size
            self.size += 1
            return index
        index = int(rng.integers(0, self.seen))
        return index if index < self.capacity else -1

    def add(self, x: torch.Tensor, y: int, task: int, rng: np.random.Generator) -> None:
        if self.capacity == 0:
            return
        index = self._slot(rng)
        if index >= 0:
            _check_u16([y, task])
            self._write_record(index, CIFAR4BitCodec.encode_batch(x.detach().reshape(1, -1),
                                                                   [int(y)], [int(task)])[0])
        self._header()

    def add_batch(self, x: torch.Tensor, y, task, rng: np.random.Generator) -> None:
        """len(x) successive add() calls with one encode launch: the slots
        and rng draws are those of the sequential calls, and a slot chosen
        twice keeps the later record."""
        if self.capacity == 0 or len(x) == 0:
            return
        slots = [self._slot(rng) for _ in range(len(x))]
        records = CIFAR4BitCodec.encode_batch(x.reshape(len(x), -1), y, task)
        last = {}
        for i, s in enumerate(slots):
            if s >= 0:
                last[s] = i
        for s, i in sorted(last.items()):
            self._write_record(s, records[i])
        self._header()

    def sample(self, count: int, rng: np.random.Generator, device=None):
        """count records drawn uniformly -> (images (count, 3, 32, 32),
        labels).  CPU tensors like the reference by default; on ``device``
        when given (decoded there, no host copy of the images)."""
        indices = rng.integers(0, self.size, size=count)
        if len(indices) == 0:  # the reference's torch.stack of no records
            raise RuntimeError("stack expects a non-empty TensorList")
        dev = torch.device(device) if device is not None else _device_of(None)
        if _has_device_io(self.channel) and getattr(self.channel, "device_io", True):
            parts = [self.channel.read_device(self._offset(int(i)), RECORD_BYTES) for i in indices]
            recs = torch.stack([p.to(dev) for p in parts]) if parts else \
                torch.empty((0, RECORD_BYTES), dtype=torch.uint8, device=dev)
        else:
            raw = b"".join(self.channel.read_bytes(self._offset(int(i)), RECORD_BYTES)
                           for i in indices)
            if len(raw) != len(indices) * RECORD_BYTES:
                raise RuntimeError("invalid CIFAR replay record")
            recs = torch.frombuffer(bytearray(raw), dtype=torch.uint8).reshape(-1, RECORD_BYTES) \
                if raw else torch.empty((0, RECORD_BYTES), dtype=torch.uint8)
            recs = recs.to(dev)
        images, labels, _ = CIFAR4BitCodec.decode_batch(recs)
        if device is None:
            return images.cpu(), labels.cpu()
        return images, labels
