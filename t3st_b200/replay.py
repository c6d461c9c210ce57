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

import numpy as np
import torch

from . import _lib

RECORD_BYTES = _lib.REPLAY_RECORD_BYTES
PIXELS = _lib.REPLAY_PIXELS


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
    """Channels joined end to end (vision_benchmark.py:41-71)."""

    def __init__(self, channels):
        self.channels = tuple(channels)
        self.ends = np.cumsum([channel.byte_capacity for channel in channels], dtype=np.int64)

    @property
    def byte_capacity(self) -> int:
        return int(self.ends[-1])

    def _segments(self, start: int, count: int):
        if start < 0 or count < 0 or start + count > self.byte_capacity:
            raise IndexError("channel range out of bounds")
        position, remaining = int(start), int(count)
        while remaining:
            index = int(np.searchsorted(self.ends, position, side="right"))
            base = 0 if index == 0 else int(self.ends[index - 1])
            local = position - base
            take = min(remaining, self.channels[index].byte_capacity - local)
            yield self.channels[index], local, take
            position += take
            remaining -= take

    def read_bytes(self, start: int, count: int) -> bytes:
        return b"".join(c.read_bytes(local, take) for c, local, take in self._segments(start, count))

    def write_bytes(self, start: int, payload) -> None:
        raw, cursor = bytes(payload), 0
        for channel, local, take in self._segments(start, len(raw)):
            channel.write_bytes(local, raw[cursor:cursor + take])
            cursor += take

    @property
    def device_io(self) -> bool:
        return all(_has_device_io(c) for c in self.channels)

    def read_device(self, start: int, count: int, device=None) -> torch.Tensor:
        parts = []
        for channel, local, take in self._segments(start, count):
            if _has_device_io(channel):
                parts.append(channel.read_device(local, take))
            else:
                raw = channel.read_bytes(local, take)
                parts.append(torch.frombuffer(bytearray(raw), dtype=torch.uint8))
        dev = torch.device(device) if device is not None else _device_of(None)
        if not parts:
            return torch.empty(0, dtype=torch.uint8, device=dev)
        return torch.cat([p.to(dev) for p in parts])

    def write_device(self, start: int, data: torch.Tensor) -> None:
        flat, cursor = data.reshape(-1), 0
        for channel, local, take in self._segments(start, flat.numel()):
            piece = flat[cursor:cursor + take]
            if _has_device_io(channel):
                channel.write_device(local, piece)
            else:
                channel.write_bytes(local, piece.cpu().numpy().tobytes())
            cursor += take


# ---- reservoir ----------------------------------------------------------------
class FiberReservoir:
    """Reservoir of replay records in a byte channel
    (vision_benchmark.py:103-151): a 16-byte header ("CVR2", size uint32,
    seen uint64) and then fixed 1552-byte slots.  Same slot choice and the
    same draws from ``rng`` as the reference, so the channel ends up holding
    the same bytes."""

    HEADER_BYTES = 16
    MAGIC = b"CVR2"

    def __init__(self, channel):
        self.channel = channel
        self.capacity = max(0, (channel.byte_capacity - self.HEADER_BYTES) // RECORD_BYTES)
        raw = channel.read_bytes(0, min(self.HEADER_BYTES, channel.byte_capacity))
        if len(raw) == self.HEADER_BYTES and raw[:4] == self.MAGIC:
            self.size = int.from_bytes(raw[4:8], "little")
            self.seen = int.from_bytes(raw[8:16], "little")
        else:
            self.size = self.seen = 0
            if channel.byte_capacity >= self.HEADER_BYTES:
                self._header()

    def _header(self) -> None:
        self.channel.write_bytes(
            0, self.MAGIC + self.size.to_bytes(4, "little") + self.seen.to_bytes(8, "little"))

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
