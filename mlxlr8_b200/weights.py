"""Read tensors and byte ranges of safetensors files straight into device
memory (``exlr8/weights.py:20-69`` ``SafeTensorFile``).

The header stays in memory; a read touches only the requested bytes.  A read
into device memory goes through pinned staging buffers: while one chunk is
copied to the device on a side stream, the next is read from the file into the
other, so a load runs at the slower of the file and the host-to-device link;
large reads are split over several reader threads, each with its own pair of
buffers and copy stream, to keep several file requests in flight.  ``raw``
keeps the reference's NumPy form (BF16 as uint16 bit patterns) for host-side
use; ``load``/``load_slice``/``read_into`` produce CUDA tensors.
"""

from __future__ import annotations

import json
import os
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import NamedTuple

import numpy as np
import torch

_DTYPES = {
    "U8": "u1", "I8": "i1", "U16": "<u2", "I16": "<i2",
    "U32": "<u4", "I32": "<i4", "U64": "<u8", "I64": "<i8",
    "F16": "<f2", "BF16": "<u2", "F32": "<f4", "F64": "<f8",
    "BOOL": "?",
}

_TORCH = {
    "U8": torch.uint8, "I8": torch.int8, "U16": torch.uint16, "I16": torch.int16,
    "U32": torch.uint32, "I32": torch.int32, "U64": torch.uint64, "I64": torch.int64,
    "F16": torch.float16, "BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64,
    "BOOL": torch.bool,
}

CHUNK_BYTES = 32 << 20
READERS = 4  # reader threads of one large read, each with its own staging pair


class _Stager:
    """Two pinned host buffers and a copy stream, reused by every read of one
    reader slot on one device."""

    _pool: dict = {}

    def __init__(self, device: torch.device):
        self.device = device
        self.buffers = [torch.empty(CHUNK_BYTES, dtype=torch.uint8, pin_memory=True) for _ in range(2)]
        self.views = [memoryview(b.numpy()) for b in self.buffers]
        self.stream = torch.cuda.Stream(device)
        self.done = [None, None]

    @classmethod
    def get(cls, device: torch.device, slot: int = 0) -> "_Stager":
        key = (device.index, slot)
        if key not in cls._pool:
            cls._pool[key] = cls(device)
        return cls._pool[key]

    def copy(self, path, offset: int, count: int, dst: torch.Tensor) -> None:
        """File bytes [offset, offset + count) -> dst (flat uint8 CUDA tensor
        of count bytes), on this stager's stream; the caller orders its own
        stream after it."""
        with open(path, "rb", buffering=0) as handle:
            done = 0
            turn = 0
            while done < count:
                n = min(CHUNK_BYTES, count - done)
                if self.done[turn] is not None:
                    self.done[turn].synchronize()  # the previous copy out of this buffer has finished
                got = os.preadv(handle.fileno(), [self.views[turn][:n]], offset + done)
                if got != n:
                    raise ValueError(f"truncated read at byte {offset + done} of {path}")
                with torch.cuda.stream(self.stream):
                    dst[done:done + n].copy_(self.buffers[turn][:n], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.stream)
                self.done[turn] = ev
                done += n
                turn ^= 1


def _copy_to_device(path, offset: int, count: int, dst: torch.Tensor) -> None:
    """Fill dst from the file, splitting large reads over READERS threads
    (each a contiguous part, its own pinned buffers and copy stream) so the
    storage sees several requests in flight."""
    device = dst.device
    caller = torch.cuda.current_stream(device)
    parts = max(1, min(READERS, count // (4 * CHUNK_BYTES)))
    step = -(-count // parts)
    step += -step % 4096
    spans = [(i * step, min(count, (i + 1) * step)) for i in range(parts) if i * step < count]
    stagers = [_Stager.get(device, i) for i in range(len(spans))]
    for st in stagers:
        st.stream.wait_stream(caller)  # dst may have been allocated or written on the caller's stream
    if len(spans) == 1:
        stagers[0].copy(path, offset, count, dst)
    else:
        with ThreadPoolExecutor(len(spans)) as pool:
            jobs = [pool.submit(st.copy, path, offset + a, b - a, dst[a:b]) for st, (a, b) in zip(stagers, spans)]
            for job in jobs:
                job.result()
    for st in stagers:
        caller.wait_stream(st.stream)
        dst.record_stream(st.stream)


class _Span(NamedTuple):
    """Where one tensor's bytes lie in the file."""

    dtype: str   # safetensors scalar type name
    shape: tuple
    offset: int  # absolute file offset of the first byte
    nbytes: int


class SafeTensorFile:
    """The header parsed once into per-tensor spans; every read touches only
    the requested bytes of the file."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        with self.path.open("rb") as handle:
            header_len = int.from_bytes(handle.read(8), "little")
            header = json.loads(handle.read(header_len))
        self.header = header
        self.data_offset = 8 + header_len
        self.metadata = header.get("__metadata__", {})
        self.tensors, self._spans = {}, {}
        for name, info in header.items():
            if name == "__metadata__":
                continue
            first, last = info["data_offsets"]
            self.tensors[name] = info
            self._spans[name] = _Span(info["dtype"], tuple(info["shape"]), self.data_offset + first, last - first)

    def _range(self, name: str, start_bytes: int, byte_count: int | None):
        """(info, absolute offset, byte count) of a checked byte range."""
        span = self._spans[name]
        count = span.nbytes - start_bytes if byte_count is None else byte_count
        unit = np.dtype(_DTYPES[span.dtype]).itemsize
        inside = 0 <= start_bytes and 0 <= count and start_bytes + count <= span.nbytes
        if not inside or start_bytes % unit or count % unit:
            raise ValueError(f"invalid byte range for {name}: {start_bytes}, {count}")
        return self.tensors[name], span.offset + start_bytes, count

    def raw(self, name: str, start_bytes: int = 0, byte_count: int | None = None) -> np.ndarray:
        """A tensor (shaped) or a byte range of it (flat) in host memory, one
        positional read of exactly those bytes; BF16 stays uint16 bit patterns."""
        _, offset, count = self._range(name, start_bytes, byte_count)
        span = self._spans[name]
        data = bytearray(count)
        view, got = memoryview(data), 0
        with self.path.open("rb", buffering=0) as handle:
            handle.seek(offset)
            while got < count:  # one read call returns at most ~2 GB
                n = handle.readinto(view[got:])
                if not n:
                    break
                got += n
        if got != count:
            raise ValueError(f"truncated tensor {name} in {self.path}")
        values = np.frombuffer(data, dtype=np.dtype(_DTYPES[span.dtype]))
        return values.reshape(span.shape) if start_bytes == 0 and byte_count is None else values

    def read_into(self, name: str, out: torch.Tensor, start_bytes: int = 0, byte_count: int | None = None) -> None:
        """Copy a byte range of a tensor into ``out``, a contiguous tensor
        holding exactly that many bytes (any dtype; CUDA tensors are filled
        through the pinned staging buffers)."""
        _, offset, byte_count = self._range(name, start_bytes, byte_count)
        if not out.is_contiguous():
            raise ValueError("read_into needs a contiguous tensor")
        flat = out.view(-1).view(torch.uint8) if out.numel() else out.view(torch.uint8)
        if flat.numel() != byte_count:
            raise ValueError(f"destination holds {flat.numel()} bytes, the range {byte_count}")
        if byte_count == 0:
            return
        if out.device.type == "cuda":
            _copy_to_device(self.path, offset, byte_count, flat)
            return
        with self.path.open("rb", buffering=0) as handle:
            handle.seek(offset)
            if handle.readinto(memoryview(flat.numpy())) != byte_count:
                raise ValueError(f"truncated tensor {name} in {self.path}")

    def load_slice(self, name: str, start_bytes: int, byte_count: int, device=None) -> torch.Tensor:
        """Read a byte range as a flat tensor with the stored scalar type (on
        the current CUDA device unless ``device`` says otherwise)."""
        info, _, byte_count = self._range(name, start_bytes, byte_count)
        dtype = _TORCH[info["dtype"]]
        itemsize = np.dtype(_DTYPES[info["dtype"]]).itemsize
        device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        out = torch.empty(byte_count // itemsize, dtype=dtype, device=device)
        self.read_into(name, out, start_bytes, byte_count)
        return out

    def load(self, name: str, device=None) -> torch.Tensor:
        """Read one complete tensor with its stored shape and scalar type."""
        info = self.tensors[name]
        begin, end = info["data_offsets"]
        return self.load_slice(name, 0, end - begin, device).reshape(info["shape"])
