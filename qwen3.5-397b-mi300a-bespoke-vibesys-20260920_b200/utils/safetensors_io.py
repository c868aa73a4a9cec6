"""A small, thread-safe safetensors reader and writer.

The published checkpoint is 94 shards with no index file, so the reader scans every shard's
header once and keeps a name -> (file, dtype, shape, byte range) directory. Reads use
``os.pread`` on a shared file descriptor, so many threads can load different tensors (or
different row ranges of one tensor, for tensor-parallel shards) at once. Reference behaviour:
``weights.py:30-79`` (``Checkpoint``) and ``model.py:807-833`` (``_Reader``).

File format: 8-byte little-endian header length, a JSON header mapping each tensor name to
``{"dtype", "shape", "data_offsets": [begin, end]}`` (offsets relative to the end of the
header), then the raw little-endian data.
"""

from __future__ import annotations

import json
import os
import struct
import threading
from dataclasses import dataclass

import numpy as np
import torch

_DTYPES = {
    "BF16": (torch.bfloat16, 2),
    "F16": (torch.float16, 2),
    "F32": (torch.float32, 4),
    "F64": (torch.float64, 8),
    "U8": (torch.uint8, 1),
    "I8": (torch.int8, 1),
    "I32": (torch.int32, 4),
    "I64": (torch.int64, 8),
    "BOOL": (torch.bool, 1),
    "F8_E4M3": (torch.float8_e4m3fn, 1),
}
_NAMES = {v[0]: k for k, v in _DTYPES.items()}


@dataclass(frozen=True)
class Entry:
    path: str
    dtype: str
    shape: tuple[int, ...]
    begin: int  # absolute byte offset in the file
    end: int

    @property
    def nbytes(self) -> int:
        return self.end - self.begin


class Checkpoint:
    """Directory of every tensor in every ``*.safetensors`` file of ``path``."""

    def __init__(self, path: str) -> None:
        self.path = path
        self.entries: dict[str, Entry] = {}
        self._fds: dict[str, int] = {}
        self._lock = threading.Lock()
        files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
        if not files:
            raise FileNotFoundError(f"no .safetensors files under {path}")
        for name in files:
            full = os.path.join(path, name)
            with open(full, "rb") as f:
                (n,) = struct.unpack("<Q", f.read(8))
                header = json.loads(f.read(n))
            base = 8 + n
            for key, meta in header.items():
                if key == "__metadata__":
                    continue
                b, e = meta["data_offsets"]
                self.entries[key] = Entry(full, meta["dtype"], tuple(meta["shape"]), base + b, base + e)

    def has(self, name: str) -> bool:
        return name in self.entries

    def names(self, prefix: str = "") -> list[str]:
        return [k for k in self.entries if k.startswith(prefix)]

    def shape(self, name: str) -> tuple[int, ...]:
        return self.entries[name].shape

    def _fd(self, path: str) -> int:
        with self._lock:
            fd = self._fds.get(path)
            if fd is None:
                fd = os.open(path, os.O_RDONLY)
                self._fds[path] = fd
            return fd

    def _pread(self, e: Entry, offset: int, nbytes: int) -> bytearray:
        buf = bytearray(nbytes)
        fd = self._fd(e.path)
        view = memoryview(buf)
        got = 0
        while got < nbytes:
            chunk = os.preadv(fd, [view[got:]], e.begin + offset + got)
            if chunk <= 0:
                raise IOError(f"short read in {e.path}")
            got += chunk
        return buf

    def load(self, name: str, rows: tuple[int, int] | None = None) -> torch.Tensor:
        """Read tensor ``name`` (optionally only rows ``[r0, r1)`` of dim 0) into CPU memory."""
        e = self.entries[name]
        dtype, size = _DTYPES[e.dtype]
        shape = list(e.shape)
        row_bytes = size * int(np.prod(shape[1:])) if len(shape) > 1 else size
        if rows is None:
            r0, r1 = 0, shape[0] if shape else 1
        else:
            r0, r1 = rows
        if not shape:
            buf = self._pread(e, 0, size)
            return torch.frombuffer(buf, dtype=dtype).reshape(())
        buf = self._pread(e, r0 * row_bytes, (r1 - r0) * row_bytes)
        out = torch.frombuffer(buf, dtype=dtype) if len(buf) else torch.empty(0, dtype=dtype)
        return out.reshape([r1 - r0] + shape[1:])

    def close(self) -> None:
        with self._lock:
            for fd in self._fds.values():
                os.close(fd)
            self._fds.clear()


def save_file(tensors: dict[str, torch.Tensor], path: str, metadata: dict[str, str] | None = None) -> None:
    """Write ``tensors`` as one safetensors file (tensors are made contiguous on CPU)."""
    header: dict = {}
    if metadata:
        header["__metadata__"] = dict(metadata)
    off = 0
    blobs = []
    for name in sorted(tensors):
        t = tensors[name].detach().to("cpu").contiguous()
        raw = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""  # 0-dim too
        header[name] = {"dtype": _NAMES[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
