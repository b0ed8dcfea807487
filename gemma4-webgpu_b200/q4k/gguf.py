"""GGUF v3 reader: the file's metadata and tensor table, and raw tensor bytes
for the device -- the host side that feeds real Q4_K tensors to libq4k.

Follows the reference parser (src/gguf.ts:11-101): little-endian header
(magic "GGUF", version, tensor count, key/value count), typed key/value
metadata (value types 0-12, arrays of any of them), a tensor table (name,
dims with ne0 fastest, type, offset) and tensor data starting at the next
32-byte boundary after the table (gguf.ts:98-99 uses a fixed alignment of
32).  Tensor byte sizes follow tensorByteSize (gguf.ts:383-395).

Unlike the reference, nothing is dequantized on the host: a Q4_K matrix is
handed to the device as the file stores it (M = dims[1] rows of N = dims[0]
columns, the engine's {M = out, N = in} binding, src/engine.ts:493), and the
GPU reproduces the reference's f16 weights itself (q4k_dequant_f16 exposes
them for a weight-probe comparison, src/diagnostics/weight-probe.ts:60-162).
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF"
ALIGNMENT = 32

# tensor type ids and their block geometry (elements per block, bytes per block)
TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q5_K, TYPE_Q6_K, TYPE_BF16 = 0, 1, 8, 12, 13, 14, 30
_BLOCKS = {
    TYPE_F32: (1, 4),
    TYPE_F16: (1, 2),
    TYPE_Q8_0: (32, 34),
    TYPE_Q4_K: (256, 144),
    TYPE_Q5_K: (256, 176),
    TYPE_Q6_K: (256, 210),
    TYPE_BF16: (1, 2),
}
TYPE_NAMES = {TYPE_F32: "F32", TYPE_F16: "F16", TYPE_Q8_0: "Q8_0", TYPE_Q4_K: "Q4_K", TYPE_Q5_K: "Q5_K",
              TYPE_Q6_K: "Q6_K", TYPE_BF16: "BF16"}


class GGUFError(ValueError):
    pass


@dataclass
class GGUFTensor:
    name: str
    dims: tuple[int, ...]  # ne0 (fastest) first
    type: int
    offset: int            # relative to the data section

    @property
    def count(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        """tensorByteSize (src/gguf.ts:383-395)."""
        if self.type not in _BLOCKS:
            raise GGUFError(f"unknown tensor type {self.type} ({self.name})")
        per, size = _BLOCKS[self.type]
        if self.count % per:
            raise GGUFError(f"{self.name}: {self.count} elements is not a whole number of blocks")
        return self.count // per * size

    @property
    def matrix_shape(self) -> tuple[int, int]:
        """(M rows, N columns) of a 2-D weight: N = dims[0], M = dims[1]."""
        if len(self.dims) != 2:
            raise GGUFError(f"{self.name} is not a matrix: dims {self.dims}")
        return self.dims[1], self.dims[0]


@dataclass
class GGUFFile:
    """A parsed GGUF file (or buffer); tensor bytes are views into it."""

    version: int
    kv: dict[str, Any]
    tensors: list[GGUFTensor]
    data_offset: int
    _buf: Any = field(repr=False, default=None)

    @property
    def by_name(self) -> dict[str, GGUFTensor]:
        return {t.name: t for t in self.tensors}

    def tensor_bytes(self, t: GGUFTensor | str) -> np.ndarray:
        """The tensor's raw bytes (uint8 view of the file, no copy)."""
        if isinstance(t, str):
            t = self.by_name[t]
        start = self.data_offset + t.offset
        end = start + t.nbytes
        if end > len(self._buf):
            raise GGUFError(f"{t.name}: data [{start}, {end}) past the end of the file ({len(self._buf)} bytes)")
        return np.frombuffer(self._buf, dtype=np.uint8, count=t.nbytes, offset=start)

    def q6k_matrix(self, name: str) -> tuple[np.ndarray, int, int]:
        """A Q6_K matrix's GGUF bytes: (bytes [M, N/256*210], M, N)."""
        t = self.by_name[name]
        if t.type != TYPE_Q6_K:
            raise GGUFError(f"{name} is {TYPE_NAMES.get(t.type, t.type)}, not Q6_K")
        M, N = t.matrix_shape
        if N % 256:
            raise GGUFError(f"{name}: N={N} is not a multiple of 256")
        return self.tensor_bytes(t).reshape(M, N // 256 * 210), M, N

    def q5k_table(self, name: str, layers: int) -> tuple[np.ndarray, int]:
        """A Q5_K per-layer embedding table (per_layer_token_embd) as
        q4k_ple_stage1 takes it: (bytes [vocab, layers*176], vocab).  GGUF
        stores it as [ne0 = layers*256, ne1 = vocab]: row v is `layers`
        consecutive super-blocks, block L being layer L's 256 values
        (src/engine.ts:681-702)."""
        t = self.by_name[name]
        if t.type != TYPE_Q5_K:
            raise GGUFError(f"{name} is {TYPE_NAMES.get(t.type, t.type)}, not Q5_K")
        vocab, width = t.matrix_shape
        if width != layers * 256:
            raise GGUFError(f"{name}: row length {width} is not layers*256 = {layers * 256}")
        return self.tensor_bytes(t).reshape(vocab, layers * 176), vocab

    def q4k_matrix(self, name: str) -> tuple[np.ndarray, int, int]:
        """A Q4_K matrix as libq4k takes it: (bytes [M, N/256*144], M, N)."""
        t = self.by_name[name]
        if t.type != TYPE_Q4_K:
            raise GGUFError(f"{name} is {TYPE_NAMES.get(t.type, t.type)}, not Q4_K")
        M, N = t.matrix_shape
        if N % 256:
            raise GGUFError(f"{name}: N={N} is not a multiple of 256")
        return self.tensor_bytes(t).reshape(M, N // 256 * 144), M, N


class _Cursor:
    def __init__(self, buf):
        self.buf = buf
        self.off = 0

    def take(self, fmt: str):
        size = struct.calcsize(fmt)
        if self.off + size > len(self.buf):
            raise GGUFError("truncated GGUF header")
        v = struct.unpack_from(fmt, self.buf, self.off)
        self.off += size
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.take("<Q")
        if self.off + n > len(self.buf):
            raise GGUFError("truncated GGUF string")
        s = bytes(self.buf[self.off:self.off + n]).decode("utf-8")
        self.off += n
        return s

    def value(self, vtype: int):
        # readValue (src/gguf.ts:53-81)
        simple = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 10: "<Q", 11: "<q", 12: "<d"}
        if vtype in simple:
            return self.take(simple[vtype])
        if vtype == 7:
            return self.take("<B") != 0
        if vtype == 8:
            return self.string()
        if vtype == 9:
            etype = self.take("<I")
            n = self.take("<Q")
            return [self.value(etype) for _ in range(n)]
        raise GGUFError(f"unknown metadata value type {vtype}")


def parse(buf) -> GGUFFile:
    """Parse GGUF bytes (bytes, bytearray, memoryview or mmap)."""
    c = _Cursor(buf)
    magic = c.take("<I")
    if magic != GGUF_MAGIC:
        raise GGUFError(f"invalid GGUF magic 0x{magic:x}")
    version = c.take("<I")
    n_tensors = c.take("<Q")
    n_kv = c.take("<Q")
    kv: dict[str, Any] = {}
    for _ in range(n_kv):
        key = c.string()
        kv[key] = c.value(c.take("<I"))
    tensors = []
    for _ in range(n_tensors):
        name = c.string()
        n_dims = c.take("<I")
        dims = tuple(c.take("<Q") for _ in range(n_dims))
        ttype = c.take("<I")
        offset = c.take("<Q")
        tensors.append(GGUFTensor(name, dims, ttype, offset))
    data_offset = (c.off + ALIGNMENT - 1) // ALIGNMENT * ALIGNMENT
    return GGUFFile(version, kv, tensors, data_offset, buf)


def open_gguf(path: str | os.PathLike) -> GGUFFile:
    """Memory-map and parse a GGUF file (tensor bytes are read lazily)."""
    with open(Path(path), "rb") as f:
        mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    return parse(mm)


def upload_q4k(f: GGUFFile, name: str, device) -> tuple["torch.Tensor", int, int]:  # noqa: F821
    """Copy a Q4_K matrix's bytes to `device` unchanged: (tensor, M, N)."""
    import torch

    raw, M, N = f.q4k_matrix(name)
    return torch.from_numpy(np.array(raw)).to(device), M, N


def upload_q6k(f: GGUFFile, name: str, ctx) -> tuple["torch.Tensor", int, int]:  # noqa: F821
    """A Q6_K matrix into the device layout on ctx's device (copy the GGUF
    bytes, then q4k_q6k_repack): (tensor, M, N)."""
    import torch

    raw, M, N = f.q6k_matrix(name)
    src = torch.from_numpy(np.array(raw)).to(ctx.device)
    return ctx.q6k_repack(src, M, N), M, N
