"""GGUF reading (zero-copy) and writing.

The container is parsed by the C++ core (``hawking_b200._native.GgufFile``; parity with
crates/hawking-core/src/gguf.rs:218-319). Tensor payloads are exposed as read-only numpy views of
one file mapping, so loading a model to the GPU is a single host->device copy per tensor with no
intermediate buffers.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence

import numpy as np

from .._ext import native
from .ggml import LAYOUTS, GgmlType, row_bytes, type_id


@dataclass
class TensorInfo:
    name: str
    dims: List[int]        # ggml order (dims[0] contiguous)
    type: int
    offset: int            # absolute file offset of the payload
    nbytes: int

    @property
    def shape(self) -> tuple:
        """Row-major (PyTorch) shape: ggml dims reversed."""
        return tuple(reversed(self.dims))

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def type_name(self) -> str:
        return LAYOUTS[self.type].name


class GgufModel:
    """A parsed GGUF file. ``raw(name)`` returns the tensor's bytes without copying."""

    def __init__(self, path: str):
        self.path = os.fspath(path)
        self._f = native().GgufFile.open(self.path)
        self.version = self._f.version
        self.alignment = self._f.alignment
        self.metadata: Dict[str, object] = self._f.metadata()
        base = self._f.data_offset
        self.tensors: Dict[str, TensorInfo] = {}
        for name, dims, t, off, nb in self._f.tensors():
            self.tensors[name] = TensorInfo(name, list(dims), int(t), base + int(off), int(nb))
        self._map = np.memmap(self.path, dtype=np.uint8, mode="r")

    @property
    def architecture(self) -> str:
        return str(self.metadata.get("general.architecture", ""))

    def get(self, key: str, default=None):
        return self.metadata.get(key, default)

    def arch_get(self, suffix: str, default=None):
        return self.metadata.get(f"{self.architecture}.{suffix}", default)

    def raw(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        return self._map[t.offset : t.offset + t.nbytes]

    def has(self, name: str) -> bool:
        return name in self.tensors

    def dequantize(self, name: str) -> np.ndarray:
        """fp32 copy in row-major shape (CPU oracle)."""
        t = self.tensors[name]
        rows = t.n_elements // t.dims[0]
        out = native().dequantize_rows(t.type, np.ascontiguousarray(self.raw(name)), rows, t.dims[0])
        return out.reshape(t.shape)


class GgufBuilder:
    """Collects metadata and tensors, then writes a GGUF v3 file atomically."""

    def __init__(self, arch: str, alignment: int = 32):
        self._w = native().GgufWriter(alignment)
        self.arch = arch
        self.set("general.architecture", arch)

    def set(self, key: str, value, kind: Optional[int] = None) -> "GgufBuilder":
        self._w.set(key, value, -1 if kind is None else kind)
        return self

    def set_f32(self, key: str, value: float) -> "GgufBuilder":
        return self.set(key, float(value), 6)

    def arch_set(self, suffix: str, value, kind: Optional[int] = None) -> "GgufBuilder":
        return self.set(f"{self.arch}.{suffix}", value, kind)

    def add(self, name: str, array: np.ndarray, qtype=GgmlType.F32, threads: int = 8) -> "GgufBuilder":
        """Quantise a row-major fp32 array into ``qtype`` and add it."""
        t = type_id(qtype)
        a = np.ascontiguousarray(array, dtype=np.float32)
        cols = a.shape[-1]
        rows = a.size // cols
        data = native().quantize_rows(t, a.reshape(rows, cols), threads)
        dims = list(reversed(a.shape))
        self._w.add_tensor(name, dims, t, data.reshape(-1))
        return self

    def add_raw(self, name: str, shape: Sequence[int], qtype, data: np.ndarray) -> "GgufBuilder":
        t = type_id(qtype)
        dims = list(reversed(list(shape)))
        self._w.add_tensor(name, dims, t, np.ascontiguousarray(data, dtype=np.uint8).reshape(-1))
        return self

    def write(self, path: str) -> str:
        self._w.write(os.fspath(path))
        return os.fspath(path)
