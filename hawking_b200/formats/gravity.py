"""`.gravity` packed artifacts: single shards, multi-shard directories and the mixed catalog.

The byte contract lives in the C++ core (``hawking_b200._native.GravityShard`` /
``GravityWriter``; parity with crates/hawking-core/src/artifact.rs:114-446 and
crates/hawking-core/src/gravity.rs:877-990). Payloads are exposed as zero-copy numpy views of the
shard mapping. Plain ggml codecs (``native.*``, ``ggml.*``) load as GGUF-equivalent tensors; the
HGRAV* mixed codecs are decoded by ``formats.mixed``.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np

from .._ext import native
from .ggml import LAYOUTS

INDEX_NAME = "model.gravity.index.json"


@dataclass
class GravityTensorInfo:
    name: str
    codec: str
    offset: int
    nbytes: int
    sha256: str
    shape: List[int]
    elements: int
    shard: str = ""

    @property
    def ggml_type(self) -> int:
        return native().gravity_codec_to_ggml(self.codec)


def is_gravity(path: str) -> bool:
    """Magic sniff (a shard file, or a directory with an index / shards)."""
    if os.path.isdir(path):
        return os.path.exists(os.path.join(path, INDEX_NAME)) or any(
            f.endswith(".gravity") for f in os.listdir(path))
    try:
        with open(path, "rb") as f:
            return f.read(8) == b"GRAVITY\0"
    except OSError:
        return False


class GravityShardFile:
    def __init__(self, path: str):
        self.path = os.fspath(path)
        self._s = native().GravityShard.open(self.path)
        self.header = self._s.header()
        self.tensors: Dict[str, GravityTensorInfo] = {}
        for name, codec, off, nb, sha, shape, el in self._s.tensors():
            self.tensors[name] = GravityTensorInfo(name, codec, off, nb, sha, list(shape), el, self.path)

    @property
    def architecture(self):
        return self.header.get("architecture", {})

    def raw(self, name: str) -> np.ndarray:
        return self._s.raw(name)

    def descriptor(self, name: str) -> dict:
        return self._s.descriptor(name)

    def verify(self) -> dict:
        return self._s.verify()

    def verify_tensor(self, name: str) -> bool:
        return self._s.verify_tensor(name)

    def dequantize(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        raw = np.ascontiguousarray(self.raw(name))
        if t.ggml_type >= 0:
            cols = t.shape[-1]
            rows = t.elements // cols
            return native().dequantize_rows(t.ggml_type, raw, rows, cols).reshape(t.shape)
        from .mixed import decode
        return decode(raw).reshape(t.shape)


class GravityModel:
    """A shard file or a directory (index + shards). Admission verifies every payload sha256
    once (``verify_on_open``); a mismatch is a hard error, never a silent fallback."""

    def __init__(self, path: str, verify_on_open: bool = False):
        self.path = os.fspath(path)
        self.shards: Dict[str, GravityShardFile] = {}
        self.index: dict = {}
        if os.path.isdir(self.path):
            ip = os.path.join(self.path, INDEX_NAME)
            if os.path.exists(ip):
                with open(ip) as f:
                    self.index = json.load(f)
                files = sorted(set(self.index.get("weight_map", {}).values()))
            else:
                files = sorted(f for f in os.listdir(self.path) if f.endswith(".gravity"))
            for fn in files:
                self.shards[fn] = GravityShardFile(os.path.join(self.path, fn))
        else:
            self.shards[os.path.basename(self.path)] = GravityShardFile(self.path)
        self.tensors: Dict[str, GravityTensorInfo] = {}
        self._owner: Dict[str, GravityShardFile] = {}
        for s in self.shards.values():
            for n, t in s.tensors.items():
                if n in self.tensors:
                    raise RuntimeError(f"gravity: tensor {n} appears in two shards")
                self.tensors[n] = t
                self._owner[n] = s
        if self.index.get("shard_sha256"):
            want = self.index["shard_sha256"]
            names = sorted(want)
            for fn, got in zip(names, files_sha256([os.path.join(self.path, fn) for fn in names])):
                if got != want[fn]:
                    raise RuntimeError(f"gravity: shard {fn} sha256 mismatch")
            # every byte of every shard is covered by its digest: the per-payload pass adds nothing
            verify_on_open = False
        if verify_on_open:
            for n in self.tensors:
                if not self._owner[n].verify_tensor(n):
                    raise RuntimeError(f"gravity: payload sha256 mismatch for {n}")
        first = next(iter(self.shards.values()))
        self.header = first.header

    @property
    def architecture(self) -> str:
        a = self.index.get("architecture") or self.header.get("architecture", {})
        return a.get("name", "") if isinstance(a, dict) else str(a)

    @property
    def metadata(self) -> dict:
        return self.header.get("gguf_metadata", {})

    def raw(self, name: str) -> np.ndarray:
        return self._owner[name].raw(name)

    def descriptor(self, name: str) -> dict:
        return self._owner[name].descriptor(name)

    def has(self, name: str) -> bool:
        return name in self.tensors

    def dequantize(self, name: str) -> np.ndarray:
        return self._owner[name].dequantize(name)

    def verify(self) -> Dict[str, dict]:
        return {fn: s.verify() for fn, s in self.shards.items()}


def write_shard(path: str, tensors: List[dict], meta: Optional[dict] = None) -> dict:
    """tensors: [{"name", "codec", "shape", "data": uint8 ndarray, ...extra descriptor fields}].
    Writes atomically; returns the header. ``elements`` defaults to prod(shape)."""
    w = native().GravityWriter(meta or {})
    for t in tensors:
        d = {k: v for k, v in t.items() if k != "data"}
        if "elements" not in d and "shape" in d:
            d["elements"] = int(np.prod(d["shape"]))
        w.add(d, np.ascontiguousarray(t["data"], dtype=np.uint8).reshape(-1))
    return w.write(os.fspath(path))


def file_sha256(path: str) -> str:
    """sha256 of a file through a read-only mapping (the native hash releases the GIL, so several
    files hash in parallel on threads)."""
    if os.path.getsize(path) == 0:
        return native().sha256_hex(np.zeros(0, dtype=np.uint8))
    return native().sha256_hex(np.memmap(path, dtype=np.uint8, mode="r"))


def files_sha256(paths: List[str]) -> List[str]:
    from concurrent.futures import ThreadPoolExecutor
    with ThreadPoolExecutor(max_workers=max(1, min(len(paths), os.cpu_count() or 1))) as ex:
        return list(ex.map(file_sha256, paths))


def write_index(directory: str, weight_map: Dict[str, str], architecture: dict, tensor_dtypes: Dict[str, str]):
    files = sorted(set(weight_map.values()))
    shard_sha = dict(zip(files, files_sha256([os.path.join(directory, fn) for fn in files])))
    idx = {"weight_map": weight_map, "tensor_dtypes": tensor_dtypes, "shard_sha256": shard_sha,
           "architecture": architecture}
    tmp = os.path.join(directory, INDEX_NAME + ".tmp")
    with open(tmp, "w") as f:
        f.write(native().canonical_json(idx))
    os.replace(tmp, os.path.join(directory, INDEX_NAME))
    return idx


GGML_CODECS = {0: "native.f32", 1: "native.f16", 30: "native.bf16", 11: "ggml.q3_k", 12: "ggml.q4_k",
               13: "ggml.q5_k", 14: "ggml.q6_k", 8: "ggml.q8_0", 6: "ggml.q5_0", 2: "ggml.q4_0"}


def codec_for_ggml(t: int) -> str:
    return GGML_CODECS[int(t)]
