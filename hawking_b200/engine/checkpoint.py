"""Sequence checkpoint / resume: paged-KV snapshots, a disk prefix cache and recurrent-state
snapshots.

``save_sequence`` writes one sequence's cached tokens and their K/V rows (gathered from its paged
blocks in logical order) to a single file; ``load_sequence`` allocates fresh blocks for a new
sequence id and scatters the rows back, so decoding continues exactly where it stopped. Files are
written atomically (tmp + rename) and carry a SHA-256 of the payload that is checked on load (a
corrupt or truncated file is refused, never half-loaded).

File layout (little endian): b"HKKVSNP1" | u32 header_len | canonical JSON header | payload.
The header holds the token ids, the cache geometry (layers, kv heads, head dim, dtype) and the
payload digest; the payload is K then V, each [n_tokens, layers, kv_heads, head_dim] bf16.

``PrefixDiskCache`` keeps such snapshots in a directory keyed by the rolling SHA-256 of the token
prefix and finds the longest cached prefix of a new prompt (LRU by file time, bounded count).

``save_recurrent`` / ``load_recurrent`` do the same for a hybrid model's fixed-size recurrent state
(DeltaNet state and conv state of one sequence slot).

Parity: crates/hawking-core/src/cache/prefill_disk.rs:1-45 (DSPRFKV2 files keyed by a rolling sha256 of
the token prefix, longest-prefix lookup, LRU), crates/hawking-core/src/engine.rs:423-445
(save_checkpoint / load_checkpoint / fork_state), crates/hawking-core/src/model/rwkv7.rs:206-220
(DSSSMV1 fixed-size state), crates/hawking-core/src/artifact.rs:332-367 (atomic tmp + rename).
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

MAGIC_KV = b"HKKVSNP1"
MAGIC_STATE = b"HKRSTAT1"


def _atomic_write(path: str, magic: bytes, header: dict, payload: bytes):
    h = json.dumps(header, sort_keys=True, separators=(",", ":")).encode()
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(magic)
        f.write(struct.pack("<I", len(h)))
        f.write(h)
        f.write(payload)
    os.replace(tmp, path)


def _read(path: str, magic: bytes) -> Tuple[dict, bytes]:
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 12 or data[:8] != magic:
        raise ValueError(f"{path}: not a {magic.decode()} file")
    (hl,) = struct.unpack("<I", data[8:12])
    if 12 + hl > len(data):
        raise ValueError(f"{path}: header runs past end of file")
    header = json.loads(data[12:12 + hl])
    payload = data[12 + hl:]
    if len(payload) != header["payload_bytes"]:
        raise ValueError(f"{path}: payload truncated ({len(payload)} of {header['payload_bytes']} bytes)")
    if hashlib.sha256(payload).hexdigest() != header["payload_sha256"]:
        raise ValueError(f"{path}: payload digest mismatch")
    return header, payload


def _token_slots(kv, seq_id: int, n: int) -> torch.Tensor:
    return torch.tensor(kv.bm.slots(seq_id, 0, n), dtype=torch.int64, device=kv.k.device)


def _token_view(cache: torch.Tensor) -> torch.Tensor:
    """[layers, blocks, kvh, bs, hd] viewed as [blocks, bs, layers, kvh, hd] (same storage)."""
    return cache.permute(1, 3, 0, 2, 4)


def _gather(cache: torch.Tensor, slots: torch.Tensor, bs: int) -> torch.Tensor:
    """Rows of the given token slots: [n, layers, kvh, hd]."""
    return _token_view(cache)[slots // bs, slots % bs]


def save_sequence(kv, seq_id: int, tokens: Sequence[int], path: str) -> dict:
    """Snapshot the first len(tokens) cached positions of ``seq_id``."""
    n = len(tokens)
    if kv.bm.num_tokens(seq_id) < n:
        raise ValueError("sequence holds fewer cached tokens than requested")
    slots = _token_slots(kv, seq_id, n)
    k = _gather(kv.k, slots, kv.block_size).contiguous().cpu()
    v = _gather(kv.v, slots, kv.block_size).contiguous().cpu()
    payload = k.view(torch.uint8).numpy().tobytes() + v.view(torch.uint8).numpy().tobytes()
    header = {"schema": "hawking_b200.kv_snapshot.v1", "tokens": [int(t) for t in tokens],
              "layers": kv.layers, "kv_heads": kv.nkv, "head_dim": kv.hd, "dtype": "bf16",
              "payload_bytes": len(payload), "payload_sha256": hashlib.sha256(payload).hexdigest()}
    _atomic_write(path, MAGIC_KV, header, payload)
    return header


def load_sequence(kv, seq_id: int, path: str) -> List[int]:
    """Restore a snapshot into the (new) sequence ``seq_id``; returns its token ids."""
    header, payload = _read(path, MAGIC_KV)
    if (header["layers"], header["kv_heads"], header["head_dim"]) != (kv.layers, kv.nkv, kv.hd):
        raise ValueError("snapshot geometry does not match this cache")
    tokens = header["tokens"]
    n = len(tokens)
    if not kv.bm.reserve(seq_id, n):
        raise RuntimeError("KV pool exhausted while restoring a snapshot")
    shape = (n, kv.layers, kv.nkv, kv.hd)
    half = len(payload) // 2
    k = torch.frombuffer(bytearray(payload[:half]), dtype=torch.bfloat16).view(shape).to(kv.k.device)
    v = torch.frombuffer(bytearray(payload[half:]), dtype=torch.bfloat16).view(shape).to(kv.k.device)
    slots = _token_slots(kv, seq_id, n)
    blk, off = slots // kv.block_size, slots % kv.block_size
    _token_view(kv.k)[blk, off] = k
    _token_view(kv.v)[blk, off] = v
    kv.sync_tables([seq_id])
    return tokens


class PrefixDiskCache:
    """Directory of KV snapshots keyed by the SHA-256 of each cached token prefix."""

    def __init__(self, directory: str, max_entries: int = 64):
        self.dir = directory
        self.max_entries = max_entries
        os.makedirs(directory, exist_ok=True)

    @staticmethod
    def key(tokens: Sequence[int]) -> str:
        return hashlib.sha256(np.asarray(tokens, dtype=np.int32).tobytes()).hexdigest()

    def _path(self, tokens) -> str:
        return os.path.join(self.dir, self.key(tokens) + ".hkkv")

    def store(self, kv, seq_id: int, tokens: Sequence[int]) -> str:
        p = self._path(tokens)
        save_sequence(kv, seq_id, tokens, p)
        self._evict()
        return p

    def longest_prefix(self, tokens: Sequence[int], granularity: int = 1) -> Optional[Tuple[int, str]]:
        """Length and file of the longest cached prefix of ``tokens`` (checked from the longest)."""
        for n in range(len(tokens), 0, -granularity):
            p = self._path(tokens[:n])
            if os.path.exists(p):
                os.utime(p)  # LRU touch
                return n, p
        return None

    def _evict(self):
        files = sorted((os.path.getmtime(os.path.join(self.dir, f)), f) for f in os.listdir(self.dir)
                       if f.endswith(".hkkv"))
        for _, f in files[:max(0, len(files) - self.max_entries)]:
            os.remove(os.path.join(self.dir, f))


def save_recurrent(states: Sequence[torch.Tensor], slot: int, path: str, meta: Optional[dict] = None) -> dict:
    """Snapshot slot ``slot`` of each per-layer state tensor ([layers, slots, ...] each)."""
    parts = [s[:, slot].contiguous().cpu() for s in states]
    payload = b"".join(p.view(torch.uint8).numpy().tobytes() for p in parts)
    header = {"schema": "hawking_b200.recurrent_state.v1", "shapes": [list(p.shape) for p in parts],
              "dtypes": [str(p.dtype) for p in parts], "meta": meta or {},
              "payload_bytes": len(payload), "payload_sha256": hashlib.sha256(payload).hexdigest()}
    _atomic_write(path, MAGIC_STATE, header, payload)
    return header


def load_recurrent(states: Sequence[torch.Tensor], slot: int, path: str) -> dict:
    header, payload = _read(path, MAGIC_STATE)
    off = 0
    for s, shape in zip(states, header["shapes"]):
        if list(s[:, slot].shape) != shape:
            raise ValueError("recurrent-state snapshot geometry does not match")
        nbytes = int(np.prod(shape)) * s.element_size()
        t = torch.frombuffer(bytearray(payload[off:off + nbytes]), dtype=s.dtype).view(shape)
        s[:, slot].copy_(t.to(s.device))
        off += nbytes
    return header["meta"]
