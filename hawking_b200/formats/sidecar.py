"""`.hawking` sidecar next to a GGUF file: predecoded Q4_K scale tables (per 144-byte block the
8 sub-block pairs (d * sc, dmin * m)), keyed by each tensor's absolute file offset, plus an
optional mixed-precision tier map, under a JSON header that names the source GGUF's SHA-256.

File layout (C++ reader/writer in ``csrc/native/codecs.cpp``): magic ``DSMTL\\x01\\0\\0`` | u32 LE
header length | JSON header | entries {u64 offset | u32 n | n x f32}. The JSON header carries the
fields in the order version, source_gguf_hash, tokenizer_hash, shader_hash, bake_profile,
contents, quality, bake_device, bake_time_secs, tier_map.

Parity: crates/hawking-core/src/sidecar.rs:1-330 (SidecarHeader, SidecarCompat, SidecarWriter,
read_predec_entries, tier map), crates/hawking-core/src/kernels/mod.rs:1849-1888.
"""
from __future__ import annotations

import hashlib
import json
import os
import time
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

from .._ext import native

SIDECAR_VERSION = 1
PROFILES = ("exact", "fast", "race", "efficient")
TIER_DTYPES = {"q4_K": "Q4_K", "Q4_K": "Q4_K", "q4k": "Q4_K", "Q4K": "Q4_K",
               "q6_K": "Q6_K", "Q6_K": "Q6_K", "q6k": "Q6_K", "Q6K": "Q6_K",
               "q8_0": "Q8_0", "Q8_0": "Q8_0", "q8": "Q8_0", "Q8": "Q8_0"}


def sidecar_path_for(gguf_path: str) -> str:
    root, _ = os.path.splitext(os.fspath(gguf_path))
    return root + ".hawking"


def file_sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def make_header(gguf_hash: str, tokenizer_hash: str = "", shader_hash: str = "", profile: str = "exact",
                predec: bool = True, tier_map: Optional[List[Dict[str, str]]] = None, device: str = "",
                quality: Optional[dict] = None) -> dict:
    if profile not in PROFILES:
        raise ValueError(f"bake profile must be one of {PROFILES}")
    q = {"top1_agreement": None, "eval_prompt_count": None, "eval_mean_tokens": None, "vocab_prune_size": 0,
         "quality_gate_passed": False, "quality_gate_spec": ""}
    q.update(quality or {})
    hdr = {"version": SIDECAR_VERSION, "source_gguf_hash": gguf_hash, "tokenizer_hash": tokenizer_hash,
           "shader_hash": shader_hash, "bake_profile": profile,
           "contents": {"q4k_predec_scales": predec, "pruned_lm_head_q4k": False, "corpus_whitelist": False,
                        "tensor_offset_table": False, "mixed_quant_tier_map": tier_map is not None},
           "quality": q, "bake_device": device, "bake_time_secs": int(time.time()),
           "tier_map": {"entries": tier_map} if tier_map is not None else None}
    return hdr


def validate_tier_map(entries: Sequence[Dict[str, str]]) -> None:
    seen = set()
    for e in entries:
        if e["tensor"] in seen:
            raise ValueError(f"sidecar tier map: duplicate entry for tensor {e['tensor']!r}")
        seen.add(e["tensor"])
        if e["dtype"] not in TIER_DTYPES:
            raise ValueError(f"sidecar tier map: unsupported dtype {e['dtype']!r} (allowed: q4_K, q6_K, q8_0)")


def write(path: str, header: dict, entries: Sequence[Tuple[int, np.ndarray]]) -> None:
    if header.get("tier_map"):
        validate_tier_map(header["tier_map"]["entries"])
    native().sidecar_write(os.fspath(path), json.dumps(header, separators=(",", ":")),
                           [(int(o), np.ascontiguousarray(s, dtype=np.float32)) for o, s in entries])


def read(path: str) -> Tuple[dict, List[Tuple[int, np.ndarray]]]:
    hj, entries = native().sidecar_read(os.fspath(path))
    return json.loads(hj), [(int(o), s) for o, s in entries]


def compatibility(header: dict, gguf_hash: str, shader_hash: str = "") -> str:
    """'compatible', 'version_too_new', 'gguf_hash_mismatch' (both fatal) or
    'shader_hash_mismatch' (loadable)."""
    if int(header.get("version", 0)) > SIDECAR_VERSION:
        return "version_too_new"
    if header.get("source_gguf_hash") != gguf_hash:
        return "gguf_hash_mismatch"
    if header.get("shader_hash", "") != shader_hash:
        return "shader_hash_mismatch"
    return "compatible"


def predecode_q4k(raw: np.ndarray) -> np.ndarray:
    return native().predecode_q4k_scales(np.ascontiguousarray(raw, dtype=np.uint8))


def bake(gguf_path: str, out_path: Optional[str] = None, profile: str = "exact",
         tier_map: Optional[List[Dict[str, str]]] = None) -> str:
    """Write the sidecar of every Q4_K tensor of ``gguf_path``."""
    from .ggml import GgmlType
    from .gguf import GgufModel
    m = GgufModel(gguf_path)
    entries = [(t.offset, predecode_q4k(m.raw(name))) for name, t in m.tensors.items() if t.type == GgmlType.Q4_K]
    out = out_path or sidecar_path_for(gguf_path)
    write(out, make_header(file_sha256(gguf_path), profile=profile, tier_map=tier_map, device="cpu"), entries)
    return out


def load_predecoded(gguf_path: str, shader_hash: str = "") -> Optional[Dict[int, np.ndarray]]:
    """The predecoded tables of a compatible sidecar ({tensor offset: table}), else None."""
    p = sidecar_path_for(gguf_path)
    if not os.path.exists(p):
        return None
    header, entries = read(p)
    if not header.get("contents", {}).get("q4k_predec_scales"):
        return None
    if compatibility(header, file_sha256(gguf_path), shader_hash) in ("version_too_new", "gguf_hash_mismatch"):
        return None
    return {o: s for o, s in entries}
