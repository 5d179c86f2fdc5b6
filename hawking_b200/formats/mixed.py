"""HGRAV* sub-2-bit codecs (binary / binary+Rice residual / low-rank / uniform group) and the
mixed artifact writer for the benchmark's Qwen3-Next configuration (<= 1.5 complete BPW:
routed experts binary or ternary with per-64 fp16 group scales, attention and shared expert Q4).

Parity: docs/QWEN80_MIXED_1P5_PACKED_FORMAT.md (envelope, codec layouts, HQ80M15 catalog).
The ternary and Q4 points are HGRAVU01 with bits 2 and 4 (extensions of the same envelope family,
as the benchmark recipe requires group size 64 for the experts).
"""
from __future__ import annotations

import numpy as np

from .._ext import native

MAGICS = (b"HGRAVB01", b"HGRAVR02", b"HGRAVS01", b"HGRAVU01")


def header(payload: np.ndarray):
    magic, hdr, body_off, body_bytes = native().mixed_header(np.ascontiguousarray(payload, dtype=np.uint8))
    return bytes(magic), hdr, int(body_off), int(body_bytes)


def decode(payload: np.ndarray) -> np.ndarray:
    """Dense fp32 reconstruction [rows, cols] (CPU oracle)."""
    return native().mixed_decode(np.ascontiguousarray(payload, dtype=np.uint8))


def encode_binary(w: np.ndarray, group: int = 64) -> np.ndarray:
    return native().encode_hgravb01(np.ascontiguousarray(w, np.float32), group)


def encode_uniform(w: np.ndarray, bits: int, group: int = 64) -> np.ndarray:
    return native().encode_hgravu01(np.ascontiguousarray(w, np.float32), group, bits)


def encode_binary_residual(w: np.ndarray, group: int = 128, ratio: float = 0.02, rice_k: int = 5) -> np.ndarray:
    return native().encode_hgravr02(np.ascontiguousarray(w, np.float32), group, ratio, rice_k)


def encode_low_rank(left: np.ndarray, right: np.ndarray, bits: int = 3, group: int = 64) -> np.ndarray:
    return native().encode_hgravs01(np.ascontiguousarray(left, np.float32), np.ascontiguousarray(right, np.float32),
                                    group, bits)


def payload_bits(payload: np.ndarray, elements: int) -> float:
    return payload.size * 8.0 / elements
