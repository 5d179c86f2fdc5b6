"""Fixed-header tensor codecs of the `.gravity` family (parse / decode / matvec oracles in C++,
``csrc/native/codecs.cpp``) with an independent NumPy restatement used to cross-check them.

* ``GLM52CPK`` product quantisation (codebooks per sub-space, MSB-first indices)
* ``LLM52RPK`` additive residual PQ (every stage spans the whole chunk)
* ``GLM52AAP`` activation-aware low rank (input or output side basis)
* ``HQ30G1B1`` complete binary, ``HQ30UQ4`` uniform 4-bit, ``HQ30GR2`` binary + sparse fp16 residual

Parity: crates/hawking-core/src/artifact_pq.rs:1-420, crates/hawking-core/src/artifact_aap.rs:4-164,
crates/hawking-core/src/model/qwen_complete_binary/mod.rs:39-80, :137-430, uniform_q4.rs:1-60.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import numpy as np

from .._ext import native

MAGICS = {
    b"GLM52CPK": "pq",
    b"LLM52RPK": "residual_pq",
    b"GLM52AAP": "activation_aware",
    b"HQ30G1B1": "complete_binary",
    b"HQ30UQ4\0": "uniform_q4",
    b"HQ30GR2\0": "binary_residual",
}


def _u8(payload) -> np.ndarray:
    return np.ascontiguousarray(np.frombuffer(payload, dtype=np.uint8) if isinstance(payload, (bytes, bytearray))
                                else payload, dtype=np.uint8)


def kind(payload) -> str:
    """Codec name of a payload from its magic (KeyError if unknown)."""
    return MAGICS[bytes(_u8(payload)[:8])]


def header(payload) -> dict:
    k = kind(payload)
    n = native()
    a = _u8(payload)
    return {"pq": n.pq_header, "residual_pq": n.rpq_header, "activation_aware": n.aap_header,
            "complete_binary": n.hq30_binary_header, "uniform_q4": n.hq30_uq4_header,
            "binary_residual": n.hq30_residual_header}[k](a)


def decode(payload) -> np.ndarray:
    """Dense fp32 tensor: [rows, cols] for the PQ/AAP codecs, the header's shape for HQ30."""
    k = kind(payload)
    n = native()
    a = _u8(payload)
    if k == "pq":
        return n.pq_decode(a)
    if k == "residual_pq":
        return n.rpq_decode(a)
    if k == "activation_aware":
        return n.aap_decode(a)
    h = header(a)
    flat = {"complete_binary": n.hq30_binary_decode, "uniform_q4": n.hq30_uq4_decode,
            "binary_residual": n.hq30_residual_decode}[k](a)
    return flat.reshape(h["shape"])


def matvec_f64(payload, x: np.ndarray) -> np.ndarray:
    k = kind(payload)
    n = native()
    a = _u8(payload)
    x = np.ascontiguousarray(x, dtype=np.float32)
    if k == "pq":
        return n.pq_matvec_f64(a, x)
    if k == "residual_pq":
        return n.rpq_matvec_f64(a, x)
    if k == "activation_aware":
        return n.aap_matvec_f64(a, x)
    return decode(a).reshape(-1, x.shape[0]).astype(np.float64) @ x.astype(np.float64)


# ---- encoders (codebooks / factors given; used by tests and converters) ----
def encode_pq(codebooks: np.ndarray, indices: np.ndarray, bits: int, seed: int = 0) -> np.ndarray:
    """codebooks [s, card, sub], indices [rows, nchunk, s] -> GLM52CPK payload."""
    s, card, sub = codebooks.shape
    rows, nchunk, s2 = indices.shape
    assert s2 == s
    d = s * sub
    return native().pq_encode(d, s, sub, card, rows, nchunk * d, nchunk, seed, bits,
                              codebooks.astype(np.float16).view(np.uint16).reshape(-1),
                              indices.astype(np.uint32).reshape(-1))


def encode_residual_pq(codebooks: np.ndarray, indices: np.ndarray, bits: int, seed: int = 0) -> np.ndarray:
    """codebooks [stages, card, d], indices [rows, nchunk, stages] -> LLM52RPK payload."""
    stages, card, d = codebooks.shape
    rows, nchunk, st2 = indices.shape
    assert st2 == stages
    return native().rpq_encode(d, stages, card, rows, nchunk * d, nchunk, seed, bits,
                               codebooks.astype(np.float16).view(np.uint16).reshape(-1),
                               indices.astype(np.uint32).reshape(-1))


def encode_aap(coeff: np.ndarray, basis: np.ndarray, side: str = "input", basis_layer: int = 0) -> np.ndarray:
    """Input side: W = coeff [rows, rank] @ basis [cols, rank]^T; output side:
    W = basis [rows, rank] @ coeff [rank, cols]."""
    if side == "input":
        rows, rank = coeff.shape
        cols = basis.shape[0]
    else:
        rank, cols = coeff.shape
        rows = basis.shape[0]
    return native().aap_encode(rows, cols, rank, basis_layer, 1 if side == "input" else 2,
                               coeff.astype(np.float16).view(np.uint16).reshape(-1),
                               basis.astype(np.float16).view(np.uint16).reshape(-1))


def encode_hq30(w: np.ndarray, codec: str, group: int, keep: int = 0) -> np.ndarray:
    n = native()
    shape = [int(d) for d in w.shape]
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    if codec == "complete_binary":
        return n.hq30_binary_encode(shape, w, group)
    if codec == "uniform_q4":
        return n.hq30_uq4_encode(shape, w, group)
    if codec == "binary_residual":
        return n.hq30_residual_encode(shape, w, group, keep)
    raise ValueError(codec)


# ---- NumPy restatement (cross-check of the C++ decoders) ----
def unpack_msb_np(stream: np.ndarray, count: int, bits: int) -> np.ndarray:
    bitsarr = np.unpackbits(np.asarray(stream, dtype=np.uint8), bitorder="big")[: count * bits]
    v = bitsarr.reshape(count, bits).astype(np.uint32)
    weights = (1 << np.arange(bits - 1, -1, -1, dtype=np.uint32))
    return (v * weights).sum(1).astype(np.uint32)


def pq_decode_np(codebooks: np.ndarray, indices: np.ndarray) -> np.ndarray:
    s, card, sub = codebooks.shape
    rows, nchunk, _ = indices.shape
    parts = codebooks[np.arange(s)[None, None, :], indices.astype(np.int64)]  # [rows, nchunk, s, sub]
    return parts.reshape(rows, nchunk * s * sub)


def rpq_decode_np(codebooks: np.ndarray, indices: np.ndarray) -> np.ndarray:
    stages, card, d = codebooks.shape
    rows, nchunk, _ = indices.shape
    parts = codebooks[np.arange(stages)[None, None, :], indices.astype(np.int64)]  # [rows, nchunk, stages, d]
    return parts.sum(2).reshape(rows, nchunk * d)


def payload_sections(payload) -> Tuple[dict, Sequence[np.ndarray]]:
    """(header, [codebooks, indices]) of a PQ / residual-PQ payload via the C++ parser."""
    a = _u8(payload)
    k = kind(a)
    if k == "pq":
        return header(a), native().pq_parts(a)
    if k == "residual_pq":
        return header(a), native().rpq_parts(a)
    raise ValueError(f"no codebook sections in a {k} payload")
