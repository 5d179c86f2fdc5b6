"""Vectorised GGML block dequantisers in plain PyTorch (fp32).

An independent restatement of the block formats, used (a) as the fp32 reference in GPU kernel
numerics tests and (b) to cross-check the C++ oracle (crates/hawking-core/src/quant.rs:34-160
plays the same role in the reference). Works on CPU or CUDA uint8 tensors of raw blocks.
"""
from __future__ import annotations

import torch

from .ggml import GgmlType, LAYOUTS


def _f16(b: torch.Tensor) -> torch.Tensor:
    """Little-endian fp16 from the last dim of a [..., 2] uint8 tensor."""
    return b.contiguous().view(torch.float16).float().squeeze(-1)


def _blocks(raw: torch.Tensor, t: int) -> torch.Tensor:
    lay = LAYOUTS[t]
    return raw.reshape(-1, lay.block_bytes)


def dequant_q4_0(raw):
    b = _blocks(raw, GgmlType.Q4_0)
    d = _f16(b[:, 0:2])[:, None]
    qs = b[:, 2:18].long()
    lo, hi = (qs & 0xF) - 8, (qs >> 4) - 8
    return (torch.cat([lo, hi], 1).float() * d).reshape(-1)


def dequant_q8_0(raw):
    b = _blocks(raw, GgmlType.Q8_0)
    d = _f16(b[:, 0:2])[:, None]
    qs = b[:, 2:34].contiguous().view(torch.int8).float()
    return (qs * d).reshape(-1)


def dequant_q5_0(raw):
    b = _blocks(raw, GgmlType.Q5_0)
    d = _f16(b[:, 0:2])[:, None]
    qh = b[:, 2:6].contiguous().view(torch.int32).long() & 0xFFFFFFFF
    qs = b[:, 6:22].long()
    j = torch.arange(16, device=raw.device)
    h0 = ((qh >> j) & 1) << 4
    h1 = ((qh >> (j + 16)) & 1) << 4
    lo = ((qs & 0xF) | h0) - 16
    hi = ((qs >> 4) | h1) - 16
    return (torch.cat([lo, hi], 1).float() * d).reshape(-1)


def _scale_min_k4(s12: torch.Tensor):
    """Unpack the 12-byte K-quant field into 8 six-bit scales and mins ([nb, 8] each)."""
    s = s12.long()
    sc = torch.empty(s.shape[0], 8, dtype=torch.long, device=s.device)
    mn = torch.empty_like(sc)
    sc[:, 0:4] = s[:, 0:4] & 63
    mn[:, 0:4] = s[:, 4:8] & 63
    sc[:, 4:8] = (s[:, 8:12] & 0xF) | ((s[:, 0:4] >> 6) << 4)
    mn[:, 4:8] = (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)
    return sc, mn


def dequant_q4_k(raw):
    b = _blocks(raw, GgmlType.Q4_K)
    d = _f16(b[:, 0:2])[:, None]
    dmin = _f16(b[:, 2:4])[:, None]
    sc, mn = _scale_min_k4(b[:, 4:16])
    qs = b[:, 16:144].long().reshape(-1, 4, 32)
    q = torch.stack([qs & 0xF, qs >> 4], 2).reshape(-1, 8, 32).float()  # sub-block j = 2*chunk + half
    return (d[:, :, None] * sc[:, :, None] * q - dmin[:, :, None] * mn[:, :, None]).reshape(-1)


def dequant_q5_k(raw):
    b = _blocks(raw, GgmlType.Q5_K)
    d = _f16(b[:, 0:2])[:, None]
    dmin = _f16(b[:, 2:4])[:, None]
    sc, mn = _scale_min_k4(b[:, 4:16])
    qh = b[:, 16:48].long()  # [nb, 32]
    ql = b[:, 48:176].long().reshape(-1, 4, 32)
    j = torch.arange(4, device=raw.device)[None, :, None]
    lo = (ql & 0xF) + (((qh[:, None, :] >> (2 * j)) & 1) << 4)
    hi = (ql >> 4) + (((qh[:, None, :] >> (2 * j + 1)) & 1) << 4)
    q = torch.stack([lo, hi], 2).reshape(-1, 8, 32).float()
    return (d[:, :, None] * sc[:, :, None] * q - dmin[:, :, None] * mn[:, :, None]).reshape(-1)


def dequant_q6_k(raw):
    b = _blocks(raw, GgmlType.Q6_K)
    ql = b[:, 0:128].long().reshape(-1, 2, 64)
    qh = b[:, 128:192].long().reshape(-1, 2, 32)
    sc = b[:, 192:208].contiguous().view(torch.int8).float().reshape(-1, 16)
    d = _f16(b[:, 208:210])[:, None]
    q1 = (ql[:, :, 0:32] & 0xF) | (((qh >> 0) & 3) << 4)
    q2 = (ql[:, :, 32:64] & 0xF) | (((qh >> 2) & 3) << 4)
    q3 = (ql[:, :, 0:32] >> 4) | (((qh >> 4) & 3) << 4)
    q4 = (ql[:, :, 32:64] >> 4) | (((qh >> 6) & 3) << 4)
    q = torch.stack([q1, q2, q3, q4], 2).reshape(-1, 256).float() - 32  # [nb, 2 halves*4*32]
    scales = sc.repeat_interleave(16, dim=1)  # element e of the block uses sc[e // 16]
    return (d * scales * q).reshape(-1)


def dequant_f16(raw):
    return raw.contiguous().view(torch.float16).float().reshape(-1)


def dequant_bf16(raw):
    return raw.contiguous().view(torch.bfloat16).float().reshape(-1)


def dequant_f32(raw):
    return raw.contiguous().view(torch.float32).reshape(-1).clone()


_TABLE = {
    GgmlType.F32: dequant_f32,
    GgmlType.F16: dequant_f16,
    GgmlType.BF16: dequant_bf16,
    GgmlType.Q4_0: dequant_q4_0,
    GgmlType.Q5_0: dequant_q5_0,
    GgmlType.Q8_0: dequant_q8_0,
    GgmlType.Q4_K: dequant_q4_k,
    GgmlType.Q5_K: dequant_q5_k,
    GgmlType.Q6_K: dequant_q6_k,
}


def dequantize(raw: torch.Tensor, t: int, shape=None) -> torch.Tensor:
    """Dequantise raw GGML blocks (uint8) to fp32; optionally reshape (row-major)."""
    fn = _TABLE.get(int(t))
    if fn is None:
        raise NotImplementedError(f"torch dequant for {LAYOUTS[int(t)].name}")
    out = fn(raw.reshape(-1))
    return out.reshape(shape) if shape is not None else out


SUPPORTED = tuple(_TABLE)
