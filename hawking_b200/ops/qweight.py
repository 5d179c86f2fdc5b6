"""Quantised weight matrices on the device.

A ``QWeight`` holds an [N, K] weight in one GGML block format, laid out for the kernels:
K-quant super-blocks whose size is a multiple of 16 bytes (Q4_K) stay as raw GGUF bytes; the
32-element formats and Q6_K are split into planes (quants / high bits / scales), which is a
lossless re-arrangement of the same bytes (``to_raw`` restores the GGUF blocks exactly).
Parity: the reference keeps GGUF bytes zero-copy and re-lays Q4_K into a "Q4K_FAST" sidecar for
its kernels (crates/hawking-core/src/q4k_fast.rs, tools/q4k_fast/src/main.rs:1-6); the planes here
play the same role for the GPU's 16-byte vector loads.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from ..formats.ggml import LAYOUTS, GgmlType, row_bytes

# Byte slices of each block for the plane formats: name -> [(start, end), ...] in plane order.
_PLANES = {
    GgmlType.Q4_K: [(16, 144), (0, 16)],   # quants plane + 16-byte header plane
    GgmlType.Q4_0: [(2, 18), (0, 2)],
    GgmlType.Q8_0: [(2, 34), (0, 2)],
    GgmlType.Q5_0: [(6, 22), (0, 2), (2, 6)],
    GgmlType.Q6_K: [(0, 128), (128, 192), (192, 208), (208, 210)],
}
DENSE = (GgmlType.F32, GgmlType.F16, GgmlType.BF16)
RAW_QUANTIZERS = (GgmlType.Q4_K,)


GEMV_FORMATS = (GgmlType.Q4_K, GgmlType.Q6_K, GgmlType.Q4_0, GgmlType.Q5_0, GgmlType.Q8_0)


@dataclass
class QWeight:
    fmt: int
    N: int
    K: int
    planes: List[torch.Tensor]

    @property
    def device(self):
        return self.planes[0].device

    @property
    def nbytes(self) -> int:
        """Device bytes held (all planes, including derived side planes)."""
        return sum(p.numel() * p.element_size() for p in self.planes)

    @property
    def gguf_nbytes(self) -> int:
        """Bytes of the GGUF payload this weight represents."""
        return self.N * row_bytes(self.fmt, self.K)

    # ---- construction ----
    @staticmethod
    def from_raw(raw: torch.Tensor, fmt: int, N: int, K: int) -> "QWeight":
        """From the GGUF bytes of an [N, K] tensor (uint8, any device)."""
        fmt = int(fmt)
        rb = row_bytes(fmt, K)
        raw = raw.reshape(N, rb)
        if fmt in _PLANES:
            lay = LAYOUTS[fmt]
            blocks = raw.reshape(N, K // lay.block_elems, lay.block_bytes)
            planes = [blocks[:, :, a:b].reshape(N, -1).contiguous() for a, b in _PLANES[fmt]]
        else:
            planes = [raw.contiguous()]
        return QWeight(fmt, N, K, planes)

    def to_raw(self) -> torch.Tensor:
        """GGUF bytes [N, row_bytes] (inverse of from_raw)."""
        if self.fmt not in _PLANES:
            return self.planes[0].reshape(self.N, -1)
        lay = LAYOUTS[self.fmt]
        nb = self.K // lay.block_elems
        out = torch.empty(self.N, nb, lay.block_bytes, dtype=torch.uint8, device=self.device)
        for p, (a, b) in zip(self.planes, _PLANES[self.fmt]):
            out[:, :, a:b] = p.reshape(self.N, nb, b - a)
        return out.reshape(self.N, -1)

    @staticmethod
    def empty(fmt: int, N: int, K: int, device) -> "QWeight":
        fmt = int(fmt)
        lay = LAYOUTS[fmt]
        if fmt in _PLANES:
            nb = K // lay.block_elems
            planes = [torch.empty(N, nb * (b - a), dtype=torch.uint8, device=device) for a, b in _PLANES[fmt]]
        else:
            planes = [torch.empty(N, row_bytes(fmt, K), dtype=torch.uint8, device=device)]
        return QWeight(fmt, N, K, planes)

    @staticmethod
    def quantize(x: torch.Tensor, fmt: int) -> "QWeight":
        """Quantise a CUDA fp32 [N, K] matrix on the device."""
        from .._ext import kernels
        fmt = int(fmt)
        N, K = x.shape
        w = QWeight.empty(fmt, N, K, x.device)
        if fmt in DENSE:
            dt = {GgmlType.F32: torch.float32, GgmlType.F16: torch.float16, GgmlType.BF16: torch.bfloat16}[fmt]
            w.planes[0].view(dt).copy_(x)
            return w
        if fmt in RAW_QUANTIZERS:  # the device quantiser writes whole GGUF blocks
            raw = torch.empty(N, row_bytes(fmt, K), dtype=torch.uint8, device=x.device)
            kernels().quantize(fmt, x.contiguous().float(), [raw])
            return QWeight.from_raw(raw, fmt, N, K)
        kernels().quantize(fmt, x.contiguous().float(), w.planes)
        return w

    @staticmethod
    def random(fmt: int, N: int, K: int, std: float, generator: torch.Generator, device,
               chunk_elems: int = 1 << 26) -> "QWeight":
        """N(0, std) weights quantised on the device, generated in row chunks."""
        w = QWeight.empty(fmt, N, K, device)
        rows = max(1, chunk_elems // K)
        for r0 in range(0, N, rows):
            r1 = min(N, r0 + rows)
            x = torch.randn(r1 - r0, K, generator=generator, device=device) * std
            part = QWeight.quantize(x, fmt)
            for p, q in zip(w.planes, part.planes):
                p[r0:r1].copy_(q)
        return w

    # ---- views ----
    def rows(self, start: int, count: int) -> "QWeight":
        return QWeight(self.fmt, count, self.K, [p[start:start + count] for p in self.planes])

    def dequantize(self) -> torch.Tensor:
        """fp32 [N, K] via the plain-PyTorch restatement of the block formats (test oracle)."""
        from ..formats import quant_torch
        return quant_torch.dequantize(self.to_raw(), self.fmt, (self.N, self.K))


def cat_rows(ws: List[QWeight]) -> QWeight:
    """Stack weights with the same K and format along N (e.g. fused Q|K|V, gate|up)."""
    f, K = ws[0].fmt, ws[0].K
    assert all(w.fmt == f and w.K == K for w in ws)
    planes = [torch.cat([w.planes[i] for w in ws], 0) for i in range(len(ws[0].planes))]
    return QWeight(f, sum(w.N for w in ws), K, planes)
