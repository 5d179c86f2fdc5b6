"""Device forms of the fixed-header `.gravity` codecs and their GEMVs (``csrc/kernels/codebook.cu``).

``gravity_weight(payload, device)`` maps a payload to a device weight with
``gemv(x: Q8Act, y, accumulate=False)`` (``y[b, :rows] (+)= W x_b`` for the nb <= 8 columns of x):

* GLM52CPK / LLM52RPK -> ``CodebookWeight`` (fp16 codebooks + the MSB-first code stream as stored;
  per-step LUT of codeword . activation-slice products, then LUT gathers per row)
* GLM52AAP -> ``LowRankWeight`` (two thin GEMVs through the rank-r latent)
* HQ30G1B1 / HQ30UQ4 -> ``MixedWeight`` (the binary / 4-bit mixed GEMV, zero point 8 for UQ4)
* HQ30GR2 -> ``ResidualBinaryWeight`` (binary GEMV + sparse fp16 corrections, CSR by row)

Parity: crates/hawking-core/src/artifact_pq.rs:300-420, crates/hawking-core/shaders/gravity_pq.metal,
crates/hawking-core/src/artifact_aap.rs:120-164, qwen_complete_binary/mod.rs:380-430.
"""
from __future__ import annotations

import numpy as np
import torch

from .._ext import kernels
from ..formats import codecs
from .mixed import MixedTable, MixedWeight


def _x_cols(x):
    return x.q, x.d


class CodebookWeight:
    """PQ (sub-spaces tile each chunk) or residual PQ (stages span the chunk)."""

    def __init__(self, payload: np.ndarray, device):
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        self.kind = codecs.kind(payload)
        h = codecs.header(payload)
        self.rows, self.cols, self.nchunk, self.card, self.bits = h["rows"], h["cols"], h["nchunk"], h["card"], h["bits"]
        if self.kind == "pq":
            if h["rotate"]:
                raise ValueError("rotated PQ payloads are not supported")
            self.nsub, self.width, self.d, self.sub_stride = h["s"], h["sub"], h["d"], h["sub"]
        elif self.kind == "residual_pq":
            self.nsub, self.width, self.d, self.sub_stride = h["stages"], h["d"], h["d"], 0
        else:
            raise ValueError(f"not a codebook payload: {self.kind}")
        cb_vals = self.nsub * self.card * self.width
        cb = payload[64:64 + 2 * cb_vals].view(np.float16)
        n_codes = self.rows * self.nchunk * self.nsub
        stream = payload[64 + 2 * cb_vals: 64 + 2 * cb_vals + (n_codes * self.bits + 7) // 8]
        codecs.payload_sections(payload)  # full validation (index range) on the host
        self.codebooks = torch.from_numpy(cb.copy()).to(device)
        self.codes = torch.from_numpy(np.concatenate([stream, np.zeros(4, np.uint8)])).to(device)
        self._lut = None

    @property
    def N(self):
        return self.rows

    @property
    def K(self):
        return self.cols

    def gemv(self, x, y: torch.Tensor, accumulate: bool = False, alpha: float = 1.0):
        from . import PDL, launches
        nb = x.q.shape[0]
        need = nb * self.nchunk * self.nsub * self.card
        if self._lut is None or self._lut.numel() < need:
            self._lut = torch.empty(need, device=self.codebooks.device)
        launches.add(2)
        xq, xd = _x_cols(x)
        kernels().codebook_gemv(self.codebooks, self.codes, self.rows, self.nchunk, self.nsub, self.card, self.width,
                                self.d, self.sub_stride, self.bits, xq, xd, self._lut, y, alpha, accumulate, PDL)


class LowRankWeight:
    """GLM52AAP: W = C . B^T (input side) or B . C (output side), fp16 factors."""

    def __init__(self, payload: np.ndarray, device):
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        h = codecs.header(payload)
        self.rows, self.cols, self.rank = h["rows"], h["cols"], h["rank"]
        self.side = 1 if h["side"] == "input" else 2
        r, c, k = self.rows, self.cols, self.rank
        nc = r * k if self.side == 1 else k * c
        coeff = payload[64:64 + 2 * nc].view(np.float16)
        basis = payload[64 + 2 * nc:].view(np.float16)
        if payload.size != 64 + 2 * (nc + (c * k if self.side == 1 else r * k)):
            raise ValueError("activation-aware payload size does not match its header")
        if self.side == 1:  # latent from the basis [cols, rank], output through the coefficients [rows, rank]
            self.in_proj, self.out_proj = basis.reshape(c, k), coeff.reshape(r, k)
        else:               # latent from the coefficients [rank, cols], output through the basis [rows, rank]
            self.in_proj, self.out_proj = coeff.reshape(k, c), basis.reshape(r, k)
        self.in_proj = torch.from_numpy(self.in_proj.copy()).to(device)
        self.out_proj = torch.from_numpy(self.out_proj.copy()).to(device)
        self._latent = None

    @property
    def N(self):
        return self.rows

    @property
    def K(self):
        return self.cols

    def gemv(self, x, y: torch.Tensor, accumulate: bool = False, alpha: float = 1.0):
        from . import PDL, launches
        nb = x.q.shape[0]
        if self._latent is None or self._latent.numel() < nb * self.rank:
            self._latent = torch.empty(nb * self.rank, device=self.in_proj.device)
        launches.add(2)
        kernels().aap_gemv(self.in_proj, self.out_proj, self.rows, self.cols, self.rank, self.side, x.q, x.d,
                           self._latent, y, alpha, accumulate, PDL)


class TableWeight:
    """One MixedWeight behind its own descriptor table (HQ30G1B1 / HQ30UQ4)."""

    def __init__(self, w: MixedWeight):
        self.w = w
        self.table = MixedTable([w])

    @property
    def N(self):
        return self.w.N

    @property
    def K(self):
        return self.w.K

    def gemv(self, x, y: torch.Tensor, accumulate: bool = False, alpha: float = 1.0):
        from . import EPI_RESID, EPI_STORE, PDL, launches
        launches.add()
        kernels().mixed_gemv(EPI_RESID if accumulate else EPI_STORE, self.table.descs, 0, 0, self.w.N, self.w.K,
                             x.q, x.d, x.s, y, alpha, None, None, None, PDL, None)


class ResidualBinaryWeight(TableWeight):
    """HQ30GR2: the binary base GEMV, then its sparse fp16 corrections (CSR by row)."""

    def __init__(self, payload: np.ndarray, device):
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        h = codecs.header(payload)
        base = payload[h["base_offset"]:h["base_offset"] + h["base_bytes"]]
        super().__init__(MixedWeight.from_hq30(base, device))
        idx = np.asarray(h["indices"], dtype=np.int64)
        vals = np.asarray(h["values"], dtype=np.float32).astype(np.float16)
        rows, cols = h["shape"]
        r, c = idx // cols, idx % cols
        row_ptr = np.zeros(rows + 1, dtype=np.int32)
        np.add.at(row_ptr, r + 1, 1)
        row_ptr = np.cumsum(row_ptr).astype(np.int32)
        self.row_ptr = torch.from_numpy(row_ptr).to(device)
        self.col = torch.from_numpy(c.astype(np.int32)).to(device)
        self.val = torch.from_numpy(vals).to(device)

    def gemv(self, x, y: torch.Tensor, accumulate: bool = False, alpha: float = 1.0):
        from . import PDL, launches
        super().gemv(x, y, accumulate, alpha)
        launches.add()
        kernels().sparse_rows(self.row_ptr, self.col, self.val, x.q, x.d, y, alpha, PDL)


def gravity_weight(payload: np.ndarray, device):
    """Device weight for any fixed-header `.gravity` codec payload."""
    k = codecs.kind(payload)
    if k in ("pq", "residual_pq"):
        return CodebookWeight(payload, device)
    if k == "activation_aware":
        return LowRankWeight(payload, device)
    if k in ("complete_binary", "uniform_q4"):
        return TableWeight(MixedWeight.from_hq30(payload, device))
    if k == "binary_residual":
        return ResidualBinaryWeight(payload, device)
    raise ValueError(k)
