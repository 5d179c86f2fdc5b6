"""Wide prefill of the mixed-codec MoE layers on the tensor cores (``csrc/kernels/moe_prefill.cu``,
bf16-weight mode of ``csrc/kernels/gemm_tc.cu``).

A forward of T > 8 rows routes T * k pairs. Every expert of the layer is decoded once into a bf16
copy (gate and up rows of expert e at rows [2F e, 2F e + 2F), down rows at [H e, H e + H)), the
pairs are gathered in expert order and two grouped tcgen05 GEMMs run all experts (gate | up with
the SwiGLU epilogue, then down); the combine adds each token's weighted expert outputs to the
residual in pair order (deterministic). A shared expert of the experts' width is one more group
(weight 1, or sigmoid of its gate logit); a wider one runs as a plain GEMM pair over the tokens.

Parity: crates/hawking-core/shaders/moe.metal moe_batched_gemm_*_indexed and
crates/hawking-core/src/model/deepseek_v2.rs:2276 (batched expert prefill).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from .._ext import kernels

BN = 64  # pairs per grouped GEMM tile
GGUF_DEQUANT = (2, 6, 8, 12, 14)  # GGUF formats the block decoder takes: Q4_0, Q5_0, Q8_0, Q4_K, Q6_K


class MoePrefill:
    """Scratch and index lists for one model (the bf16 expert copies are reused layer by layer)."""

    def __init__(self, table, device, E: int, F: int, H: int, max_pairs: int, status: torch.Tensor):
        self.table, self.dev = table, device
        self.E, self.F, self.H = E, F, H
        self.E1 = E + 1  # room for a folded shared expert
        self.w_gu = torch.empty(self.E1 * 2 * F, H, dtype=torch.bfloat16, device=device)
        self.w_dn = torch.empty(self.E1 * H, F, dtype=torch.bfloat16, device=device)
        self.xg = torch.empty(max_pairs, H, dtype=torch.bfloat16, device=device)
        self.h = torch.empty(max_pairs, F, dtype=torch.bfloat16, device=device)
        self.y = torch.empty(max_pairs, H, device=device)
        self.pos = torch.empty(max_pairs, dtype=torch.int32, device=device)
        self.max_tiles = (max_pairs + BN - 1) // BN + self.E1
        self.tiles = torch.zeros(3 * self.max_tiles, dtype=torch.int32, device=device)
        self.n_tiles = torch.zeros(1, dtype=torch.int32, device=device)
        self.status = status
        self._lists: Dict[tuple, tuple] = {}
        self.shared_w: Optional[tuple] = None

    def _lists_for(self, idx: Dict[str, int], fold: bool, e_lo: int, ne: int):
        key = (idx["eg"], idx["eu"], idx["ed"], idx.get("sg", -1), fold, e_lo, ne)
        if key not in self._lists:
            E, F, H = self.E, self.F, self.H
            gi, gr, di, dr = [], [], [], []
            # table entry j of a matrix is expert e_lo + j (this rank's experts); the shared expert
            # goes to slot E
            slots = [(e_lo + j, idx["eg"] + j, idx["eu"] + j, idx["ed"] + j) for j in range(ne)]
            if fold:
                slots.append((E, idx["sg"], idx["su"], idx["sd"]))
            for e, g, u, d in slots:
                gi += [g, u]
                gr += [2 * F * e, 2 * F * e + F]
                di.append(d)
                dr.append(H * e)
            t = lambda v: torch.tensor(v, dtype=torch.int32, device=self.dev)  # noqa: E731
            self._lists[key] = (t(gi), t(gr), t(di), t(dr), E + (1 if fold else 0))
        return self._lists[key]

    def run(self, idx: Dict[str, int], rows: int, k: int, xb: torch.Tensor, x: torch.Tensor, counts, offsets,
            sorted_pairs, route_w, fold: bool, shared_gate: Optional[torch.Tensor] = None, pdl: bool = False,
            e_lo: int = 0, e_count: int = 0, ids: Optional[torch.Tensor] = None):
        """Experts of one layer for ``rows`` tokens. ``xb``: bf16 normed rows [rows, H]; ``x``: the
        fp32 residual rows (updated); counts / offsets / sorted_pairs from the counting sort
        (with the shared expert as expert E when ``fold``); route_w [rows, k]. Under expert
        parallelism (``e_count`` > 0) the table holds experts e_lo .. e_lo + e_count - 1 only:
        just their pairs run, and ``ids`` [rows, k] tells the combine which pairs those are."""
        K = kernels()
        ne = e_count or self.E
        gi, gr, di, dr, n = self._lists_for(idx, fold, e_lo if e_count else 0, ne)
        F, H = self.F, self.H
        K.mixed_dequant_bf16(self.table.descs, gi, gr, F, H, self.w_gu, pdl)
        K.mixed_dequant_bf16(self.table.descs, di, dr, H, F, self.w_dn, pdl)
        self._experts(n, rows, k, xb, x, counts, offsets, sorted_pairs, route_w, fold, shared_gate, pdl,
                      e_lo if e_count else 0, (e_lo + e_count) if e_count else 0, ids)

    def run_gguf(self, w_gate, w_up, w_down, rows: int, k: int, xb: torch.Tensor, x: torch.Tensor, counts,
                 offsets, sorted_pairs, route_w, pdl: bool = False):
        """The same for stacked GGUF expert tensors (QWeight [E F, H] gate / up, [E H, F] down): the
        blocks are decoded into the bf16 copies by the GGUF-format kernel."""
        K = kernels()
        F, H = self.F, self.H
        K.qweight_dequant_bf16(w_gate.fmt, w_gate.planes, H, F, 2 * F, 0, self.w_gu, pdl)
        K.qweight_dequant_bf16(w_up.fmt, w_up.planes, H, F, 2 * F, F, self.w_gu, pdl)
        K.qweight_dequant_bf16(w_down.fmt, w_down.planes, F, H, H, 0, self.w_dn, pdl)
        self._experts(self.E, rows, k, xb, x, counts, offsets, sorted_pairs, route_w, False, None, pdl)

    def _experts(self, n, rows, k, xb, x, counts, offsets, sorted_pairs, route_w, fold, shared_gate, pdl,
                 e_lo: int = 0, e_hi: int = 0, ids: Optional[torch.Tensor] = None):
        K = kernels()
        F, H = self.F, self.H
        P = rows * k
        PS = P + (rows if fold else 0)
        K.moe_tiles(counts, offsets, n, BN, self.tiles, self.n_tiles, pdl, e_lo, e_hi, self.E if fold else -1)
        K.moe_gather_bf16(sorted_pairs, PS, P, k, xb, self.xg, self.pos, pdl)
        mt = (PS + BN - 1) // BN + n
        K.tc_gemm_bf16(self.w_gu, self.xg[:PS], 2 * F, PS, h=self.h, bn=BN, status=self.status, pdl=pdl,
                       tiles=self.tiles, n_tiles=self.n_tiles, max_tiles=mt, group_rows=2 * F)
        K.tc_gemm_bf16(self.w_dn, self.h[:PS], H, PS, y=self.y, bn=BN, status=self.status, pdl=pdl,
                       tiles=self.tiles, n_tiles=self.n_tiles, max_tiles=mt, group_rows=H)
        K.moe_combine(self.y, self.pos, route_w, rows, k, fold, shared_gate, x, pdl, ids if e_hi else None, e_lo,
                      e_hi)
        from . import launches
        launches.add(7)

    def dense_shared(self, idx: Dict[str, int], Fs: int, rows: int, xb: torch.Tensor, x: torch.Tensor,
                     pdl: bool = False):
        """A shared expert wider than the routed ones: plain GEMMs over the tokens (residual add)."""
        K = kernels()
        if self.shared_w is None or self.shared_w[0].shape[0] != 2 * Fs:
            self.shared_w = (torch.empty(2 * Fs, self.H, dtype=torch.bfloat16, device=self.dev),
                             torch.empty(self.H, Fs, dtype=torch.bfloat16, device=self.dev),
                             torch.empty(self.xg.shape[0], Fs, dtype=torch.bfloat16, device=self.dev))
        wgu, wdn, hs = self.shared_w
        t = lambda v: torch.tensor(v, dtype=torch.int32, device=self.dev)  # noqa: E731
        K.mixed_dequant_bf16(self.table.descs, t([idx["sg"], idx["su"]]), t([0, Fs]), Fs, self.H, wgu, pdl)
        K.mixed_dequant_bf16(self.table.descs, t([idx["sd"]]), t([0]), self.H, Fs, wdn, pdl)
        K.tc_gemm_bf16(wgu, xb[:rows], 2 * Fs, rows, h=hs, bn=128 if rows > 64 else 64, status=self.status, pdl=pdl)
        K.tc_gemm_bf16(wdn, hs[:rows], self.H, rows, y=x[:rows], atomic=True, bn=128 if rows > 64 else 64,
                       status=self.status, pdl=pdl)
        from . import launches
        launches.add(4)


class WideLinear:
    """Dense table projections of a wide forward on the tensor cores: the weight is decoded into a
    bf16 copy (reused buffer per shape) and multiplied by the bf16 rows with the bf16-weight
    tcgen05 GEMM; outputs are stored, or added to the fp32 residual."""

    def __init__(self, table, device, status: torch.Tensor):
        self.table, self.dev, self.status = table, device, status
        self._buf: Dict[tuple, torch.Tensor] = {}
        self._idx: Dict[tuple, tuple] = {}

    def _weights(self, ids, rows: int, K: int) -> torch.Tensor:
        n = rows * len(ids)
        buf = self._buf.get((n, K))
        if buf is None:
            buf = self._buf[(n, K)] = torch.empty(n, K, dtype=torch.bfloat16, device=self.dev)
        key = tuple(ids)
        if key not in self._idx:
            t = lambda v: torch.tensor(v, dtype=torch.int32, device=self.dev)  # noqa: E731
            self._idx[key] = (t(list(ids)), t([rows * j for j in range(len(ids))]))
        didx, drow = self._idx[key]
        kernels().mixed_dequant_bf16(self.table.descs, didx, drow, rows, K, buf)
        return buf

    def linear(self, i: int, xb: torch.Tensor, y: torch.Tensor, residual: bool = False):
        """y (+)= W_i xb for the rows of xb (y fp32 [rows, N], any row stride)."""
        w = self.table.weights[i]
        buf = self._weights([i], w.N, w.K)
        rows = xb.shape[0]
        kernels().tc_gemm_bf16(buf, xb, w.N, rows, y=y, atomic=residual, bn=128 if rows > 64 else 64,
                               status=self.status)
        from . import launches
        launches.add(2)

    def swiglu(self, ig: int, iu: int, xb: torch.Tensor, h: torch.Tensor):
        """h = silu(W_g xb) * (W_u xb) as bf16 rows (gate and up decoded into one [2F, K] copy)."""
        w = self.table.weights[ig]
        buf = self._weights([ig, iu], w.N, w.K)
        rows = xb.shape[0]
        kernels().tc_gemm_bf16(buf, xb, 2 * w.N, rows, h=h, bn=128 if rows > 64 else 64, status=self.status)
        from . import launches
        launches.add(2)


def q8_to_bf16(x, out: torch.Tensor):
    """int8 activation blocks (Q8Act view) -> bf16 rows."""
    from . import launches
    launches.add()
    kernels().q8_to_bf16(x.q, x.d, out)


class QWideLinear:
    """GGUF dense projections of a wide forward on the tensor cores: the QWeight is decoded into a
    bf16 copy (one reused buffer per shape) and multiplied with the bf16-weight tcgen05 GEMM."""

    def __init__(self, device, status: torch.Tensor):
        self.dev, self.status = device, status
        self._buf: Dict[tuple, torch.Tensor] = {}

    @staticmethod
    def supports(w, rows_ok: bool = True) -> bool:
        return w.fmt in GGUF_DEQUANT and w.K % 256 == 0

    def linear(self, w, xb: torch.Tensor, y: torch.Tensor, residual: bool = False):
        """y (+)= W xb for the rows of xb (y fp32 [rows, N], any row stride)."""
        buf = self._buf.get((w.N, w.K))
        if buf is None:
            buf = self._buf[(w.N, w.K)] = torch.empty(w.N, w.K, dtype=torch.bfloat16, device=self.dev)
        K = kernels()
        K.qweight_dequant_bf16(w.fmt, w.planes, w.K, w.N, w.N, 0, buf)
        rows = xb.shape[0]
        K.tc_gemm_bf16(buf, xb, w.N, rows, y=y, atomic=residual, bn=128 if rows > 64 else 64, status=self.status)
        from . import launches
        launches.add(2)
