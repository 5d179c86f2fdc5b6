"""`.gravity` mixed low-bit weights on the device (binary HGRAVB01, uniform HGRAVU01 2/4/8 bits).

A ``MixedWeight`` holds one [N, K] tensor as two planes taken straight from the codec payload: the
LSB-first code stream of every row and the fp16 group scales. ``MixedTable`` packs the device
descriptors of many tensors (e.g. 512 experts x 3 matrices whose codecs differ per tensor) so one
kernel launch can mix codecs. Quantisers here restate the codecs in PyTorch (device side) and are
cross-checked against the C++ payload encoders/decoders.

Parity: crates/hawking-core/src/model/qwen_complete_binary/q80_mixed_decode.rs (binary sign + mean-abs
scale; uniform code = signed + bound, absmax / bound scale; LSB-first packing).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import numpy as np
import torch

from .._ext import kernels

BINARY, UNIFORM, FP8, Q4K, FP4 = 0, 1, 2, 3, 4  # Q4K: a GGUF Q4_K tensor's quant + header planes
# FP4: e2m1 codes two per byte (even column in the low nibble) with a power-of-two (e8m0) scale
# per 32 columns, stored as fp32

# e2m1 magnitudes of codes 0..7 (bit 3 is the sign): exponent 0 is subnormal (m / 2), otherwise
# 2^(e - 1) (1 + m / 2)
E2M1_MAGNITUDES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def e2m1_decode(codes: torch.Tensor) -> torch.Tensor:
    """fp32 values of 4-bit e2m1 codes (any integer tensor of values 0..15)."""
    mag = torch.tensor(E2M1_MAGNITUDES, device=codes.device)[(codes & 7).long()]
    return torch.where((codes & 8) != 0, -mag, mag)


def _pack_lsb(codes: torch.Tensor, bits: int) -> torch.Tensor:
    """[N, K] small unsigned ints -> [N, K * bits / 8] bytes, LSB-first."""
    N, K = codes.shape
    per = 8 // bits
    c = codes.to(torch.int32).reshape(N, K // per, per)
    shifts = torch.arange(per, device=codes.device, dtype=torch.int32) * bits
    return (c << shifts).sum(-1).to(torch.uint8)


def _unpack_lsb(packed: torch.Tensor, bits: int, K: int) -> torch.Tensor:
    N = packed.shape[0]
    per = 8 // bits
    shifts = torch.arange(per, device=packed.device, dtype=torch.int32) * bits
    return ((packed.to(torch.int32).unsqueeze(-1) >> shifts) & ((1 << bits) - 1)).reshape(N, -1)[:, :K]


@dataclass
class MixedWeight:
    kind: int
    bits: int
    group: int
    N: int
    K: int
    codes: torch.Tensor   # uint8 [N, K * bits / 8]
    scales: torch.Tensor  # fp16 [N, K / group]
    zero: int = -1        # uniform code zero point; -1 = 2^(bits-1) - 1 (HGRAVU01), 8 for HQ30UQ4

    @property
    def bound(self) -> int:
        if self.kind != UNIFORM:
            return 0
        return self.zero if self.zero >= 0 else (1 << (self.bits - 1)) - 1

    @property
    def nbytes(self) -> int:
        return self.codes.numel() + self.scales.numel() * self.scales.element_size()

    @property
    def bpw(self) -> float:
        return self.nbytes * 8.0 / (self.N * self.K)

    # ---- construction ----
    @staticmethod
    def quantize(w: torch.Tensor, kind: int, bits: int = 1, group: int = 64) -> "MixedWeight":
        """Encode fp32 [N, K] (any device) with the codec's own rule."""
        N, K = w.shape
        g = w.float().reshape(N, K // group, group)
        if kind == BINARY:
            scale = g.abs().mean(-1)
            codes = (w >= 0).to(torch.uint8)
            bits = 1
        else:
            bound = (1 << (bits - 1)) - 1
            scale = g.abs().amax(-1) / bound
            s16 = scale.to(torch.float16).float()
            inv = torch.where(s16 > 0, 1.0 / s16, torch.zeros_like(s16))
            codes = (torch.round(g * inv.unsqueeze(-1)).clamp(-bound, bound) + bound).reshape(N, K).to(torch.uint8)
        return MixedWeight(kind, bits, group, N, K, _pack_lsb(codes, bits).contiguous(),
                           scale.to(torch.float16).contiguous())

    @staticmethod
    def quantize_fp8(w: torch.Tensor, block: int = 128) -> "MixedWeight":
        """fp8 e4m3 with one fp32 scale per block x block tile (scale = amax / 448), the scale of a
        row's tile stored per row ([N, K / block])."""
        N, K = w.shape
        nbr, nbc = -(-N // block), K // block
        wp = torch.zeros(nbr * block, K, device=w.device)
        wp[:N] = w.float()
        tiles = wp.view(nbr, block, nbc, block)
        sc = tiles.abs().amax(dim=(1, 3)) / 448.0
        sc = torch.where(sc > 0, sc, torch.ones_like(sc))
        q = (tiles / sc[:, None, :, None]).view(nbr * block, K)[:N].to(torch.float8_e4m3fn)
        scales = sc.repeat_interleave(block, 0)[:N].contiguous()
        return MixedWeight(FP8, 8, block, N, K, q.view(torch.uint8).contiguous(), scales)

    @staticmethod
    def quantize_fp4(w: torch.Tensor) -> "MixedWeight":
        """fp4 e2m1 with one power-of-two scale per 32 columns (the MX rule: the scale is
        2^(floor(log2 amax) - 2), 2 being the largest e2m1 exponent, and each element takes the
        nearest e2m1 value of w / scale, saturated at +-6; exactly halfway values take the even
        code)."""
        N, K = w.shape
        if K % 32:
            raise ValueError("fp4: K must be a multiple of 32")
        g = w.float().reshape(N, K // 32, 32)
        amax = g.abs().amax(-1)
        e = torch.where(amax > 0, torch.floor(torch.log2(amax)) - 2, torch.full_like(amax, -127.0)).clamp(-127, 127)
        scale = torch.exp2(e)
        x = (g / scale.unsqueeze(-1)).clamp(-6.0, 6.0)
        grid = torch.tensor(E2M1_MAGNITUDES, device=w.device)
        dist = (x.abs().unsqueeze(-1) - grid).abs()
        # nearest magnitude; ties to the even code (the lower one here: codes 2i are even)
        idx = torch.argmin(dist + 1e-6 * (torch.arange(8, device=w.device) & 1), dim=-1)
        codes = (idx | ((x < 0) & (idx > 0)).long() << 3).to(torch.uint8).reshape(N, K)
        return MixedWeight(FP4, 4, 32, N, K, _pack_lsb(codes, 4).contiguous(), scale.float().contiguous())

    @staticmethod
    def from_e2m1_e8m0(packed: torch.Tensor, e8m0: torch.Tensor, N: int, K: int, device) -> "MixedWeight":
        """The source layout of fp4 weights: packed e2m1 pairs [N, K/2] (column c in byte c / 2, the
        high nibble for odd c) and e8m0 exponents [N, K/32] (scale 2^(e - 127)); the codes are kept
        as they are and the exponents become exact fp32 scales."""
        packed = packed.reshape(N, K // 2).to(torch.uint8)
        e = e8m0.reshape(N, K // 32).to(torch.int32)
        if bool((e == 255).any()):
            raise ValueError("fp4: e8m0 exponent 255 (NaN) in the scales")
        scale = torch.exp2((e - 127).float())
        return MixedWeight(FP4, 4, 32, N, K, packed.to(device).contiguous(), scale.to(device).contiguous())

    @staticmethod
    def random_fp8(N: int, K: int, std: float, gen: torch.Generator, device, block: int = 128,
                   chunk_rows: int = 8192) -> "MixedWeight":
        """Random-init N(0, std) weights in fp8 e4m3 with 128 x 128 block scales, generated in row
        chunks (benchmark weights)."""
        codes = torch.empty(N, K, dtype=torch.uint8, device=device)
        nbc = K // block
        scales = torch.empty(N, nbc, dtype=torch.float32, device=device)
        for r0 in range(0, N, chunk_rows):
            r1 = min(N, r0 + chunk_rows)
            part = MixedWeight.quantize_fp8(torch.randn(r1 - r0, K, generator=gen, device=device) * std, block)
            codes[r0:r1] = part.codes
            scales[r0:r1] = part.scales
        return MixedWeight(FP8, 8, block, N, K, codes, scales)

    @staticmethod
    def random(N: int, K: int, kind: int, bits: int, group: int, std: float, gen: torch.Generator, device) -> "MixedWeight":
        """The codec of N(0, std) weights without materialising them: uniform random codes and
        group scales at the statistics a Gaussian gives (benchmark weights)."""
        bits = 1 if kind == BINARY else bits
        codes = torch.randint(0, 256, (N, K * bits // 8), generator=gen, device=device, dtype=torch.int32).to(torch.uint8)
        if kind == BINARY:
            sc = std * 0.7979  # E|w| of a Gaussian
        else:
            bound = (1 << (bits - 1)) - 1
            sc = std * 2.5 / bound  # ~ absmax of 64 Gaussian draws / bound
            if bits == 2:  # codes 0..2 only
                c = torch.randint(0, 3, (N, K), generator=gen, device=device, dtype=torch.int32)
                codes = _pack_lsb(c, 2)
        scales = torch.full((N, K // group), sc, dtype=torch.float16, device=device)
        return MixedWeight(kind, bits, group, N, K, codes.contiguous(), scales)

    @staticmethod
    def from_payload(payload: np.ndarray, device) -> "MixedWeight":
        """From an HGRAVB01 / HGRAVU01 envelope (bytes as in the artifact)."""
        from ..formats import mixed as mx
        magic, hdr, off, nbody = mx.header(payload)
        rows, cols = int(hdr["shape"][0]), int(hdr["shape"][1])
        gs = int(hdr["group_size"])
        groups = rows * cols // gs
        body = np.asarray(payload[off:off + nbody])
        if magic == b"HGRAVB01":
            kind, bits = BINARY, 1
        elif magic == b"HGRAVU01":
            kind, bits = UNIFORM, int(hdr["bits"])
        else:
            raise ValueError(f"no device layout for {magic!r}")
        scales = torch.from_numpy(body[:groups * 2].copy().view(np.float16).reshape(rows, cols // gs))
        codes = torch.from_numpy(body[groups * 2:].copy().reshape(rows, cols * bits // 8))
        return MixedWeight(kind, bits, gs, rows, cols, codes.to(device).contiguous(), scales.to(device).contiguous())

    @staticmethod
    def from_gguf(raw: torch.Tensor, fmt: int, N: int, K: int, device) -> "MixedWeight":
        """A GGUF tensor's bytes ([N, row_bytes] uint8, any device) as a table weight. Q4_K keeps
        its own planes (kind Q4K), Q8_0 becomes 8-bit codes q + 128 with its fp16 block scales and
        Q4_0 4-bit codes (zero point 8) with its nibbles re-ordered LSB-first: all three are the
        file's values bit for bit. Other formats are decoded and re-encoded as 8-bit codes with
        one fp16 scale per 32 elements (absmax / 127; error at most half a code step)."""
        from ..formats.ggml import GgmlType
        from .qweight import QWeight
        fmt = int(fmt)
        raw = raw.to(device)
        if fmt == GgmlType.Q4_K:
            q = QWeight.from_raw(raw, fmt, N, K)
            return MixedWeight(Q4K, 4, 256, N, K, q.planes[0].contiguous(),
                               q.planes[1].contiguous().view(torch.float16))
        if fmt == GgmlType.Q8_0:
            b = raw.reshape(N, K // 32, 34)
            scales = b[:, :, :2].contiguous().view(torch.float16).reshape(N, K // 32)
            codes = (b[:, :, 2:] ^ 0x80).reshape(N, K)
            return MixedWeight(UNIFORM, 8, 32, N, K, codes.contiguous(), scales.contiguous(), zero=128)
        if fmt == GgmlType.Q4_0:
            b = raw.reshape(N, K // 32, 18)
            scales = b[:, :, :2].contiguous().view(torch.float16).reshape(N, K // 32)
            qs = b[:, :, 2:].to(torch.int32)
            nib = torch.cat([qs & 0xF, qs >> 4], -1).reshape(N, K)  # element i: low nibble i, i + 16: high
            return MixedWeight(UNIFORM, 4, 32, N, K, _pack_lsb(nib, 4).contiguous(), scales.contiguous(), zero=8)
        from ..formats import quant_torch
        w = quant_torch.dequantize(raw, fmt, (N, K)).float()
        return MixedWeight.quantize(w, UNIFORM, bits=8, group=32)

    def dequantize(self) -> torch.Tensor:
        if self.kind == Q4K:
            from ..formats import quant_torch
            from ..formats.ggml import GgmlType
            nb = self.K // 256
            raw = torch.cat([self.scales.view(torch.uint8).reshape(self.N, nb, 16),
                             self.codes.reshape(self.N, nb, 128)], -1).reshape(self.N, nb * 144)
            return quant_torch.dequantize(raw, GgmlType.Q4_K, (self.N, self.K)).float()
        if self.kind == FP8:
            return self.codes.view(torch.float8_e4m3fn).float() * self.scales.repeat_interleave(self.group, 1)
        if self.kind == FP4:
            return e2m1_decode(_unpack_lsb(self.codes, 4, self.K)) * self.scales.repeat_interleave(32, 1)
        c = _unpack_lsb(self.codes, self.bits, self.K).float()
        s = self.scales.float().repeat_interleave(self.group, 1)
        if self.kind == BINARY:
            return torch.where(c > 0, s, -s)
        return (c - self.bound) * s

    def rows(self, start: int, count: int) -> "MixedWeight":
        return MixedWeight(self.kind, self.bits, self.group, count, self.K, self.codes[start:start + count],
                           self.scales[start:start + count], self.zero)

    def cols(self, k0: int, k1: int) -> "MixedWeight":
        """Columns [k0, k1) as a new contiguous tensor (whole scale groups: the row-parallel shard
        of a tensor-parallel projection)."""
        if k0 % self.group or k1 % self.group or k0 % 32 or k1 % 32:
            raise ValueError("column slice must align to the scale groups and 32-element blocks")
        b0, b1 = k0 * self.bits // 8, k1 * self.bits // 8
        s0, s1 = (k0 // 32, k1 // 32) if self.kind == Q4K else (k0 // self.group, k1 // self.group)
        return MixedWeight(self.kind, self.bits, self.group, self.N, k1 - k0, self.codes[:, b0:b1].contiguous(),
                           self.scales[:, s0:s1].contiguous(), self.zero)

    def contiguous(self) -> "MixedWeight":
        return MixedWeight(self.kind, self.bits, self.group, self.N, self.K, self.codes.contiguous(),
                           self.scales.contiguous(), self.zero)

    @staticmethod
    def from_hq30(payload: np.ndarray, device) -> "MixedWeight":
        """A 2-D HQ30G1B1 (binary) or HQ30UQ4 (4-bit, zero point 8) payload whose groups tile the
        rows: the body maps onto the device layout as is (scales [N, K / group], codes LSB-first)."""
        from ..formats import codecs
        payload = np.ascontiguousarray(payload, dtype=np.uint8)
        k = codecs.kind(payload)
        h = codecs.header(payload)
        if k not in ("complete_binary", "uniform_q4") or len(h["shape"]) != 2:
            raise ValueError("from_hq30: a rank-2 HQ30G1B1 or HQ30UQ4 payload")
        rows, cols = h["shape"]
        gs = h["group_size"]
        if cols % gs or gs % 32:
            raise ValueError("from_hq30: groups must tile the rows (cols % group == 0, group % 32 == 0)")
        so, co = h["scale_offset"], h["code_offset"]
        scales = torch.from_numpy(payload[so:co].copy().view(np.float16).reshape(rows, cols // gs))
        if k == "complete_binary":
            codes = torch.from_numpy(payload[co:].copy().reshape(rows, cols // 8))
            return MixedWeight(BINARY, 1, gs, rows, cols, codes.to(device).contiguous(), scales.to(device).contiguous())
        codes = torch.from_numpy(payload[co:].copy().reshape(rows, cols // 2))
        return MixedWeight(UNIFORM, 4, gs, rows, cols, codes.to(device).contiguous(), scales.to(device).contiguous(),
                           zero=8)


class MixedTable:
    """Device descriptor array over a list of MixedWeights (index i = weights[i])."""

    def __init__(self, weights: List[MixedWeight]):
        self.weights = list(weights)
        self.descs = kernels().mixed_descs([w.codes for w in weights], [w.scales for w in weights],
                                           [w.kind for w in weights], [w.bits for w in weights],
                                           [w.group for w in weights], [w.zero for w in weights])

    @property
    def nbytes(self) -> int:
        return sum(w.nbytes for w in self.weights)


def mixed_gemv(table: MixedTable, i: int, x, y: torch.Tensor, residual: bool = False, gate_logit=None,
               argmax_slots=None, argmax_offset: int = 0):
    """y (+)= W_i x; with ``argmax_slots`` (store only) every output also folds into the packed
    greedy keys (index + ``argmax_offset``), as the GGUF GEMV's fused argmax."""
    from . import EPI_RESID, EPI_STORE, PDL, launches
    w = table.weights[i]
    launches.add()
    kernels().mixed_gemv(EPI_RESID if residual else EPI_STORE, table.descs, i, i, w.N, w.K, x.q, x.d, x.s, y, 1.0,
                         None, None, None, PDL, gate_logit, argmax_slots=argmax_slots, argmax_offset=argmax_offset)


def mixed_gemv_push(table: MixedTable, i: int, x, tp, site: int):
    """Row-parallel projection: this rank's partial W_i x goes to every rank's receive region of
    ``site`` (the tensor-parallel all-reduce push; the next RMSNorm sums the ranks)."""
    from . import EPI_PUSH, PDL, launches
    w = table.weights[i]
    launches.add()
    kernels().mixed_gemv(EPI_PUSH, table.descs, i, i, w.N, w.K, x.q, x.d, x.s, None, 1.0, None, None, None, PDL,
                         None, push_table=tp.push_recv[site], push_epoch=tp.epoch)


def mixed_gemv_swiglu(table: MixedTable, i_gate: int, i_up: int, x, out):
    from . import EPI_SWIGLU_Q8, PDL, launches
    w = table.weights[i_gate]
    launches.add()
    kernels().mixed_gemv(EPI_SWIGLU_Q8, table.descs, i_gate, i_up, w.N, w.K, x.q, x.d, x.s, None, 1.0, out.q, out.d,
                         out.s, PDL, None)


@dataclass
class RiceResidualWeight:
    """HGRAVR02 on the device: the binary base (a MixedWeight) plus the outlier residual as CSR
    rows (columns and +-1 signs of each row's outliers, one fp16-derived rms scale)."""
    base: MixedWeight
    row_ptr: torch.Tensor   # int32 [N + 1]
    cols: torch.Tensor      # int32 [nnz]
    signs: torch.Tensor     # int8 [nnz]
    scale: float

    @property
    def N(self) -> int:
        return self.base.N

    @property
    def K(self) -> int:
        return self.base.K

    @property
    def nbytes(self) -> int:
        return self.base.nbytes + self.cols.numel() * 4 + self.signs.numel() + self.row_ptr.numel() * 4

    @staticmethod
    def from_payload(payload: np.ndarray, device) -> "RiceResidualWeight":
        from .._ext import native
        p = native().hgravr02_parts(np.ascontiguousarray(payload, dtype=np.uint8))
        N, K, gs = int(p["rows"]), int(p["cols"]), int(p["group"])
        scales = torch.from_numpy(np.asarray(p["scales"]).copy().view(np.float16).reshape(N, K // gs))
        codes = torch.from_numpy(np.asarray(p["signs"]).copy().reshape(N, K // 8))
        base = MixedWeight(BINARY, 1, gs, N, K, codes.to(device).contiguous(), scales.to(device).contiguous())
        idx = np.asarray(p["indices"]).astype(np.int64)
        rows, cols = idx // K, idx % K
        rs = np.asarray(p["residual_signs"])
        bits = (rs[np.arange(len(idx)) >> 3] >> (np.arange(len(idx)) & 7)) & 1
        order = np.lexsort((cols, rows))  # rows, then columns (the flat indices are already ascending)
        row_ptr = np.zeros(N + 1, dtype=np.int32)
        np.add.at(row_ptr, rows + 1, 1)
        row_ptr = np.cumsum(row_ptr).astype(np.int32)
        t = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a, dtype=dt)).to(device)  # noqa: E731
        return RiceResidualWeight(base, t(row_ptr, np.int32), t(cols[order], np.int32),
                                  t(np.where(bits[order] > 0, 1, -1), np.int8), float(p["residual_scale"]))

    def dequantize(self) -> torch.Tensor:
        w = self.base.dequantize()
        rp = self.row_ptr.cpu().tolist()
        for n in range(self.N):
            for j in range(rp[n], rp[n + 1]):
                w[n, int(self.cols[j])] += self.scale * float(self.signs[j])
        return w


@dataclass
class LowRankWeight:
    """HGRAVS01 on the device: W ~= L @ R with both factors uniform-group MixedWeights; y = L (R x),
    the rank-wide intermediate re-quantised to int8 blocks between the two GEMVs."""
    left: MixedWeight    # [N, rank]
    right: MixedWeight   # [rank, K]

    @property
    def N(self) -> int:
        return self.left.N

    @property
    def K(self) -> int:
        return self.right.K

    @property
    def rank(self) -> int:
        return self.right.N

    @property
    def nbytes(self) -> int:
        return self.left.nbytes + self.right.nbytes

    @staticmethod
    def from_payload(payload: np.ndarray, device) -> "LowRankWeight":
        from .._ext import native
        p = native().hgravs01_parts(np.ascontiguousarray(payload, dtype=np.uint8))

        def factor(f) -> MixedWeight:
            r, c, gs, bits = int(f["rows"]), int(f["cols"]), int(f["group"]), int(f["bits"])
            if c % gs:
                raise ValueError("HGRAVS01 on the device: factor groups must tile the rows")
            sc = torch.from_numpy(np.asarray(f["scales"]).copy().view(np.float16).reshape(r, c // gs))
            codes = torch.from_numpy(np.asarray(f["codes"]).copy().reshape(r, c * bits // 8))
            return MixedWeight(UNIFORM, bits, gs, r, c, codes.to(device).contiguous(), sc.to(device).contiguous())

        return LowRankWeight(factor(p["left"]), factor(p["right"]))

    def dequantize(self) -> torch.Tensor:
        return self.left.dequantize() @ self.right.dequantize()


_SINGLE_TABLES: dict = {}


def _table_of(w: MixedWeight) -> MixedTable:
    t = _SINGLE_TABLES.get(id(w))
    if t is None or t.weights[0] is not w:
        t = _SINGLE_TABLES[id(w)] = MixedTable([w])
    return t


def mixed_linear(w, x, y: torch.Tensor, residual: bool = False):
    """y (+)= W x for one `.gravity` weight of any device codec (binary / uniform: one GEMV;
    HGRAVR02: the base GEMV then the outlier residual; HGRAVS01: R x, re-quantised, then L)."""
    from . import PDL, Q8Act, launches, rmsnorm_q8
    rows = x.q.shape[0]
    if isinstance(w, MixedWeight):
        mixed_gemv(_table_of(w), 0, x, y, residual=residual)
    elif isinstance(w, RiceResidualWeight):
        mixed_gemv(_table_of(w.base), 0, x, y, residual=residual)
        launches.add()
        kernels().sparse_residual(w.row_ptr, w.cols, w.signs, w.scale, w.N, x.q, x.d, w.K, rows, y, PDL)
    elif isinstance(w, LowRankWeight):
        t = torch.zeros(rows, w.rank, device=y.device)
        mixed_gemv(_table_of(w.right), 0, x, t)
        tq = Q8Act(rows, w.rank, y.device)
        rmsnorm_q8(t, None, 0.0, tq, norm=False)
        mixed_gemv(_table_of(w.left), 0, tq, y, residual=residual)
    else:
        raise TypeError(f"mixed_linear: {type(w).__name__}")
