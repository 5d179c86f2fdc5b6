"""Full-precision small-batch GEMV (W4A16) on the tensor cores: Python surface of mma_gemv.cu.

``MgWeight`` is a Q4_K matrix re-laid once into fragment-ordered tiles of 16 rows x 256 columns
(a lossless permutation of the GGUF bytes: the 16-byte super-block headers are copied unchanged and
the quant nibbles are reordered). ``pack(w)`` keeps row order; ``pack(w_gate_up, swiglu=F)``
interleaves the gate and up halves of a fused [gate | up] matrix 8 + 8 rows per tile so the
SwiGLU product can be formed in the GEMV epilogue.

Inputs: ``x_norm`` (fp32 rows + RMSNorm weight, normalised inside the kernel), ``xb`` (bf16 rows)
or ``xfrag`` (a ``FragAct``: bf16 already in the tensor-core fragment order, as written by the
SwiGLU epilogue). Outputs: fp32 rows (store or residual add), SwiGLU h (``FragAct`` and/or bf16
rows), or the tensor-parallel push.

Parity: crates/hawking-core/shaders/quant.metal gemm_q4_k_m_fused* (fp32 activations; the W4A8
variant is off by default in the reference, workspace/docs/reference/env_flags.md:38).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

from .._ext import kernels
from ..formats.ggml import GgmlType
from .qweight import QWeight

MG_X_NORM, MG_X_BF16, MG_X_FRAG = 0, 1, 2
MG_STORE, MG_RESID, MG_SWIGLU, MG_PUSH, MG_ROPE = 0, 1, 2, 3, 4
MG_FORMATS = (GgmlType.Q4_K,)
# Math of the packed tiles: "int" (default) takes each activation as 16-bit fixed point per
# 32-element block (fp32 block scale; two int8 limbs on the u8 x s8 tensor-core MMA; rounding error
# at most 1/64516 of the block's largest magnitude), "bf16" rounds activations to bf16 (bf16 MMA).
MATHS = {"bf16": 0, "int": 1}


@dataclass
class MgWeight:
    tiles: torch.Tensor
    fmt: int
    N: int          # logical output rows (SwiGLU: h rows F)
    K: int
    G: int          # row groups of 16 tile rows
    KT: int         # 256-column tiles per row group
    swiglu: bool = False
    math: str = "int"
    rope: Optional[tuple] = None  # (q+k heads, head_dim, rot_dim, style): rows packed in RoPE-pair order

    @property
    def nbytes(self) -> int:
        return self.tiles.numel()


def supported(w: Optional[QWeight]) -> bool:
    return w is not None and w.fmt in MG_FORMATS and w.K % 256 == 0


def rope_pair_rows(heads: int, hd: int, rot: int, style: int, n_rows: int) -> torch.Tensor:
    """Source row of every packed row when a QKV matrix is packed in RoPE-pair order: within each
    of the first ``heads`` heads (q then k), tile rows r and r + 8 of every 16-row group are the two
    members of a rotation pair (adjacent dims 2i, 2i+1 for style 0; i, i + rot/2 for style 1), dims
    past ``rot`` keep their order; later rows (v) are unchanged. The GEMV epilogues map back."""
    if hd % 16 or rot % 16 or rot > hd:
        raise ValueError("rope_pair_rows: head_dim and rot_dim must be multiples of 16, rot <= head_dim")
    w = torch.arange(hd)
    j, rr = w // 16, w % 16
    r = rr % 8
    rotated = 16 * j < rot
    if style == 0:
        da, db = 16 * j + 2 * r, 16 * j + 2 * r + 1
    else:
        da, db = 8 * j + r, 8 * j + r + rot // 2
    da = torch.where(rotated, da, 16 * j + r)
    db = torch.where(rotated, db, 16 * j + r + 8)
    dim = torch.where(rr < 8, da, db)
    rows = torch.arange(n_rows)
    head = rows // hd
    perm = head * hd + dim[rows % hd]
    return torch.where(head < heads, perm, rows)


def pack(w: QWeight, swiglu: Optional[int] = None, math: str = "int", rope: Optional[tuple] = None) -> MgWeight:
    """Re-lay ``w`` (Q4_K) into fragment-ordered tiles for ``math`` ("int" or "bf16").
    ``swiglu=F``: w is [gate (F rows) | up (F rows)] and tile g holds gate rows 8g..8g+7 followed by
    the matching up rows. ``rope=(q+k heads, hd, rot, style)``: a QKV matrix in RoPE-pair row order
    (``rope_pair_rows``; the store epilogue writes logical rows, the decode-step kernel rotates
    each pair in registers)."""
    if math not in MATHS:
        raise ValueError(f"mg.pack: math must be one of {sorted(MATHS)}")
    if not supported(w):
        raise ValueError(f"mg.pack: format {w.fmt} / K {w.K} not supported by the W4A16 GEMV")
    dev = w.device
    if swiglu:
        F = int(swiglu)
        if w.N != 2 * F:
            raise ValueError("mg.pack: swiglu expects a fused [gate | up] matrix of 2F rows")
        G = (F + 7) // 8
        o = torch.arange(G * 8, dtype=torch.int64).view(G, 8)
        gate = torch.where(o < F, o, torch.full_like(o, -1))
        up = torch.where(o < F, o + F, torch.full_like(o, -1))
        rowmap = torch.cat([gate, up], 1).reshape(-1)
        N = F
    else:
        G = (w.N + 15) // 16
        r = torch.arange(G * 16, dtype=torch.int64)
        src = r
        if rope is not None:
            if w.N % 16:
                raise ValueError("mg.pack: a RoPE-ordered QKV matrix needs a multiple of 16 rows")
            src = rope_pair_rows(*rope, n_rows=G * 16)
        rowmap = torch.where(r < w.N, src, torch.full_like(r, -1))
        N = w.N
    KT = w.K // 256
    tiles = torch.empty(G * KT * kernels().mg_tile_bytes(int(w.fmt)), dtype=torch.uint8, device=dev)
    kernels().mg_pack(int(w.fmt), w.planes, rowmap.to(torch.int32).to(dev), G, KT, tiles, math=MATHS[math])
    return MgWeight(tiles, int(w.fmt), N, w.K, G, KT, bool(swiglu), math, tuple(rope) if rope is not None else None)


def frag_index(K: int, nb: int, cstride: int, device) -> torch.Tensor:
    """Flat bf16 index of x[n][k] in the B-fragment order, for n < nb, k < K (row-major [nb, K])."""
    k = torch.arange(K, device=device)
    ks, kk = k // 16, k % 16
    q, reg, half = (kk % 8) // 2, kk // 8, kk % 2
    u4 = ((ks // 4) * 4 + q) * 2 + (ks % 4) // 2
    u32 = u4 * 4 + (ks % 2) * 2 + reg
    col = torch.arange(nb, device=device)[:, None] * (cstride * 8)
    return (col + (u32 * 2 + half)[None, :]).reshape(-1)


class FragAct:
    """bf16 activations of up to 8 columns in the tensor-core B-fragment order (K % 64 == 0)."""

    def __init__(self, K: int, device, cols: int = 8):
        if K % 64:
            raise ValueError("FragAct: K must be a multiple of 64")
        self.K = K
        self.buf = torch.zeros(cols, K, dtype=torch.bfloat16, device=device)
        self.cstride = K // 8  # uint4s per column (K bf16 = 2K bytes)

    def to_plain(self, nb: int) -> torch.Tensor:
        """[nb, K] bf16 in natural order (test helper)."""
        return self.buf.reshape(-1)[frag_index(self.K, nb, self.cstride, self.buf.device)].view(nb, self.K)


class IntFragAct:
    """Activations of up to 8 columns for the integer math, written by ``quantize``: two int8 limbs
    per element in the tensor-core B-fragment order and per 32-element block (d2, block sum)."""

    def __init__(self, K: int, device, cols: int = 8):
        if K % 256:
            raise ValueError("IntFragAct: K must be a multiple of 256")
        self.K = K
        self.buf = torch.zeros(cols, 2 * K, dtype=torch.uint8, device=device)
        self.cstride = K // 8  # uint4s per column (2K bytes)
        self.info = torch.zeros(cols, K // 32, 2, dtype=torch.float32, device=device)


def quantize(x: torch.Tensor, nb: int, out: IntFragAct, pdl: Optional[bool] = None):
    """bf16 rows [nb, K] -> the two-limb fragment layout of ``out`` (one launch)."""
    from . import PDL, launches
    launches.add()
    kernels().mg_quant(x, nb, out.K, out.buf, out.cstride, out.info, PDL if pdl is None else pdl)


class MgScratch:
    """Per-device partial-sum scratch and row-group counters shared by consecutive GEMV launches
    (each launch writes scratch only after the previous kernel has completed, and leaves every
    counter at zero)."""

    _cache: Dict[int, "MgScratch"] = {}

    def __init__(self, device, max_groups: int = 1 << 16):
        dev = torch.device(device)
        sms = kernels().mg_num_sms(dev.index or 0)
        self.part = torch.zeros(sms * 3 * 8 * 2 * 32 * 4, dtype=torch.float32, device=dev)  # 3 CTAs of 8 warps per SM
        self.counters = torch.zeros(max_groups, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)

    @classmethod
    def get(cls, device) -> "MgScratch":
        dev = torch.device(device)
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        s = cls._cache.get(dev.index)
        if s is None:
            s = cls._cache[dev.index] = MgScratch(dev)
        return s

    def reset(self):
        """Clear counters and status (after a failed step left a row group half counted)."""
        self.counters.zero_()
        self.status.zero_()


def gemv(mw: MgWeight, nb: int, *, x_norm=None, xb: Optional[torch.Tensor] = None,
         xfrag=None, y: Optional[torch.Tensor] = None, residual: bool = False,
         bias=None, hfrag: Optional[FragAct] = None, hb: Optional[torch.Tensor] = None, argmax_slots=None,
         argmax_offset: int = 0, push=None, status: Optional[torch.Tensor] = None, pdl: Optional[bool] = None,
         scratch: Optional[MgScratch] = None, rope_append=None):
    """One W4A16 GEMV launch over ``nb`` batch columns.

    ``x_norm=(x_f32, norm_w, eps)`` (norm_w may be None), ``xb`` or ``xfrag`` (a ``FragAct`` for the
    bf16 math, an ``IntFragAct`` for the integer math) selects the input.
    ``y`` with ``residual`` selects store / add; a SwiGLU-packed weight writes ``hfrag`` / ``hb``;
    ``push=(recv_table, epoch)`` selects the tensor-parallel push. ``rope_append=(rope table,
    positions, row_seq, block_tables, k_cache, v_cache, q_out, nh, nkv, block_size)`` (a QKV matrix
    packed in RoPE-pair order): RoPE and the paged K/V append in the epilogue, q to q_out.
    """
    from . import PDL, launches
    sc = scratch or MgScratch.get(mw.tiles.device)
    if x_norm is not None:
        xin = MG_X_NORM
    elif xb is not None:
        xin = MG_X_BF16
    elif xfrag is not None:
        xin = MG_X_FRAG
    else:
        raise ValueError("mg.gemv: an input is required")
    if mw.swiglu:
        epi = MG_SWIGLU
    elif rope_append is not None:
        if mw.rope is None:
            raise ValueError("mg.gemv: the RoPE epilogue needs a matrix packed in RoPE-pair order")
        epi = MG_ROPE
    elif push is not None:
        epi = MG_PUSH
    else:
        epi = MG_RESID if residual else MG_STORE
    xf, nw, eps = (x_norm if x_norm is not None else (None, None, 1e-5))
    launches.add()
    kernels().mg_gemv(
        mw.fmt, xin, epi, mw.tiles, mw.G, mw.KT, mw.N, mw.K, nb,
        x_f32=xf, norm_w=nw, eps=float(eps), xb=xb,
        xfrag=xfrag.buf if xfrag is not None else None, xfrag_cstride=xfrag.cstride if xfrag is not None else 0,
        y=y, bias=bias, F=mw.N if mw.swiglu else 0,
        hfrag=hfrag.buf if hfrag is not None else None, hfrag_cstride=hfrag.cstride if hfrag is not None else 0,
        hb=hb, argmax_slots=argmax_slots, argmax_offset=argmax_offset,
        push_recv=push[0] if push is not None else None, push_epoch=push[1] if push is not None else None,
        part=sc.part, counters=sc.counters, status=status if status is not None else sc.status,
        pdl=PDL if pdl is None else pdl, math=MATHS[mw.math],
        xinfo=xfrag.info if isinstance(xfrag, IntFragAct) else None,
        rope_order=list(mw.rope) if mw.rope is not None else [],
        rope_epi=list(rope_append[:7]) if rope_append is not None else [],
        rope_dims=list(rope_append[7:]) if rope_append is not None else [])
