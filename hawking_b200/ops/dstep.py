"""Persistent decode step: Python surface of decode_step.cu.

One launch runs every layer of a dense Llama-family model (Q4_K weights packed for the W4A16
integer-math GEMV, QKV in RoPE-pair order) and the LM head for up to ``MAX_ROWS`` batch rows:
the embedding lookup before it and the greedy argmax / sampler after it stay separate launches.

``DecodeStep.build(model)`` returns None when the model or its shapes are outside what the kernel
covers (MoE, per-head q/k norms, sliding windows, attention sinks, tensor parallelism, a format
other than Q4_K, shapes the kernel does not tile); the model then keeps its per-kernel path.

Parity: the decode step of crates/hawking-core/src/engine.rs (embed -> layers -> norm -> LM head),
whose per-layer kernels are the GEMV / attention kernels the stand-alone ops of this package
cover; the one-launch fusion has no counterpart in the reference.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from .._ext import kernels
from . import launches

MAX_ROWS = 4


class DecodeStep:
    """Pointer table, scratch and launch of the persistent decode-step kernel for one model."""

    def __init__(self, model, table: torch.Tensor):
        cfg, dev = model.cfg, model.dev
        self.model = model
        self.table = table
        nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        self.G = nh // nkv
        self.Ka = nh * hd
        self.F = model.w.layers[0].w_down.K
        self.H = cfg.hidden
        self.grid = kernels().ds_grid(dev.index or 0)
        R = MAX_ROWS
        self.max_splits = 32
        Ka, F = self.Ka, self.F
        self.att_o = torch.zeros(R * nkv * self.max_splits * self.G * hd, device=dev)
        self.att_ml = torch.zeros(R * nkv * self.max_splits * self.G * 2, device=dev)
        self.att_cnt = torch.zeros(R * nkv, dtype=torch.int32, device=dev)
        self.a_limbs = torch.zeros(R, 2 * Ka, dtype=torch.uint8, device=dev)
        self.a_info = torch.zeros(R, Ka // 32, 2, device=dev)
        self.hf = torch.zeros(R, F, device=dev)
        self.h_limbs = torch.zeros(R, 2 * F, dtype=torch.uint8, device=dev)
        self.h_info = torch.zeros(R, F // 32, 2, device=dev)
        self.h_cnt = torch.zeros(F // 32, dtype=torch.int32, device=dev)
        self.part = torch.zeros(self.grid * 16 * 2 * 32 * 4, device=dev)
        gmax = max((model.w.lm_head.N + 15) // 16, (nh + 2 * nkv) * hd // 16, F // 8, self.H // 16)
        self.counters = torch.zeros(gmax, dtype=torch.int32, device=dev)
        self.bar = torch.zeros(2, dtype=torch.int32, device=dev)
        self.wait_ns = int(os.environ.get("HK_DS_WAIT_NS", "0"))
        # per CTA: barriers passed, first failed wait (site, phase, warp); read by ``trace_report``
        self.trace = torch.zeros(self.grid, 4, dtype=torch.int32, device=dev)
        # per-phase device timestamps (set ``timing = True``; read by ``phase_times``)
        self.timing = False
        self.tstamp = torch.zeros(5 * len(model.w.layers) + 2, 4, dtype=torch.int64, device=dev)

    @staticmethod
    def eligible(model) -> bool:
        cfg, w = model.cfg, model.w
        if model.tp is not None or model.small_batch != "w4a16" or model.mg_math != "int":
            return False
        if w.mg_head is None or w.mg_head.math != "int" or w.mg_head.rope is not None:
            return False
        if getattr(cfg, "sliding_window", 0) or getattr(cfg, "attn_sinks", False):
            return False
        for lw in w.layers:
            if lw.moe is not None or lw.q_norm is not None or lw.k_norm is not None:
                return False
            if lw.mg_qkv is None or lw.mg_o is None or lw.mg_gu is None or lw.mg_down is None:
                return False
            if lw.mg_qkv.rope is None or any(m.math != "int" for m in (lw.mg_qkv, lw.mg_o, lw.mg_gu, lw.mg_down)):
                return False
            if getattr(lw, "sinks", None) is not None:
                return False
        F = w.layers[0].w_down.K
        return all(lw.w_down.K == F for lw in w.layers)

    @classmethod
    def build(cls, model) -> Optional["DecodeStep"]:
        if not torch.cuda.is_available() or not cls.eligible(model):
            return None
        w = model.w
        rows = [(lw.mg_qkv.tiles, lw.mg_o.tiles, lw.mg_gu.tiles, lw.mg_down.tiles, lw.attn_norm, lw.ffn_norm,
                 lw.qkv_bias) for lw in w.layers]
        ds = cls(model, kernels().ds_layer_table(rows, model.dev))
        if not kernels().ds_supported(ds.dims(1, 1)):
            return None
        return ds

    def splits(self, rows: int) -> int:
        """KV splits per (row, KV head): items for about a quarter of the SMs (longer splits keep
        each item's K/V ring busy; fewer partials to merge), capped at 32, unless the model forces
        a split count (speculative verify)."""
        m = self.model
        if m.force_splits:
            return min(m.force_splits, self.max_splits)
        s = 1
        while s < self.max_splits and rows * m.cfg.n_kv_heads * s * 4 <= self.grid:
            s *= 2
        return s

    def dims(self, rows: int, splits: int):
        cfg, kv = self.model.cfg, self.model.kv
        return [self.H, self.F, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.rope_dim, cfg.rope_style,
                kv.block_size, kv.block_tables.shape[1], kv.k.shape[1], rows, splits, self.model.w.lm_head.N,
                len(self.model.w.layers)]

    def supports(self, rows: int) -> bool:
        return 1 <= rows <= MAX_ROWS

    def reset(self):
        """Clear the barrier, counters and status after a failed step."""
        for t in (self.att_cnt, self.h_cnt, self.counters, self.bar, self.trace):
            t.zero_()

    def run(self, rows: int, argmax: bool = True):
        """Layers + LM head for ``rows`` rows from model.x (embeddings): logits into model.logits,
        greedy keys into model.argmax_slots when ``argmax``."""
        m = self.model
        cfg, kv, inp = m.cfg, m.kv, m.inp
        launches.add()
        kernels().ds_step(
            self.table, self.dims(rows, self.splits(rows)), float(cfg.eps), float(m.scale),
            inp.positions, inp.row_seq, inp.row_ctx, kv.block_tables, m.rope, m.x, m.q, kv.k, kv.v,
            self.att_o, self.att_ml, self.att_cnt, self.a_limbs, self.a_info, self.hf, self.h_limbs, self.h_info,
            self.h_cnt, self.part, self.counters, m.w.mg_head.tiles, m.w.out_norm, logits=m.logits,
            argmax_slots=m.argmax_slots if argmax else None, bar=self.bar, status=m.status, wait_ns=self.wait_ns,
            trace=self.trace, tstamp=self._arm_tstamp() if self.timing else None)

    def _arm_tstamp(self):
        self.tstamp.zero_()
        self.tstamp[:, 1] = 2 ** 62  # earliest-arrival column starts high
        return self.tstamp

    def phase_times(self) -> dict:
        """Mean microseconds per phase kind over the layers of the last timed step, from CTA 0's
        barrier exits: ``span`` (barrier to barrier), ``first`` / ``last`` (earliest / latest CTA
        arrival at the closing barrier, from the opening one), ``stage`` (CTA 0's activation
        staging, phases that stage)."""
        t = self.tstamp.cpu().double() / 1000.0
        L = len(self.model.w.layers)
        ex = t[:, 0]
        names = ("qkv_rope", "attention", "o_proj", "gate_up", "down")
        out = {}
        for i, n in enumerate(names):
            rows = torch.arange(L) * 5 + i + 1
            prev = ex[rows - 1]
            d = {"span": ex[rows] - prev, "first": t[rows, 1] - prev, "last": t[rows, 2] - prev}
            if i in (0, 3):
                d["stage"] = t[rows, 3] - prev
            out[n] = {k: round(float(v.mean()), 2) for k, v in d.items()}
        out["lm_head"] = round(float(ex[5 * L + 1] - ex[5 * L]), 2)
        out["total"] = round(float(ex[5 * L + 1] - ex[0]), 2)
        return out
