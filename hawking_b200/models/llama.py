"""Llama-family decoder on the sm_100a kernels (llama / mistral / qwen2 / qwen3 dense; the MoE
families plug their FFN into the same layer loop).

A forward pass processes R "rows": each row is one token of some sequence at some position, so
a decode step (one row per sequence), a prefill chunk (consecutive rows of one sequence, causal
through the per-row context length) and a speculative verify step are the same call. All inputs
live in static device buffers so a step can be captured once in a CUDA graph and replayed.

Per layer: RMSNorm->q8, fused QKV GEMV, RoPE + paged-KV append, split-KV attention (output
re-quantised to q8), O GEMV + residual, RMSNorm->q8, gate/up GEMV with SwiGLU (+q8), down GEMV +
residual. Rows beyond 8 run the GEMVs in groups of 8 (the tensor-core GEMM path takes over for
large row counts).

Parity: crates/hawking-core/src/model/llama.rs:1336 (LlamaDense), :2779 (forward_token),
crates/hawking-core/src/model/qwen_dense.rs:4338 (forward_token_greedy_tcb: one command buffer per
token), :9131 (forward_tokens_multiseq_greedy), :9384 (forward_tokens_verify).
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .. import ops
from ..formats.ggml import GgmlType, type_id
from ..formats.gguf import GgufModel
from ..ops import Q8Act, QWeight, cat_rows
from ..ops import mg
from .config import ModelConfig

GEMV_COLS = 8  # rows per GEMV launch (dp4a GEMV batch limit)
# Prefill-sized FFNs: gate/up with the SwiGLU fused in the persistent GEMM's epilogue (1), or the
# plain persistent GEMM plus the vectorised SwiGLU kernel (0, default)
FUSED_SWIGLU_PREFILL = os.environ.get("HK_FUSED_SWIGLU_PREFILL", "0") == "1"
# RoPE + paged K/V append in the W4A16 QKV GEMV epilogue where the weights allow it
ROPE_EPI = os.environ.get("HK_ROPE_EPI", "1") == "1"
# prefill-sized forwards of GGUF formats other than Q4_K run their dense projections as tensor-core
# GEMMs over bf16 copies of the weights (0: the dp4a GEMV)
WIDE_GGUF = os.environ.get("HK_WIDE_GGUF", "1") == "1"


@dataclass
class LayerWeights:
    attn_norm: torch.Tensor
    wqkv: List[QWeight]          # fused [Q|K|V] (one entry) or three separate weights
    wo: QWeight
    ffn_norm: torch.Tensor
    w_gate: Optional[QWeight] = None
    w_up: Optional[QWeight] = None
    w_down: Optional[QWeight] = None
    qkv_bias: Optional[torch.Tensor] = None
    q_norm: Optional[torch.Tensor] = None
    k_norm: Optional[torch.Tensor] = None
    moe: Optional[object] = None  # MoE FFN module (models/moe.py)
    w_gu: Optional[QWeight] = None  # fused [gate | up] rows (w_gate / w_up are views of it)
    # the same matrices re-laid for the W4A16 small-batch GEMV (ops/mg.py), when supported
    mg_qkv: Optional[object] = None
    mg_o: Optional[object] = None
    mg_gu: Optional[object] = None
    mg_down: Optional[object] = None

    def mg_ready(self) -> bool:
        return self.mg_qkv is not None and self.mg_o is not None and (
            self.moe is not None or (self.mg_gu is not None and self.mg_down is not None))

    def fuse_gate_up(self):
        if self.w_gate is not None and self.w_gate.fmt == self.w_up.fmt and self.w_gu is None:
            F = self.w_gate.N
            self.w_gu = cat_rows([self.w_gate, self.w_up])
            self.w_gate, self.w_up = self.w_gu.rows(0, F), self.w_gu.rows(F, F)


@dataclass
class LlamaWeights:
    embed: QWeight
    out_norm: torch.Tensor
    lm_head: QWeight
    layers: List[LayerWeights]
    rope_freqs: Optional[torch.Tensor] = None
    mg_head: Optional[object] = None

    def prepare_mg(self, math: str = "int", rope: Optional[tuple] = None):
        """Re-lay every supported projection for the W4A16 small-batch GEMV (once; the planar
        GGUF copy stays for the tensor-core GEMM of prefill and large batches). ``rope`` =
        (q+k heads, head_dim, rot_dim, style) packs QKV in RoPE-pair order (the decode-step kernel
        rotates in its epilogue; the stand-alone GEMV writes logical rows)."""
        for l in self.layers:
            if l.mg_qkv is None and len(l.wqkv) == 1 and mg.supported(l.wqkv[0]):
                order = rope if rope is not None and l.wqkv[0].N % 16 == 0 else None
                l.mg_qkv = mg.pack(l.wqkv[0], math=math, rope=order)
            if l.mg_o is None and mg.supported(l.wo):
                l.mg_o = mg.pack(l.wo, math=math)
            if l.moe is None and l.mg_gu is None and l.w_gu is not None and mg.supported(l.w_gu) \
                    and l.w_gu.N == 2 * l.w_down.K and l.w_down.K % 256 == 0:
                l.mg_gu = mg.pack(l.w_gu, swiglu=l.w_down.K, math=math)
            if l.moe is None and l.mg_down is None and mg.supported(l.w_down):
                l.mg_down = mg.pack(l.w_down, math=math)
        if self.mg_head is None and mg.supported(self.lm_head):
            self.mg_head = mg.pack(self.lm_head, math=math)

    @property
    def mg_nbytes(self) -> int:
        n = self.mg_head.nbytes if self.mg_head is not None else 0
        for l in self.layers:
            for m in (l.mg_qkv, l.mg_o, l.mg_gu, l.mg_down):
                if m is not None:
                    n += m.nbytes
        return n

    @property
    def nbytes(self) -> int:
        n = self.embed.nbytes + self.lm_head.nbytes
        for l in self.layers:
            ws = l.wqkv + [l.wo, l.w_down] + ([l.w_gu] if l.w_gu is not None else [l.w_gate, l.w_up])
            for w in ws:
                if w is not None:
                    n += w.nbytes
            if l.moe is not None:
                n += l.moe.nbytes
        return n


def _gemv_fmt_ok(fmt: int) -> bool:
    return fmt in ops.qweight.GEMV_FORMATS


def load_llama_weights(m: GgufModel, cfg: ModelConfig, device) -> LlamaWeights:
    """Upload GGUF tensors (one host->device copy each) and re-lay them for the kernels."""
    def raw(name):
        return torch.from_numpy(m.raw(name).copy()).to(device, non_blocking=True)

    def qw(name) -> QWeight:
        t = m.tensors[name]
        N, K = t.shape[0], t.shape[-1]
        if len(t.shape) == 3:
            N = t.shape[0] * t.shape[1]
        w = QWeight.from_raw(raw(name), t.type, N, K)
        if not _gemv_fmt_ok(w.fmt) and name != "token_embd.weight":
            w = QWeight.quantize(torch.from_numpy(m.dequantize(name).reshape(N, K)).to(device), GgmlType.Q8_0)
        return w

    def vec(name):
        return torch.from_numpy(m.dequantize(name).reshape(-1).copy()).float().to(device)

    layers = []
    for l in range(cfg.layers):
        p = f"blk.{l}."
        q, k, v = qw(p + "attn_q.weight"), qw(p + "attn_k.weight"), qw(p + "attn_v.weight")
        wqkv = [cat_rows([q, k, v])] if q.fmt == k.fmt == v.fmt else [q, k, v]
        bias = None
        if m.has(p + "attn_q.bias"):
            bias = torch.cat([vec(p + "attn_q.bias"), vec(p + "attn_k.bias"), vec(p + "attn_v.bias")])
        lw = LayerWeights(
            attn_norm=vec(p + "attn_norm.weight"), wqkv=wqkv, wo=qw(p + "attn_output.weight"),
            ffn_norm=vec(p + "ffn_norm.weight"), qkv_bias=bias,
            q_norm=vec(p + "attn_q_norm.weight") if m.has(p + "attn_q_norm.weight") else None,
            k_norm=vec(p + "attn_k_norm.weight") if m.has(p + "attn_k_norm.weight") else None)
        if cfg.layer_is_moe(l):
            from .moe import MoEFFN
            lw.moe = MoEFFN.from_gguf(m, cfg, l, device, qw, vec)
        else:
            lw.w_gate, lw.w_up, lw.w_down = qw(p + "ffn_gate.weight"), qw(p + "ffn_up.weight"), qw(p + "ffn_down.weight")
            lw.fuse_gate_up()
        layers.append(lw)
    embed = QWeight.from_raw(raw("token_embd.weight"), m.tensors["token_embd.weight"].type, cfg.vocab, cfg.hidden)
    head = qw("output.weight") if m.has("output.weight") else (
        embed if _gemv_fmt_ok(embed.fmt) else QWeight.quantize(
            torch.from_numpy(m.dequantize("token_embd.weight")).to(device), GgmlType.Q8_0))
    rf = vec("rope_freqs.weight") if m.has("rope_freqs.weight") else None
    torch.cuda.synchronize(device)
    return LlamaWeights(embed=embed, out_norm=vec("output_norm.weight"), lm_head=head, layers=layers, rope_freqs=rf)


def random_llama_weights(cfg: ModelConfig, device, seed: int = 0, std: float = 0.02) -> LlamaWeights:
    """Random-init N(0, std) weights quantised on the device (benchmark configs)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    fmt = type_id(cfg.weight_type)
    efmt = type_id(cfg.embed_type or cfg.weight_type)
    H, hd = cfg.hidden, cfg.head_dim

    def W(N, K, f=fmt):
        return QWeight.random(f, N, K, std, g, device)

    layers = []
    for l in range(cfg.layers):
        qkv = W((cfg.n_heads + 2 * cfg.n_kv_heads) * hd, H)
        lw = LayerWeights(attn_norm=torch.ones(H, device=device), wqkv=[qkv], wo=W(H, cfg.n_heads * hd),
                          ffn_norm=torch.ones(H, device=device))
        if cfg.qkv_bias:
            lw.qkv_bias = torch.randn((cfg.n_heads + 2 * cfg.n_kv_heads) * hd, generator=g, device=device) * std
        if cfg.qk_norm:
            lw.q_norm = torch.ones(hd, device=device)
            lw.k_norm = torch.ones(hd, device=device)
        if cfg.layer_is_moe(l):
            from .moe import MoEFFN
            lw.moe = MoEFFN.random(cfg, device, g, std)
        else:
            gu = W(2 * cfg.ffn, H)
            lw.w_gu, lw.w_gate, lw.w_up = gu, gu.rows(0, cfg.ffn), gu.rows(cfg.ffn, cfg.ffn)
            lw.w_down = W(H, cfg.ffn)
        layers.append(lw)
    embed = W(cfg.vocab, H, efmt)
    head = embed if cfg.tie_embeddings else W(cfg.vocab, H)
    torch.cuda.synchronize(device)
    return LlamaWeights(embed=embed, out_norm=torch.ones(H, device=device), lm_head=head, layers=layers)


class StepInputs:
    """Static per-step device inputs (rows)."""

    def __init__(self, max_rows: int, device):
        self.ids = torch.zeros(max_rows, dtype=torch.int32, device=device)
        self.positions = torch.zeros(max_rows, dtype=torch.int32, device=device)
        self.slots = torch.zeros(max_rows, dtype=torch.int32, device=device)
        self.row_seq = torch.zeros(max_rows, dtype=torch.int32, device=device)
        self.row_ctx = torch.ones(max_rows, dtype=torch.int32, device=device)
        # Packed host staging: one H2D copy per step, from a ring of two pinned buffers. A buffer
        # is rewritten only after the copy that last read it has run (its event), so a host that
        # runs ahead of the GPU cannot change the inputs of a step that is still queued.
        self._packed_dev = torch.zeros(5, max_rows, dtype=torch.int32, device=device)
        self._host_ring = [torch.zeros(5, max_rows, dtype=torch.int32).pin_memory() for _ in range(2)]
        self._host_done = [None, None]
        self._turn = 0
        self.ids, self.positions, self.slots, self.row_seq, self.row_ctx = self._packed_dev.unbind(0)

    def upload(self, ids, positions, slots, row_seq, row_ctx):
        n = len(ids)
        i = self._turn
        self._turn ^= 1
        if self._host_done[i] is not None:
            self._host_done[i].synchronize()
        h = self._host_ring[i]
        h[0, :n] = torch.as_tensor(ids, dtype=torch.int32)
        h[1, :n] = torch.as_tensor(positions, dtype=torch.int32)
        h[2, :n] = torch.as_tensor(slots, dtype=torch.int32)
        h[3, :n] = torch.as_tensor(row_seq, dtype=torch.int32)
        h[4, :n] = torch.as_tensor(row_ctx, dtype=torch.int32)
        self._packed_dev[:, :n].copy_(h[:, :n], non_blocking=True)
        ev = self._host_done[i] or torch.cuda.Event()
        ev.record()
        self._host_done[i] = ev
        return n * 5 * 4


class LlamaModel:
    """Runs the forward over static buffers for up to ``max_rows`` rows."""

    def __init__(self, cfg: ModelConfig, weights: LlamaWeights, kv, max_rows: int = 8, device="cuda",
                 max_splits: int = 64, tp=None):
        """``cfg`` describes this rank's shard when ``tp`` (parallel.tp.TPComm) is given: heads and
        FFN width already divided by the tensor-parallel degree."""
        self.cfg, self.w, self.kv, self.dev = cfg, weights, kv, torch.device(device)
        self.tp = tp
        self.max_rows = max_rows
        self.max_splits = max_splits
        self.force_splits = 0
        H, hd, nh, nkv = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
        F = max([cfg.ffn, cfg.expert_ffn, cfg.shared_ffn, 32])
        qkv_n = (nh + 2 * nkv) * hd
        R = max_rows
        self.inp = StepInputs(R, self.dev)
        self.x = torch.zeros(R, H, device=self.dev)
        self.xa = Q8Act(R, H, self.dev)
        self.att = Q8Act(R, nh * hd, self.dev)
        self.hq = Q8Act(R, F, self.dev)
        self.qkv = torch.zeros(R, qkv_n, device=self.dev)
        self.q = torch.zeros(R, nh, hd, device=self.dev)
        cap = max(r * self.num_splits(r) for r in range(1, R + 1))
        self.part_o = torch.zeros(cap * nh * hd, device=self.dev)
        self.part_lse = torch.zeros(cap * nh, device=self.dev)
        self.attn_counters = torch.zeros(R * nkv, dtype=torch.int32, device=self.dev)
        self.max_logit_rows = min(R, 256)  # rows whose logits one forward can return
        # dense Q4_K forwards of at least this many rows run on the W4A16 tensor-core GEMM, smaller
        # ones on the W4A8 dp4a GEMV (the runtime profile "exact" sets 1)
        self.tc_min_rows = GEMV_COLS + 1
        self.logits = torch.zeros(self.max_logit_rows, weights.lm_head.N, device=self.dev)
        # set by the caller when the forward's rows hold long runs of one sequence (prefill chunks):
        # attention then runs on the tensor-core prefill kernel instead of the split-KV decode kernel
        self.long_runs = False
        # SwiGLU in the tensor-core GEMM epilogue (the persistent GEMM overlaps that epilogue with
        # the next tile's main loop; the fp32 gate/up activations never reach global memory)
        self.fuse_swiglu_tc = True
        if tp is not None:
            self.x2 = torch.zeros(R, H, device=self.dev)       # second residual buffer (push all-reduce)
            self.partial = torch.zeros(R, H, device=self.dev)  # prefill partial sums (NCCL all-reduce)
        # tensor-core path buffers (bf16 activations; fp32 outputs kept zeroed between uses)
        self.xb = torch.zeros(R, H, dtype=torch.bfloat16, device=self.dev)
        self.attb = torch.zeros(R, nh * hd, dtype=torch.bfloat16, device=self.dev)
        self.hb = torch.zeros(R, F, dtype=torch.bfloat16, device=self.dev)
        self.gu = torch.zeros(R, 2 * F, device=self.dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        self.logit_rows = torch.zeros(R, dtype=torch.int32, device=self.dev)
        self.next_ids = torch.zeros(R, dtype=torch.int32, device=self.dev)
        # pruned LM head: int32 original token id of every kept head row (None: the full vocabulary)
        self.vocab_map = None
        self.rope = ops.rope_table(cfg.max_ctx, cfg.rope_dim, cfg.rope_theta, weights.rope_freqs, self.dev)
        self.scale = 1.0 / math.sqrt(hd)
        # sampling inputs (per row)
        self.temperature = torch.zeros(R, device=self.dev)
        self.top_k = torch.zeros(R, dtype=torch.int32, device=self.dev)
        self.top_p = torch.ones(R, device=self.dev)
        self.rep_penalty = torch.ones(R, device=self.dev)
        self.uniforms = torch.zeros(R, device=self.dev)
        self.argmax_slots = torch.zeros(R, ops.ARGMAX_SLOTS, dtype=torch.int64, device=self.dev)
        self._graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}
        self.launches_per_forward = 0
        # batches of up to 8 rows: "w4a16" (default; bf16 activations on the tensor-core GEMV,
        # ops/mg.py) or "w4a8" (int8 activation blocks on the dp4a GEMV, opt-in)
        self.small_batch = os.environ.get("HK_SMALL_BATCH", "w4a16")
        if self.small_batch not in ("w4a16", "w4a8"):
            raise ValueError(f"HK_SMALL_BATCH must be w4a16 or w4a8, not {self.small_batch!r}")
        # math of the W4A16 GEMV: "int" (activations as 16-bit fixed point per 32-element block on the
        # integer tensor-core MMA, default) or "bf16" (activations rounded to bf16); ops/mg.py
        self.mg_math = os.environ.get("HK_MG_MATH", "int")
        self.hfrag = None
        if self.small_batch == "w4a16":
            hd_ok = hd % 16 == 0 and cfg.rope_dim % 16 == 0 and cfg.rope_dim <= hd
            weights.prepare_mg(self.mg_math, rope=(nh + nkv, hd, cfg.rope_dim, cfg.rope_style) if hd_ok else None)
            if any(lw.mg_gu is not None for lw in weights.layers):
                Fm = max(lw.w_down.K for lw in weights.layers if lw.mg_gu is not None)
                self.hfrag = mg.FragAct(Fm, self.dev) if self.mg_math == "bf16" else mg.IntFragAct(Fm, self.dev)
        # bs <= 4 decode as one persistent launch: opt-in (HK_DSTEP=1); measured slower than the
        # per-kernel path on B200 so far (per-phase barrier, staging and K/V-ring latencies)
        self.dstep = None
        if os.environ.get("HK_DSTEP", "0") == "1" and self.small_batch == "w4a16":
            from ..ops.dstep import DecodeStep
            self.dstep = DecodeStep.build(self)

    def num_splits(self, rows: int) -> int:
        """KV splits per (row, kv head): the smallest power of two (at most 8, the portable
        thread-block cluster size; 16-CTA clusters measured slower) that puts at least one CTA on
        every SM. ``force_splits``
        overrides it (speculative verify uses the single-row split so its logits are bitwise those
        of plain greedy decode)."""
        if self.force_splits:
            return self.force_splits
        s = 1
        while s < min(8, self.max_splits) and rows * self.cfg.n_kv_heads * s < 148:
            s *= 2
        return s

    # ---- forward ----
    def _gemv_cols(self, fn, rows):
        for c0 in range(0, rows, GEMV_COLS):
            fn(c0, min(rows, c0 + GEMV_COLS))

    @property
    def row_limit(self) -> int:
        """Most rows one forward takes: all of ``max_rows``, except under tensor parallelism
        without the tensor-core path, whose push all-reduce sites hold GEMV_COLS rows."""
        if self.tp is not None and not self.use_tensor_cores(GEMV_COLS + 1):
            return GEMV_COLS
        return self.max_rows

    def use_tensor_cores(self, rows: int) -> bool:
        if rows < self.tc_min_rows:
            return False
        ok = getattr(self, "_tc_layers_ok", None)
        if ok is None:  # every layer dense Q4_K (a quantisation tier map can mix formats across layers)
            ok = self._tc_layers_ok = all(
                all(w.fmt == GgmlType.Q4_K for w in l.wqkv + [l.wo]) and l.moe is None and l.w_gu is not None
                and l.w_gu.fmt == GgmlType.Q4_K and l.w_down.fmt == GgmlType.Q4_K for l in self.w.layers)
        return ok

    def forward(self, rows: int, sample: str = "greedy", advance: bool = False, n_logits: int = 0):
        """Forward ``rows`` rows from the static inputs; leaves logits and (greedy) next_ids.

        ``n_logits`` > 0 computes logits only for the rows listed in ``self.logit_rows[:n_logits]``
        (their logits land in ``self.logits[:n_logits]``). ``advance`` feeds next_ids back as the
        next step's inputs on the device (back-to-back decode without a host round trip)."""
        cfg, w, kv = self.cfg, self.w, self.kv
        nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        inp = self.inp
        x = self.x[:rows]
        tc = self.use_tensor_cores(rows)
        tp = self.tp
        # tensor-core forwards of up to tp.wide_rows rows all-reduce through the P2P-read sites
        wide = tp is not None and tc and 0 < rows <= getattr(tp, "wide_rows", 0)
        if tp is not None and (not tc or wide):
            ops.tp_begin(tp)  # one epoch per forward that uses the push / P2P all-reduce sites
        ops.embed(w.embed, inp.ids[:rows], x)
        if self.dstep is not None and tp is None and not tc and n_logits == 0 and not self.long_runs \
                and self.small_batch == "w4a16" and self.dstep.supports(rows):
            # every layer and the LM head in one persistent launch (ops/dstep.py)
            self.dstep.run(rows, argmax=sample == "greedy")
            if sample == "greedy":
                ops.argmax_finalize(self.argmax_slots, rows, self.next_ids)
            elif sample == "sample":
                ops.sample(self.logits[:rows], self.temperature[:rows], self.top_k[:rows], self.top_p[:rows],
                           self.rep_penalty[:rows], None, self.uniforms[:rows], self.next_ids[:rows])
            if advance:
                ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)
            return
        splits = self.num_splits(rows)
        for l, lw in enumerate(w.layers):
            if tp is not None and not tc:
                self._layer_gemv_tp(l, lw, rows, splits)
                continue
            if tc:
                self._attention_block_tc(l, lw, rows, splits, wide)
                self._ffn_block_tc(lw, rows, l, wide)
            elif self._mg_layer(lw):
                self._layer_mg(l, lw, rows, splits)
            else:
                self._attention_block_gemv(l, lw, rows, splits)
                if lw.moe is not None:
                    ops.rmsnorm_q8(x, lw.ffn_norm, cfg.eps, self.xa.view(rows))
                    lw.moe.forward(self, rows)
                else:
                    nxt = w.layers[l + 1].wqkv if l + 1 < len(w.layers) else None
                    ops.rmsnorm_q8(x, lw.ffn_norm, cfg.eps, self.xa.view(rows))
                    self._gemv_cols(lambda c0, c1: ops.gemv_swiglu(lw.w_gate, lw.w_up, self.xa_view(c0, c1),
                                                                   self._q8_slice(self.hq, c0, c1),
                                                                   prefetch=[lw.w_down] if c0 == 0 else None), rows)
                    self._gemv_cols(lambda c0, c1: ops.gemv(lw.w_down,
                                                            self._q8_slice(self.hq, c0, c1, lw.w_down.K),
                                                            x[c0:c1], residual=True,
                                                            prefetch=nxt if c0 == 0 else None), rows)
        if n_logits < 0:  # no row of this chunk is sampled
            if advance:
                ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)
            return
        nl = n_logits or rows
        if nl > self.max_logit_rows:
            raise ValueError(f"forward: logits for {nl} rows requested, at most {self.max_logit_rows}")
        if tp is not None:
            self._lm_head_tp(rows, nl, n_logits, tc, sample)
            if advance:
                ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)
            return
        # a few sampled rows take the GEMV, unless the tensor-core path was asked for at every size
        if tc and w.lm_head.fmt == GgmlType.Q4_K and w.lm_head.N % 128 == 0 and \
                (nl > GEMV_COLS or self.tc_min_rows <= 1):
            ops.rmsnorm(x, w.out_norm, cfg.eps, yb=self.xb[:rows])
            src = self.xb[:rows]
            if n_logits:
                src = self.xb.index_select(0, self.logit_rows[:nl].long())
            self.logits[:nl].zero_()
            ops.tc_gemm(w.lm_head, src, self.logits[:nl], self.status, y_zeroed=True)
        elif self.small_batch == "w4a16" and w.mg_head is not None:
            src = x
            if n_logits:
                src = self.x.index_select(0, self.logit_rows[:nl].long())
            fuse = sample == "greedy"
            self._gemv_cols(lambda c0, c1: mg.gemv(w.mg_head, c1 - c0, x_norm=(src[c0:c1], w.out_norm, cfg.eps),
                                                   y=self.logits[c0:c1], status=self.status,
                                                   argmax_slots=self.argmax_slots[c0:c1] if fuse else None), nl)
            if fuse:
                ops.argmax_finalize(self.argmax_slots, nl, self.next_ids)
                sample = "done"
        else:
            ops.rmsnorm_q8(x, w.out_norm, cfg.eps, self.xa.view(rows))
            xa = self.xa
            if n_logits:
                idx = self.logit_rows[:nl].long()
                xa = Q8Act.__new__(Q8Act)
                xa.K, xa.q, xa.d, xa.s = self.xa.K, self.xa.q.index_select(0, idx), \
                    self.xa.d.index_select(0, idx), self.xa.s.index_select(0, idx)
            fuse = sample == "greedy"
            self._gemv_cols(lambda c0, c1: ops.gemv(w.lm_head, self._q8_slice(xa, c0, c1, cfg.hidden),
                                                    self.logits[c0:c1],
                                                    argmax_slots=self.argmax_slots[c0:c1] if fuse else None), nl)
            if fuse:
                ops.argmax_finalize(self.argmax_slots, nl, self.next_ids)
                sample = "done"
        if sample == "greedy":
            ops.argmax(self.logits[:nl], self.next_ids[:nl])
        elif sample == "sample":
            ops.sample(self.logits[:nl], self.temperature[:nl], self.top_k[:nl], self.top_p[:nl],
                       self.rep_penalty[:nl], None, self.uniforms[:nl], self.next_ids[:nl])
        if self.vocab_map is not None and sample != "none":
            # pruned head: row index -> original token id, before the id becomes the next input
            torch.index_select(self.vocab_map, 0, self.next_ids[:nl].long(), out=self.next_ids[:nl])
        if advance:
            ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)

    def _rope_attention(self, l, lw, rows, splits, out_q8=None, out_bf16=None, roped: bool = False):
        """RoPE + paged append (unless the QKV GEMV's epilogue did both: ``roped``), then attention."""
        cfg, kv, inp = self.cfg, self.kv, self.inp
        if not roped:
            ops.rope_append(self.qkv[:rows], inp.positions[:rows], None, self.rope, cfg.rope_dim,
                            cfg.rope_style, self.q[:rows], kv.k[l], kv.v[l], cfg.n_heads, cfg.n_kv_heads,
                            cfg.head_dim, kv.block_size, bias=lw.qkv_bias, q_norm=lw.q_norm, k_norm=lw.k_norm,
                            eps=cfg.eps, block_tables=kv.block_tables, row_seq=inp.row_seq[:rows])
        if self.long_runs and rows > GEMV_COLS and cfg.head_dim in (64, 128):
            ops.attention_prefill(self.q[:rows], kv.k[l], kv.v[l], kv.block_tables, inp.row_seq[:rows],
                                  inp.row_ctx[:rows], self.scale, out_q8=out_q8, out_bf16=out_bf16)
            return
        ops.attention_decode(self.q[:rows], kv.k[l], kv.v[l], kv.block_tables, inp.row_seq[:rows],
                             inp.row_ctx[:rows], self.scale, splits, self.part_o, self.part_lse,
                             out_q8=out_q8, out_bf16=out_bf16, counters=self.attn_counters)

    # ---- W4A16 small-batch path (ops/mg.py) ----
    def _rope_in_qkv(self, lw) -> bool:
        """RoPE and the paged append run in the QKV GEMV epilogue (QKV packed in RoPE-pair
        order, no per-head q/k norm, whose reduction spans the head; HK_ROPE_EPI=0 turns it off)."""
        return ROPE_EPI and lw.mg_qkv is not None and lw.mg_qkv.rope is not None and lw.q_norm is None \
            and lw.k_norm is None

    def _rope_args(self, l, c0, c1):
        cfg, kv, inp = self.cfg, self.kv, self.inp
        return (self.rope, inp.positions[c0:c1], inp.row_seq[c0:c1], kv.block_tables, kv.k[l], kv.v[l],
                self.q[c0:c1], cfg.n_heads, cfg.n_kv_heads, kv.block_size)

    def _mg_layer(self, lw) -> bool:
        return self.small_batch == "w4a16" and lw.mg_ready()

    def _layer_mg(self, l, lw, rows, splits):
        """One layer for up to 8 rows per launch: fused RMSNorm -> QKV, RoPE + paged append,
        split-KV attention (bf16 out), O projection + residual, fused RMSNorm -> gate/up + SwiGLU
        (h in fragment order), down projection + residual. Five launches per 8 rows."""
        cfg, x, st = self.cfg, self.x, self.status
        fused = self._rope_in_qkv(lw)
        self._gemv_cols(lambda c0, c1: mg.gemv(lw.mg_qkv, c1 - c0, x_norm=(x[c0:c1], lw.attn_norm, cfg.eps),
                                               y=self.qkv[c0:c1], status=st,
                                               rope_append=self._rope_args(l, c0, c1) if fused else None), rows)
        self._rope_attention(l, lw, rows, splits, out_bf16=self.attb[:rows], roped=fused)
        self._gemv_cols(lambda c0, c1: mg.gemv(lw.mg_o, c1 - c0, xb=self.attb[c0:c1], y=x[c0:c1], residual=True,
                                               status=st), rows)
        if lw.moe is not None:
            ops.rmsnorm_q8(x[:rows], lw.ffn_norm, cfg.eps, self.xa.view(rows))
            lw.moe.forward(self, rows)
            return

        def ffn(c0, c1):
            self._mg_ffn(lw, c1 - c0, dict(x_norm=(x[c0:c1], lw.ffn_norm, cfg.eps)), dict(y=x[c0:c1], residual=True))
        self._gemv_cols(ffn, rows)

    def _mg_ffn(self, lw, nb, gu_in: dict, down_out: dict):
        """gate/up + SwiGLU, then down, on the W4A16 GEMV. The bf16 math hands h over in fragment
        order; the integer math writes h as bf16 rows, which the down GEMV quantises while staging
        them (or, when too wide for shared memory, one quantiser launch writes its input layout)."""
        st = self.status
        F = lw.w_down.K
        if self.mg_math == "bf16":
            mg.gemv(lw.mg_gu, nb, hfrag=self.hfrag, status=st, **gu_in)
            mg.gemv(lw.mg_down, nb, xfrag=self.hfrag, status=st, **down_out)
            return
        hb = self.hb[:nb, :F]
        mg.gemv(lw.mg_gu, nb, hb=hb, status=st, **gu_in)
        if nb * F * 2 <= 32 * 1024:
            mg.gemv(lw.mg_down, nb, xb=hb, status=st, **down_out)
        else:
            mg.quantize(hb, nb, self.hfrag)
            mg.gemv(lw.mg_down, nb, xfrag=self.hfrag, status=st, **down_out)

    def _wide_gguf(self, lw, rows) -> bool:
        """Projections of this prefill-sized forward on the tensor cores over bf16 copies of the GGUF
        weights (dense formats the tensor-core Q4_K GEMM does not take, e.g. Mixtral's Q8_0)."""
        from ..ops.prefill import QWideLinear
        # MoE layers only: their prefill already runs the experts wide; dense GGUF models keep the
        # GEMV, whose rows do not depend on the batch they share (prefix reuse is exact)
        if self.tp is not None or rows <= 32 or not WIDE_GGUF or lw.moe is None:
            return False
        ws = list(lw.wqkv) + [lw.wo]
        if not all(QWideLinear.supports(w) for w in ws) or self.cfg.hidden % 128:
            return False
        if getattr(self, "_qwide", None) is None:
            self._qwide = QWideLinear(self.dev, self.status)
        return True

    def _attention_block_gemv(self, l, lw, rows, splits):
        x = self.x[:rows]
        ops.rmsnorm_q8(x, lw.attn_norm, self.cfg.eps, self.xa.view(rows))
        if self._wide_gguf(lw, rows):
            from ..ops.prefill import q8_to_bf16
            q8_to_bf16(self.xa.view(rows), self.xb[:rows])
            off = 0
            for wt in lw.wqkv:
                self._qwide.linear(wt, self.xb[:rows], self.qkv[:rows, off:off + wt.N])
                off += wt.N
            self._rope_attention(l, lw, rows, splits, out_q8=self.att.view(rows))
            q8_to_bf16(self.att.view(rows), self.attb[:rows])
            self._qwide.linear(lw.wo, self.attb[:rows], x, residual=True)
            return

        def qkv_fn(c0, c1):
            xa = self.xa_view(c0, c1)
            off = 0
            for i, wt in enumerate(lw.wqkv):
                last = i == len(lw.wqkv) - 1 and c0 == 0
                ops.gemv(wt, xa, self.qkv[c0:c1, off:off + wt.N], prefetch=[lw.wo] if last else None)
                off += wt.N
        self._gemv_cols(qkv_fn, rows)
        self._rope_attention(l, lw, rows, splits, out_q8=self.att.view(rows))
        ffn_next = None if lw.moe is not None else ([lw.w_gu] if lw.w_gu is not None else [lw.w_gate, lw.w_up])
        self._gemv_cols(lambda c0, c1: ops.gemv(lw.wo, self._q8_slice(self.att, c0, c1), x[c0:c1],
                                                residual=True, prefetch=ffn_next if c0 == 0 else None), rows)

    # ---- tensor parallel (decode GEMV path: fused push all-reduce; see parallel/tp.py) ----
    def _tp_norm_out(self, l_next: int, rows: int):
        """Output form of an all-reduce site whose normalised rows feed layer ``l_next`` (or the LM
        head when l_next == layers): bf16 rows for the W4A16 GEMV, q8 blocks for the dp4a GEMV."""
        w = self.w
        if l_next < len(w.layers):
            bf16 = self._mg_layer(w.layers[l_next])
        else:
            bf16 = self.small_batch == "w4a16" and w.mg_head is not None
        return (None, self.xb[:rows]) if bf16 else (self.xa.view(rows), None)

    def _layer_mg_tp(self, l, lw, rows, splits):
        """Tensor-parallel layer on the W4A16 GEMV: the row-parallel projections push their
        partials (flagged words over NVLink) and the all-reduce + RMSNorm kernel leaves bf16
        normalised rows for the next column-parallel projection."""
        cfg, w, tp, st = self.cfg, self.w, self.tp, self.status
        xa_res, xb_res = self.x[:rows], self.x2[:rows]
        if l == 0:
            mg.gemv(lw.mg_qkv, rows, x_norm=(xa_res, lw.attn_norm, cfg.eps), y=self.qkv[:rows], status=st)
        else:  # the previous layer's all-reduce left norm(x) (bf16) in self.xb
            mg.gemv(lw.mg_qkv, rows, xb=self.xb[:rows], y=self.qkv[:rows], status=st)
        self._rope_attention(l, lw, rows, splits, out_bf16=self.attb[:rows])
        mg.gemv(lw.mg_o, rows, xb=self.attb[:rows], push=(tp.push_recv[2 * l], tp.epoch), status=st)
        if lw.moe is not None:
            ops.tp_allreduce_rmsnorm_q8(tp, 2 * l, xa_res, xb_res, lw.ffn_norm, cfg.eps, self.xa.view(rows))
            lw.moe.forward_ep(self, rows, 2 * l + 1)
        else:
            ops.tp_allreduce_rmsnorm_q8(tp, 2 * l, xa_res, xb_res, lw.ffn_norm, cfg.eps, out_bf16=self.xb[:rows])
            self._mg_ffn(lw, rows, dict(xb=self.xb[:rows]), dict(push=(tp.push_recv[2 * l + 1], tp.epoch)))
        nxt = w.layers[l + 1].attn_norm if l + 1 < len(w.layers) else w.out_norm
        q8, bf = self._tp_norm_out(l + 1, rows)
        ops.tp_allreduce_rmsnorm_q8(tp, 2 * l + 1, xb_res, xa_res, nxt, cfg.eps, q8, bf)

    def _layer_gemv_tp(self, l, lw, rows, splits):
        cfg, w, tp = self.cfg, self.w, self.tp
        if rows > GEMV_COLS:
            raise RuntimeError("tensor-parallel GEMV path takes at most 8 rows")
        if self._mg_layer(lw):
            self._layer_mg_tp(l, lw, rows, splits)
            return
        xa_res, xb_res = self.x[:rows], self.x2[:rows]
        if l == 0:
            ops.rmsnorm_q8(xa_res, lw.attn_norm, cfg.eps, self.xa.view(rows))
        # (for l > 0 the previous layer's FFN all-reduce already left norm(x) in self.xa)
        xa = self.xa_view(0, rows)
        off = 0
        for i, wt in enumerate(lw.wqkv):
            ops.gemv(wt, xa, self.qkv[:rows, off:off + wt.N], prefetch=[lw.wo] if i == len(lw.wqkv) - 1 else None)
            off += wt.N
        self._rope_attention(l, lw, rows, splits, out_q8=self.att.view(rows))
        ffn_next = None if lw.moe is not None else ([lw.w_gu] if lw.w_gu is not None else [lw.w_gate, lw.w_up])
        ops.gemv_push(lw.wo, self._q8_slice(self.att, 0, rows), tp, 2 * l, prefetch=ffn_next)
        ops.tp_allreduce_rmsnorm_q8(tp, 2 * l, xa_res, xb_res, lw.ffn_norm, cfg.eps, self.xa.view(rows))
        if lw.moe is not None:  # expert parallel; the experts' combine is this site's push
            lw.moe.forward_ep(self, rows, 2 * l + 1)
        else:
            nxt = w.layers[l + 1].wqkv if l + 1 < len(w.layers) else None
            ops.gemv_swiglu(lw.w_gate, lw.w_up, self.xa_view(0, rows), self._q8_slice(self.hq, 0, rows),
                            prefetch=[lw.w_down])
            ops.gemv_push(lw.w_down, self._q8_slice(self.hq, 0, rows, lw.w_down.K), tp, 2 * l + 1, prefetch=nxt)
        nxt = w.layers[l + 1].attn_norm if l + 1 < len(w.layers) else w.out_norm
        q8, bf = self._tp_norm_out(l + 1, rows)
        ops.tp_allreduce_rmsnorm_q8(tp, 2 * l + 1, xb_res, xa_res, nxt, cfg.eps, q8, bf)

    def _allreduce_partial_tc(self, rows):
        """Prefill (tensor-core path): NCCL all-reduce of this rank's partial, added to x."""
        import torch.distributed as dist
        p = self.partial[:rows]
        if self.tp.world > 1:
            dist.all_reduce(p, group=self.tp.group)
        self.x[:rows].add_(p)

    def _lm_head_tp(self, rows, nl, n_logits, tc, sample):
        w, cfg, tp = self.w, self.cfg, self.tp
        if n_logits < 0:
            return
        if sample == "sample":  # vocabulary-parallel logits, gathered; every rank draws the same token
            self._lm_head_tp(rows, nl, n_logits, tc, "none")
            full = self.gathered_logits(nl)
            ops.sample(full, self.temperature[:nl], self.top_k[:nl], self.top_p[:nl], self.rep_penalty[:nl], None,
                       self.uniforms[:nl], self.next_ids[:nl])
            return
        if self.small_batch == "w4a16" and w.mg_head is not None:
            off = tp.rank * w.lm_head.N
            if tc or n_logits:
                src = self.x[:rows]
                if n_logits:
                    src = self.x.index_select(0, self.logit_rows[:nl].long())
                kw = lambda c0, c1: dict(x_norm=(src[c0:c1], w.out_norm, cfg.eps))  # noqa: E731
            else:  # the last layer's all-reduce left norm(x) (bf16) in self.xb
                kw = lambda c0, c1: dict(xb=self.xb[c0:c1])  # noqa: E731
            greedy = sample != "none"
            self._gemv_cols(lambda c0, c1: mg.gemv(w.mg_head, c1 - c0, y=self.logits[c0:c1], status=self.status,
                                                   argmax_slots=self.argmax_slots[c0:c1] if greedy else None,
                                                   argmax_offset=off, **kw(c0, c1)), nl)
            if greedy:
                ops.tp_argmax(tp, self.argmax_slots, nl, self.next_ids)
            return
        if tc or n_logits:
            # the residual is in self.x; normalise the sampled rows here
            src = self.x[:rows]
            if n_logits:
                src = self.x.index_select(0, self.logit_rows[:nl].long())
            ops.rmsnorm_q8(src, w.out_norm, cfg.eps, self.xa.view(nl))
        # else: the last layer's all-reduce left norm(x) in self.xa
        if sample == "none":  # this rank's vocabulary slice of the logits only
            self._gemv_cols(lambda c0, c1: ops.gemv(w.lm_head, self.xa_view(c0, c1), self.logits[c0:c1]), nl)
            return
        self._gemv_cols(lambda c0, c1: ops.gemv(w.lm_head, self.xa_view(c0, c1), self.logits[c0:c1],
                                                argmax_slots=self.argmax_slots[c0:c1],
                                                argmax_offset=tp.rank * w.lm_head.N), nl)
        ops.tp_argmax(tp, self.argmax_slots, nl, self.next_ids)

    def gathered_logits(self, nl: int) -> torch.Tensor:
        """Logits of the first ``nl`` logit rows over the whole vocabulary: ``self.logits`` on one
        GPU; under tensor parallelism the ranks' vocabulary slices gathered (a collective: every
        rank calls it for the same rows)."""
        if self.tp is None:
            return self.logits[:nl]
        from ..parallel.tp import gather_vocab_logits
        return gather_vocab_logits(self.tp, self.logits[:nl], self._full_logits(nl))

    def _full_logits(self, nl: int) -> torch.Tensor:
        """[nl, vocab] buffer for the gathered tensor-parallel logits (allocated on first use)."""
        V = self.w.lm_head.N * self.tp.world
        if getattr(self, "_tp_full", None) is None or self._tp_full.shape[0] < nl:
            self._tp_full = torch.zeros(self.max_logit_rows, V, device=self.dev)
        return self._tp_full[:nl]

    def _attention_block_tc(self, l, lw, rows, splits, wide: bool = False):
        """``wide``: tensor parallel over the P2P-read sites; the previous layer's site already
        left norm(x) in self.xb, and this layer's O site writes the residual into self.x2."""
        x = self.x[:rows]
        if not (wide and l > 0):
            ops.rmsnorm(x, lw.attn_norm, self.cfg.eps, yb=self.xb[:rows])
        qkv = self.qkv[:rows]
        once = ops.tc_gemm_overwrites(rows)  # persistent GEMM: plain stores, nothing to zero
        if not once:
            qkv.zero_()
        off = 0
        for wt in lw.wqkv:
            ops.tc_gemm(wt, self.xb[:rows], qkv[:, off:off + wt.N], self.status, y_zeroed=not once)
            off += wt.N
        self._rope_attention(l, lw, rows, splits, out_bf16=self.attb[:rows])
        if wide:
            part = self.tp.wide_part(2 * l)[:rows]
            self._tc_partial(lw.wo, self.attb[:rows], part, once)
            ops.tp_p2p_allreduce_rmsnorm(self.tp, 2 * l, x, self.x2[:rows], lw.ffn_norm, self.cfg.eps,
                                         out_bf16=self.xb[:rows])
        elif self.tp is not None:
            if once:
                ops.tc_gemm(lw.wo, self.attb[:rows], self.partial[:rows], self.status)
            else:
                self.partial[:rows].zero_()
                ops.tc_gemm(lw.wo, self.attb[:rows], self.partial[:rows], self.status, atomic=True, y_zeroed=True)
            self._allreduce_partial_tc(rows)
        else:
            ops.tc_gemm(lw.wo, self.attb[:rows], x, self.status, atomic=True)

    def _tc_partial(self, wt, src, out, once: bool):
        """This rank's partial of a row-parallel projection into ``out`` (plain stores from the
        persistent GEMM, else split-K accumulation into a zeroed buffer)."""
        if once:
            ops.tc_gemm(wt, src, out, self.status)
        else:
            out.zero_()
            ops.tc_gemm(wt, src, out, self.status, atomic=True, y_zeroed=True)

    def _ffn_block_tc(self, lw, rows, l: int = 0, wide: bool = False):
        x = self.x2[:rows] if wide else self.x[:rows]
        F = lw.w_down.K
        if not wide:  # wide: the O site left norm(x2) in self.xb
            ops.rmsnorm(x, lw.ffn_norm, self.cfg.eps, yb=self.xb[:rows])
        bn = max(64, ops.tc_gemm_bn(rows))
        once = ops.tc_gemm_overwrites(rows)
        if self.fuse_swiglu_tc and F % 64 == 0 and lw.w_gu.N == 2 * F and (F // 64) * -(-rows // bn) >= 148 \
                and not ops.tc_gemm_stream_k(rows, lw.w_gu.N) and not (once and not FUSED_SWIGLU_PREFILL):
            # SwiGLU in the GEMM epilogue (enough tiles to fill the GPU without split-K); decode
            # batches instead run gate/up stream-K and the SwiGLU kernel (no partial last wave)
            ops.tc_gemm_swiglu(lw.w_gu, self.xb[:rows], self.hb[:rows, :F], self.status, bn=bn)
        elif once:
            # prefill-sized: the persistent GEMM stores gate/up (no zeroing) and the SwiGLU kernel
            # streams them once; it re-zeroes only the rows the split-K paths (< 192 rows) reuse
            gu = self.gu[:rows, : 2 * F]
            ops.tc_gemm(lw.w_gu, self.xb[:rows], gu, self.status)
            keep = min(rows, ops.SPLIT_K_MAX_ROWS)
            ops.swiglu_bf16(gu[:keep], F, self.hb[:keep, :F], clear=True)
            ops.swiglu_bf16(gu[keep:], F, self.hb[keep:rows, :F], clear=False)
        else:
            gu = self.gu[:rows, : 2 * F]
            ops.tc_gemm(lw.w_gu, self.xb[:rows], gu, self.status, y_zeroed=True)
            ops.swiglu_bf16(gu, F, self.hb[:rows, :F], clear=True)
        if wide:
            part = self.tp.wide_part(2 * l + 1)[:rows]
            self._tc_partial(lw.w_down, self.hb[:rows, :F], part, ops.tc_gemm_overwrites(rows))
            layers = self.w.layers
            nxt = layers[l + 1].attn_norm if l + 1 < len(layers) else self.w.out_norm
            ops.tp_p2p_allreduce_rmsnorm(self.tp, 2 * l + 1, x, self.x[:rows], nxt, self.cfg.eps,
                                         out_bf16=self.xb[:rows])
        elif self.tp is not None:
            if ops.tc_gemm_overwrites(rows):
                ops.tc_gemm(lw.w_down, self.hb[:rows, :F], self.partial[:rows], self.status)
            else:
                self.partial[:rows].zero_()
                ops.tc_gemm(lw.w_down, self.hb[:rows, :F], self.partial[:rows], self.status, atomic=True,
                            y_zeroed=True)
            self._allreduce_partial_tc(rows)
        else:
            ops.tc_gemm(lw.w_down, self.hb[:rows, :F], x, self.status, atomic=True)

    def forward_tokens(self, tokens, seq_id: int = -1, start_pos: int = 0) -> torch.Tensor:
        """Teacher-forced forward of ``tokens`` for one sequence (positions start_pos..), returning
        fp32 logits [len(tokens), vocab]. Uses (and extends) the sequence's paged KV."""
        kv = self.kv
        n = len(tokens)
        if not kv.bm.reserve(seq_id, start_pos + n):
            raise RuntimeError("KV pool exhausted")
        kv.sync_tables([seq_id])
        r = kv.row(seq_id)
        out = torch.empty(n, self.logits.shape[1], device=self.dev)  # this rank's vocabulary slice under TP
        step = min(self.max_logit_rows, self.row_limit)
        self.long_runs = True
        try:
            for c0 in range(0, n, step):
                c1 = min(n, c0 + step)
                pos = list(range(start_pos + c0, start_pos + c1))
                self.inp.upload(tokens[c0:c1], pos, [0] * (c1 - c0), [r] * (c1 - c0), [p + 1 for p in pos])
                self.forward(c1 - c0, "none", n_logits=0)
                out[c0:c1] = self.logits[: c1 - c0]
        finally:
            self.long_runs = False
        return out

    def xa_view(self, c0, c1, K=None):
        return self._q8_slice(self.xa, c0, c1, K or self.cfg.hidden)

    @staticmethod
    def _q8_slice(a: Q8Act, c0, c1, K=None):
        v = Q8Act.__new__(Q8Act)
        K = K or a.K
        v.K = K
        v.q, v.d, v.s = a.q[c0:c1, :K], a.d[c0:c1, : K // 32], a.s[c0:c1, : K // 32]
        return v

    # ---- CUDA graphs ----
    def graph_forward(self, rows: int, sample: str = "greedy", advance: bool = False):
        if self.tp is not None and self.use_tensor_cores(rows):
            # the tensor-core path all-reduces with NCCL: run it eagerly rather than capture NCCL
            n0 = ops.launches.n
            self.forward(rows, sample, advance)
            self.launches_per_graph = ops.launches.n - n0
            return
        key = (rows, sample, advance)
        g = self._graphs.get(key)
        if g is None:
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(s):
                self.forward(rows, sample)  # warm-up (lazy module init, allocator)
            torch.cuda.current_stream(self.dev).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            n0 = ops.launches.n
            with torch.cuda.graph(g):
                self.forward(rows, sample, advance)
            self.launches_per_graph = ops.launches.n - n0
            self._graphs[key] = g
        g.replay()

    def release_graphs(self):
        self._graphs.clear()
