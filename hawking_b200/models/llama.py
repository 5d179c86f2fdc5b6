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
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .. import ops
from ..formats.ggml import GgmlType, type_id
from ..formats.gguf import GgufModel
from ..ops import Q8Act, QWeight, cat_rows
from .config import ModelConfig

GEMV_COLS = 8  # rows per GEMV launch (dp4a GEMV batch limit)


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


@dataclass
class LlamaWeights:
    embed: QWeight
    out_norm: torch.Tensor
    lm_head: QWeight
    layers: List[LayerWeights]
    rope_freqs: Optional[torch.Tensor] = None

    @property
    def nbytes(self) -> int:
        n = self.embed.nbytes + self.lm_head.nbytes
        for l in self.layers:
            for w in l.wqkv + [l.wo, l.w_gate, l.w_up, l.w_down]:
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
            lw.w_gate, lw.w_up, lw.w_down = W(cfg.ffn, H), W(cfg.ffn, H), W(H, cfg.ffn)
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
        # Packed host staging: one H2D copy per step.
        self._packed_dev = torch.zeros(5, max_rows, dtype=torch.int32, device=device)
        self._packed_host = torch.zeros(5, max_rows, dtype=torch.int32).pin_memory()
        self.ids, self.positions, self.slots, self.row_seq, self.row_ctx = self._packed_dev.unbind(0)

    def upload(self, ids, positions, slots, row_seq, row_ctx):
        n = len(ids)
        h = self._packed_host
        h[0, :n] = torch.as_tensor(ids, dtype=torch.int32)
        h[1, :n] = torch.as_tensor(positions, dtype=torch.int32)
        h[2, :n] = torch.as_tensor(slots, dtype=torch.int32)
        h[3, :n] = torch.as_tensor(row_seq, dtype=torch.int32)
        h[4, :n] = torch.as_tensor(row_ctx, dtype=torch.int32)
        self._packed_dev.copy_(h, non_blocking=True)
        return n * 5 * 4


class LlamaModel:
    """Runs the forward over static buffers for up to ``max_rows`` rows."""

    def __init__(self, cfg: ModelConfig, weights: LlamaWeights, kv, max_rows: int = 8, device="cuda",
                 max_splits: int = 64):
        self.cfg, self.w, self.kv, self.dev = cfg, weights, kv, torch.device(device)
        self.max_rows = max_rows
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
        self.max_splits = max_splits
        self.part_o = torch.zeros(R * nh * max_splits * hd, device=self.dev)
        self.part_lse = torch.zeros(R * nh * max_splits, device=self.dev)
        self.logits = torch.zeros(R, cfg.vocab, device=self.dev)
        self.next_ids = torch.zeros(R, dtype=torch.int32, device=self.dev)
        self.rope = ops.rope_table(cfg.max_ctx, cfg.rope_dim, cfg.rope_theta, weights.rope_freqs, self.dev)
        self.scale = 1.0 / math.sqrt(hd)
        # sampling inputs (per row)
        self.temperature = torch.zeros(R, device=self.dev)
        self.top_k = torch.zeros(R, dtype=torch.int32, device=self.dev)
        self.top_p = torch.ones(R, device=self.dev)
        self.rep_penalty = torch.ones(R, device=self.dev)
        self.uniforms = torch.zeros(R, device=self.dev)
        self._graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}
        self.launches_per_forward = 0

    def num_splits(self, rows: int) -> int:
        target = 2 * 148
        return max(1, min(self.max_splits, -(-target // (rows * self.cfg.n_kv_heads))))

    # ---- forward ----
    def _gemv_cols(self, fn, rows):
        for c0 in range(0, rows, GEMV_COLS):
            fn(c0, min(rows, c0 + GEMV_COLS))

    def forward(self, rows: int, sample: str = "greedy", advance: bool = False):
        """Forward ``rows`` rows from the static inputs; leaves logits and (greedy) next_ids.
        ``advance`` feeds next_ids back as the next step's inputs on the device (back-to-back
        decode without a host round trip)."""
        cfg, w, kv = self.cfg, self.w, self.kv
        nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        inp = self.inp
        x = self.x[:rows]
        ops.embed(w.embed, inp.ids[:rows], x)
        splits = self.num_splits(rows)
        for l, lw in enumerate(w.layers):
            ops.rmsnorm_q8(x, lw.attn_norm, cfg.eps, self.xa.view(rows))

            def qkv_fn(c0, c1):
                xa = self.xa_view(c0, c1)
                off = 0
                for wt in lw.wqkv:
                    ops.gemv(wt, xa, self.qkv[c0:c1, off:off + wt.N])
                    off += wt.N
            self._gemv_cols(qkv_fn, rows)
            ops.rope_append(self.qkv[:rows], inp.positions[:rows], None, self.rope, cfg.rope_dim,
                            cfg.rope_style, self.q[:rows], kv.k[l], kv.v[l], nh, nkv, hd, kv.block_size,
                            bias=lw.qkv_bias, q_norm=lw.q_norm, k_norm=lw.k_norm, eps=cfg.eps,
                            block_tables=kv.block_tables, row_seq=inp.row_seq[:rows])
            ops.attention_decode(self.q[:rows], kv.k[l], kv.v[l], kv.block_tables, inp.row_seq[:rows],
                                 inp.row_ctx[:rows], self.scale, splits, self.part_o, self.part_lse,
                                 out_q8=self.att.view(rows))
            self._gemv_cols(lambda c0, c1: ops.gemv(lw.wo, self._q8_slice(self.att, c0, c1), x[c0:c1],
                                                    residual=True), rows)
            ops.rmsnorm_q8(x, lw.ffn_norm, cfg.eps, self.xa.view(rows))
            if lw.moe is not None:
                lw.moe.forward(self, rows)
            else:
                self._gemv_cols(lambda c0, c1: ops.gemv_swiglu(lw.w_gate, lw.w_up, self.xa_view(c0, c1),
                                                               self._q8_slice(self.hq, c0, c1)), rows)
                self._gemv_cols(lambda c0, c1: ops.gemv(lw.w_down, self._q8_slice(self.hq, c0, c1, lw.w_down.K),
                                                        x[c0:c1], residual=True), rows)
        ops.rmsnorm_q8(x, w.out_norm, cfg.eps, self.xa.view(rows))
        self._gemv_cols(lambda c0, c1: ops.gemv(w.lm_head, self.xa_view(c0, c1), self.logits[c0:c1]), rows)
        if sample == "greedy":
            ops.argmax(self.logits[:rows], self.next_ids[:rows])
        elif sample == "sample":
            ops.sample(self.logits[:rows], self.temperature[:rows], self.top_k[:rows], self.top_p[:rows],
                       self.rep_penalty[:rows], None, self.uniforms[:rows], self.next_ids[:rows])
        if advance:
            ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)

    def forward_tokens(self, tokens, seq_id: int = -1, start_pos: int = 0) -> torch.Tensor:
        """Teacher-forced forward of ``tokens`` for one sequence (positions start_pos..), returning
        fp32 logits [len(tokens), vocab]. Uses (and extends) the sequence's paged KV."""
        kv = self.kv
        n = len(tokens)
        if not kv.bm.reserve(seq_id, start_pos + n):
            raise RuntimeError("KV pool exhausted")
        kv.sync_tables([seq_id])
        r = kv.row(seq_id)
        out = torch.empty(n, self.cfg.vocab, device=self.dev)
        for c0 in range(0, n, self.max_rows):
            c1 = min(n, c0 + self.max_rows)
            pos = list(range(start_pos + c0, start_pos + c1))
            self.inp.upload(tokens[c0:c1], pos, [0] * (c1 - c0), [r] * (c1 - c0), [p + 1 for p in pos])
            self.forward(c1 - c0, "none")
            out[c0:c1] = self.logits[: c1 - c0]
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
