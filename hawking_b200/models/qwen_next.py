"""Qwen3-Next-style hybrid MoE decoder on `.gravity` mixed low-bit weights.

Layers: gated DeltaNet linear attention on most layers, gated full attention (q/k RMSNorm, partial
RoPE, sigmoid output gate) on every ``full_attn_interval``-th layer, and after every mixer a
routed MoE (softmax top-k with renormalisation over many small experts) plus one shared expert
scaled by sigmoid(shared-gate logit). RMSNorm weights are zero-centred (the stored w acts as
1 + w); they are folded to 1 + w at load. Every projection is a `.gravity` mixed tensor (binary /
ternary experts, Q4 attention, shared expert and head) run by the K8 kernels; DeltaNet runs the K7
kernels; full attention uses the paged split-KV kernel (head_dim 256).

Decode is one token per row; rows of different sequences batch together. The recurrence makes a
prompt a sequence of single-token steps (the chunked WY-form prefill is not built).

Parity: crates/hawking-core/src/model/qwen80_hybrid_token_graph.rs:22-168 (operator groups),
crates/hawking-core/src/model/qwen80_mixed_hybrid_decode.rs (deltanet_mixer :3361, gqa_mixer :3521,
moe_suffix :3636, terminal_greedy :3754), crates/hawking-core/shaders/qwen80_device_activations.metal
(math of every elementwise step), docs/QWEN80_MIXED_1P5_PACKED_FORMAT.md:79 (layer % 4 == 3 is
full attention).
"""
from __future__ import annotations

import math
import random
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .. import ops
from .._ext import kernels
from ..ops import Q8Act, QWeight
from ..ops.mixed import (BINARY, UNIFORM, MixedTable, MixedWeight, mixed_gemv, mixed_gemv_push,
                         mixed_gemv_swiglu)
from .config import ModelConfig

# prefill forwards (> 8 rows) run the experts as grouped tensor-core GEMMs (0: the GEMV kernels)
MOE_PREFILL = __import__("os").environ.get("HK_MOE_PREFILL", "1") == "1"


@dataclass
class QNLayer:
    full: bool
    attn_norm: torch.Tensor
    post_norm: torch.Tensor
    idx: Dict[str, int] = field(default_factory=dict)   # table indices of the projections
    q_norm: Optional[torch.Tensor] = None
    k_norm: Optional[torch.Tensor] = None
    conv_w: Optional[torch.Tensor] = None
    a_log: Optional[torch.Tensor] = None
    dt_bias: Optional[torch.Tensor] = None
    ssm_norm: Optional[torch.Tensor] = None
    router: Optional[torch.Tensor] = None               # fp32 [E, H]
    shared_gate: Optional[torch.Tensor] = None          # fp32 [1, H]
    shared_here: bool = True                            # expert parallel: this rank runs the shared expert


@dataclass
class QNWeights:
    table: MixedTable
    embed: QWeight
    out_norm: torch.Tensor
    layers: List[QNLayer]
    lm_head: int
    e_lo: int = 0                       # expert parallel: this rank's routed experts are
    e_count: int = 0                    # e_lo .. e_lo + e_count - 1 (0: all of them)

    @property
    def nbytes(self) -> int:
        n = self.table.nbytes + self.embed.nbytes
        for l in self.layers:
            n += l.router.numel() * 4
        return n


def dims(cfg: ModelConfig):
    kh, vh, d = cfg.linear_k_heads, cfg.linear_v_heads, cfg.linear_head_dim
    return dict(kh=kh, vh=vh, dk=d, dv=d, r=vh // kh, qkvz=2 * kh * d + 2 * vh * d, ba=2 * vh,
                conv_ch=2 * kh * d + vh * d, vdim=vh * d)


def expert_codec(rng: random.Random, ternary_fraction: float):
    """Per-tensor codec of a routed expert matrix: binary, or ternary (2-bit uniform) with the
    given probability (drawn from the artifact seed)."""
    return (UNIFORM, 2) if rng.random() < ternary_fraction else (BINARY, 1)


def random_qwen_next_weights(cfg: ModelConfig, device, seed: int = 0, std: float = 0.02,
                             ternary_fraction: float = 0.10, group: int = 64, materialise: bool = False,
                             shard: Optional[tuple] = None) -> QNWeights:
    """Random-init weights in the benchmark's mixed recipe. ``materialise`` draws Gaussian weights
    and encodes them (small configs / tests); otherwise random codes and Gaussian-statistics
    scales are written directly (the 80B benchmark model). ``shard`` = (rank, world): only that
    rank's tensor / expert-parallel shard, in its shapes (``parallel.ep.local_qwen_next_config``);
    the replicated router and shared-expert gate agree on every rank."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    gs = torch.Generator(device=device)
    gs.manual_seed(seed + 7919)  # replicated tensors
    rng = random.Random(seed)
    rank, world = shard or (0, 1)
    E_all = cfg.n_experts
    if world > 1:
        from ..parallel.ep import local_qwen_next_config
        g.manual_seed(seed * 1009 + 1 + rank)
        cfg = local_qwen_next_config(cfg, world)
    H, E, F, Fs, V = cfg.hidden, cfg.n_experts // world, cfg.expert_ffn, cfg.shared_ffn, cfg.vocab // world
    nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    dm = dims(cfg)
    ws: List[MixedWeight] = []

    def add(N, K, kind, bits):
        if materialise:
            w = torch.randn(N, K, generator=g, device=device) * std
            ws.append(MixedWeight.quantize(w, kind, bits, group))
        else:
            ws.append(MixedWeight.random(N, K, kind, bits, group, std, g, device))
        return len(ws) - 1

    def ones(n):
        return torch.ones(n, device=device)

    layers = []
    for l in range(cfg.layers):
        full = cfg.layer_is_full_attention(l)
        L = QNLayer(full, attn_norm=ones(H), post_norm=ones(H))
        if full:
            L.idx["q"] = add(nh * hd, H, UNIFORM, 4)
            L.idx["g"] = add(nh * hd, H, UNIFORM, 4)
            L.idx["k"] = add(nkv * hd, H, UNIFORM, 4)
            L.idx["v"] = add(nkv * hd, H, UNIFORM, 4)
            L.idx["o"] = add(H, nh * hd, UNIFORM, 4)
            L.q_norm, L.k_norm = ones(hd), ones(hd)
        else:
            L.idx["qkvz"] = add(dm["qkvz"], H, UNIFORM, 4)
            L.idx["ba"] = add(dm["ba"], H, UNIFORM, 4)
            L.idx["out"] = add(H, dm["vdim"], UNIFORM, 4)
            L.conv_w = torch.randn(dm["conv_ch"], cfg.conv_kernel, generator=g, device=device) * 0.3
            L.a_log = torch.log(torch.rand(dm["vh"], generator=g, device=device) * 15 + 1)
            L.dt_bias = torch.randn(dm["vh"], generator=g, device=device) * 0.5
            L.ssm_norm = ones(dm["dv"])
        L.router = torch.randn(E_all, H, generator=gs if world > 1 else g, device=device) * std
        L.shared_gate = torch.randn(1, H, generator=gs if world > 1 else g, device=device) * std
        L.shared_here = (l % world) == rank
        for m, sm in (("eg", "sg"), ("eu", "su"), ("ed", "sd")):
            n, k = (F, H) if m != "ed" else (H, F)
            L.idx[m] = len(ws)
            for _ in range(E):
                add(n, k, *expert_codec(rng, ternary_fraction))
            if world > 1 and L.shared_here:  # the shared expert follows this rank's routed experts
                L.idx[sm] = add(Fs if m != "ed" else H, H if m != "ed" else Fs, UNIFORM, 4)
        if world == 1:
            L.idx["sg"] = add(Fs, H, UNIFORM, 4)
            L.idx["su"] = add(Fs, H, UNIFORM, 4)
            L.idx["sd"] = add(H, Fs, UNIFORM, 4)
        layers.append(L)
    head = add(V, H, UNIFORM, 4)
    emb = QWeight.quantize(torch.randn(cfg.vocab, H, generator=gs if world > 1 else g, device=device) * std, 1)
    torch.cuda.synchronize(device)
    return QNWeights(MixedTable(ws), emb, ones(H), layers, head, e_lo=rank * E if world > 1 else 0,
                     e_count=E if world > 1 else 0)


class QwenNextModel:
    """Decode forward over static buffers (rows <= 8, one token per row)."""

    def __init__(self, cfg: ModelConfig, w: QNWeights, kv, max_rows: int = 8, max_seqs: int = 8, device="cuda",
                 tp=None):
        """With ``tp`` (parallel.tp.TPComm), ``cfg`` and ``w`` are this rank's shard
        (``parallel.ep.local_qwen_next_config`` / ``shard_qwen_next_weights``): two push all-reduce
        sites per layer (mixer output, expert combine), each consumed by the next RMSNorm."""
        self.cfg, self.w, self.kv, self.dev = cfg, w, kv, torch.device(device)
        self.tp = tp
        # decode takes up to 8 rows; a prompt prefills in forwards of up to max_rows rows (every
        # kernel loops its rows; the expert kernels read each expert's codes once per CTA for all
        # of its pairs); tensor-parallel forwards stay at 8 rows (push all-reduce sites)
        self.max_rows = R = max_rows
        self.max_logit_rows = min(R, 64)  # rows whose logits one forward can return
        dev = self.dev
        H, nh, nkv, hd = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        dm = self.dm = dims(cfg)
        E, k, F, Fs = cfg.n_experts, cfg.top_k, cfg.expert_ffn, cfg.shared_ffn
        self.full_index = {}
        self.lin_index = {}
        for l in range(cfg.layers):
            if cfg.layer_is_full_attention(l):
                self.full_index[l] = len(self.full_index)
            else:
                self.lin_index[l] = len(self.lin_index)
        from .llama import StepInputs
        self.inp = StepInputs(R, dev)
        self.x = torch.zeros(R, H, device=dev)
        self.xa = Q8Act(R, H, dev)
        self.qkv = torch.zeros(R, (nh + 2 * nkv) * hd, device=dev)
        self.gate = torch.zeros(R, nh * hd, device=dev)
        self.q = torch.zeros(R, nh, hd, device=dev)
        self.att = torch.zeros(R, nh * hd, device=dev)
        self.attq = Q8Act(R, nh * hd, dev)
        self.qkvz = torch.zeros(R, dm["qkvz"], device=dev)
        self.ba = torch.zeros(R, dm["ba"], device=dev)
        self.dq = torch.zeros(R, dm["vh"], dm["dk"], device=dev)
        self.dk_ = torch.zeros(R, dm["vh"], dm["dk"], device=dev)
        self.dv_ = torch.zeros(R, dm["vdim"], device=dev)
        self.dz = torch.zeros(R, dm["vdim"], device=dev)
        self.dout = Q8Act(R, dm["vdim"], dev)
        nl = max(1, len(self.lin_index))
        self.conv_state = torch.zeros(nl, max_seqs, dm["conv_ch"], cfg.conv_kernel - 1, device=dev)
        self.ssm_state = torch.zeros(nl, max_seqs, dm["vh"], dm["dk"], dm["dv"], device=dev)
        self.rlog = torch.zeros(R, E, device=dev)
        self.sglog = torch.zeros(R, 1, device=dev)
        self.ids = torch.zeros(R, k, dtype=torch.int32, device=dev)
        self.rw = torch.zeros(R, k, device=dev)
        self.counts = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        self.offsets = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        self.sorted = torch.zeros(R * k + R, dtype=torch.int32, device=dev)
        self.active = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        self.n_active = torch.zeros(1, dtype=torch.int32, device=dev)
        self.route_counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fused_route = cfg.hidden % 512 == 0 and E < 1024
        self.gx = Q8Act(R * k + R, H, dev)
        self.hx = Q8Act(R * k + R, F, dev)
        self.hs = Q8Act(R, Fs, dev)
        # this rank's vocabulary slice under tensor parallelism
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.prefill = None  # ops/prefill.py MoePrefill, made at the first forward of more than 8 rows
        self.wide = None     # ops/prefill.py WideLinear (dense projections of wide forwards)
        self.xb = self.attb = self.doutb = None
        if R > 8:  # bf16 rows of the wide forwards' tensor-core GEMMs
            bf = dict(dtype=torch.bfloat16, device=dev)
            self.xb = torch.zeros(R, H, **bf)
            self.attb = torch.zeros(R, nh * hd, **bf)
            self.doutb = torch.zeros(R, dm["vdim"], **bf)
        self.logits = torch.zeros(self.max_logit_rows, w.table.weights[w.lm_head].N, device=dev)
        self.xh = Q8Act(self.max_logit_rows, H, dev)  # normed rows of the requested logits
        if tp is not None:
            if not self.fused_route:
                raise ValueError("qwen3next tensor parallelism needs the fused routing kernel (hidden % 512 == 0)")
            self.x2 = torch.zeros(R, H, device=dev)  # second residual buffer of the push all-reduce
            if R > 8:
                self.partial = torch.zeros(R, H, device=dev)  # wide forwards: NCCL all-reduce partials
            self.argmax_slots = torch.zeros(R, ops.ARGMAX_SLOTS, dtype=torch.int64, device=dev)
        self.next_ids = torch.zeros(R, dtype=torch.int32, device=dev)
        self.rope = ops.rope_table(cfg.max_ctx, cfg.rope_dim, cfg.rope_theta, None, dev)
        self.scale = 1.0 / math.sqrt(hd)
        self.part_o = torch.zeros(R * 8 * nh * hd, device=dev)
        self.part_lse = torch.zeros(R * 8 * nh, device=dev)
        self.attn_counters = torch.zeros(R * nkv, dtype=torch.int32, device=dev)
        self._graphs = {}
        self.launches_per_graph = 0
        from .deepseek import engine_buffers
        engine_buffers(self, R)

    row_limit = property(lambda self: self.max_rows)  # rows one forward takes (engine chunking)
    # rows of one sequence may share a forward (consecutive, in position order): the DeltaNet
    # kernels walk such a run token by token with the states carried across it
    serial_rows = False

    def reset_state(self, slot: int):
        self.conv_state[:, slot].zero_()
        self.ssm_state[:, slot].zero_()

    def num_splits(self, rows: int) -> int:
        s = 1
        while s < 8 and rows * self.cfg.n_kv_heads * s < 148:
            s *= 2
        return s

    def _wide(self, rows) -> bool:
        """This forward's projections run as tensor-core GEMMs over bf16 rows (prefill)."""
        if rows <= 8 or self.xb is None:
            return False
        c, dm = self.cfg, self.dm
        if any(d % 128 for d in (c.hidden, c.n_heads * c.head_dim, dm["vdim"])):
            return False  # the GEMM's K runs in 128-element stages
        if self.wide is None:
            from ..ops.prefill import WideLinear
            self.wide = WideLinear(self.w.table, self.dev, self.status)
        return True

    def _full(self, l, L, rows, site: int = -1, resid: Optional[torch.Tensor] = None):
        cfg, w, kv, inp = self.cfg, self.w, self.kv, self.inp
        nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        t, xa = w.table, self.xa.view(rows)
        Qn, Kn = nh * hd, nkv * hd
        wide = site < 0 and self._wide(rows)
        if wide:
            ops.rmsnorm(self.x[:rows], L.attn_norm, cfg.eps, yb=self.xb[:rows])
            xb, W = self.xb[:rows], self.wide
            W.linear(L.idx["q"], xb, self.qkv[:rows, :Qn])
            W.linear(L.idx["k"], xb, self.qkv[:rows, Qn:Qn + Kn])
            W.linear(L.idx["v"], xb, self.qkv[:rows, Qn + Kn:])
            W.linear(L.idx["g"], xb, self.gate[:rows])
        else:
            mixed_gemv(t, L.idx["q"], xa, self.qkv[:rows, :Qn])
            mixed_gemv(t, L.idx["k"], xa, self.qkv[:rows, Qn:Qn + Kn])
            mixed_gemv(t, L.idx["v"], xa, self.qkv[:rows, Qn + Kn:])
            mixed_gemv(t, L.idx["g"], xa, self.gate[:rows])
        kl = self.full_index[l]
        ops.rope_append(self.qkv[:rows], inp.positions[:rows], None, self.rope, cfg.rope_dim, cfg.rope_style,
                        self.q[:rows], kv.k[kl], kv.v[kl], nh, nkv, hd, kv.block_size, q_norm=L.q_norm,
                        k_norm=L.k_norm, eps=cfg.eps, block_tables=kv.block_tables, row_seq=inp.row_seq[:rows])
        ops.attention_decode(self.q[:rows], kv.k[kl], kv.v[kl], kv.block_tables, inp.row_seq[:rows],
                             inp.row_ctx[:rows], self.scale, self.num_splits(rows), self.part_o, self.part_lse,
                             out=self.att[:rows], counters=self.attn_counters)
        ops.launches.add()
        kernels().sigmoid_gate_q8(self.att[:rows], self.gate[:rows], self.attq.q[:rows], self.attq.d[:rows],
                                  self.attq.s[:rows], ops.PDL)
        if site >= 0:
            mixed_gemv_push(t, L.idx["o"], self.attq.view(rows), self.tp, site)
        elif wide:
            from ..ops.prefill import q8_to_bf16
            q8_to_bf16(self.attq.view(rows), self.attb[:rows])
            self.wide.linear(L.idx["o"], self.attb[:rows], resid if resid is not None else self.x[:rows],
                             residual=True)
        else:
            mixed_gemv(t, L.idx["o"], self.attq.view(rows), self.x[:rows], residual=True)

    def _linear(self, l, L, rows, site: int = -1, resid: Optional[torch.Tensor] = None):
        cfg, t, dm, inp = self.cfg, self.w.table, self.dm, self.inp
        xa = self.xa.view(rows)
        li = self.lin_index[l]
        wide = site < 0 and self._wide(rows)
        if wide:
            ops.rmsnorm(self.x[:rows], L.attn_norm, cfg.eps, yb=self.xb[:rows])
            self.wide.linear(L.idx["qkvz"], self.xb[:rows], self.qkvz[:rows])
            self.wide.linear(L.idx["ba"], self.xb[:rows], self.ba[:rows])
        else:
            mixed_gemv(t, L.idx["qkvz"], xa, self.qkvz[:rows])
            mixed_gemv(t, L.idx["ba"], xa, self.ba[:rows])
        ops.launches.add(2)
        kernels().deltanet_conv(self.qkvz[:rows], L.conv_w, self.conv_state[li], inp.row_seq[:rows], dm["kh"], dm["r"],
                                dm["dk"], dm["dv"], cfg.conv_kernel, cfg.eps, self.dq[:rows], self.dk_[:rows],
                                self.dv_[:rows], self.dz[:rows], ops.PDL)
        kernels().deltanet_recurrent(self.ssm_state[li], inp.row_seq[:rows], self.dq[:rows], self.dk_[:rows],
                                     self.dv_[:rows], self.dz[:rows], self.ba[:rows], L.a_log, L.dt_bias, dm["r"],
                                     dm["dk"], dm["dv"], L.ssm_norm, cfg.eps, None, self.dout.q[:rows],
                                     self.dout.d[:rows], self.dout.s[:rows], ops.PDL)
        if site >= 0:
            mixed_gemv_push(t, L.idx["out"], self.dout.view(rows), self.tp, site)
        elif wide:
            from ..ops.prefill import q8_to_bf16
            q8_to_bf16(self.dout.view(rows), self.doutb[:rows])
            self.wide.linear(L.idx["out"], self.doutb[:rows], resid if resid is not None else self.x[:rows],
                             residual=True)
        else:
            mixed_gemv(t, L.idx["out"], self.dout.view(rows), self.x[:rows], residual=True)

    def _moe_tp(self, L, rows, site: int):
        """Expert-parallel MoE: routing replicated (every rank scores all experts from the same
        hidden state), this rank's experts plus, on rank l mod N, the shared expert as one more
        pair per token weighted by sigmoid(shared-gate logit); the combine pushes each token's sum
        into every rank's receive region of ``site``."""
        cfg, t, tp, K = self.cfg, self.w.table, self.tp, kernels()
        k, H, F = cfg.top_k, cfg.hidden, cfg.expert_ffn
        xa = self.xa.view(rows)
        ne, e_lo = self.w.e_count, self.w.e_lo
        fold = L.shared_here
        ops.router_logits(L.shared_gate, xa, self.sglog[:rows])
        ops.moe_route(L.router, xa, k, 0, None, 1, 1, cfg.norm_topk, 1.0, self.rlog[:rows], self.ids[:rows],
                      self.rw[:rows], self.counts, self.offsets, self.sorted, self.active, self.n_active, fold,
                      self.route_counter, e_lo=e_lo, e_hi=e_lo + ne)
        ops.launches.add(2)
        na = min(ne, rows * k) + (1 if fold else 0)
        ep = dict(e_lo=e_lo, e_count=ne)
        K.moe_mixed_gemv(0, t.descs, L.idx["eg"], L.idx["eu"], F, H, k, self.counts, self.offsets, self.sorted,
                         self.active, self.n_active, na, xa.q, xa.d, xa.s, self.hx.q, self.hx.d, self.hx.s, None, None,
                         ops.PDL, rows * k, True, **ep)
        K.moe_mixed_gemv(2, t.descs, L.idx["ed"], L.idx["ed"], H, F, k, self.counts, self.offsets, self.sorted,
                         self.active, self.n_active, na, self.hx.q, self.hx.d, self.hx.s, None, None, None, None,
                         self.rw[:rows].reshape(-1), ops.PDL, rows * k, T=rows, push_table=tp.push_recv[site],
                         push_epoch=tp.epoch, shared_gate=self.sglog[:rows], **ep)

    def _moe(self, L, rows, resid: Optional[torch.Tensor] = None):
        cfg, t = self.cfg, self.w.table
        E, k, H, F = cfg.n_experts, cfg.top_k, cfg.hidden, cfg.expert_ffn
        xa = self.xa.view(rows)
        ops.router_logits(L.shared_gate, xa, self.sglog[:rows])
        K = kernels()
        if rows > 8 and cfg.shared_ffn == F and F % 128 == 0 and H % 128 == 0 and MOE_PREFILL:
            # prefill: experts as two grouped tensor-core GEMMs (ops/prefill.py), the gated shared
            # expert folded in as one more group weighted by sigmoid(its gate logit)
            from ..ops.prefill import MoePrefill
            if self.prefill is None:
                self.prefill = MoePrefill(t, self.dev, E, F, H, self.max_rows * (k + 1), self.status)
            ops.rmsnorm(self.x[:rows], L.post_norm, cfg.eps, yb=self.xb[:rows])
            ops.router_logits(L.router, xa, self.rlog[:rows])
            ops.moe_topk(self.rlog[:rows], None, k, 0, 1, 1, cfg.norm_topk, 1.0, self.ids[:rows], self.rw[:rows])
            # under expert parallelism: this rank's experts, and the shared expert where it lives
            fold = "sg" in L.idx
            ops.moe_align(self.ids[:rows], E, xa, self.counts, self.offsets, self.sorted, None, shared=fold)
            self.prefill.run(L.idx, rows, k, self.xb[:rows], resid if resid is not None else self.x[:rows],
                             self.counts, self.offsets, self.sorted, self.rw[:rows], fold,
                             shared_gate=self.sglog[:rows], pdl=ops.PDL, e_lo=self.w.e_lo, e_count=self.w.e_count,
                             ids=self.ids[:rows])
            return
        fused = self.fused_route and rows <= 8
        if fused:  # router GEMV, top-k, sort by expert and active list in one launch
            ops.moe_route(L.router, xa, k, 0, None, 1, 1, cfg.norm_topk, 1.0, self.rlog[:rows], self.ids[:rows],
                          self.rw[:rows], self.counts, self.offsets, self.sorted, self.active, self.n_active, False,
                          self.route_counter)
            gin = xa
        else:
            ops.router_logits(L.router, xa, self.rlog[:rows])
            ops.moe_topk(self.rlog[:rows], None, k, 0, 1, 1, cfg.norm_topk, 1.0, self.ids[:rows], self.rw[:rows])
            ops.moe_align(self.ids[:rows], E, xa, self.counts, self.offsets, self.sorted, self.gx)
            ops.launches.add()
            K.moe_active(self.counts, self.active, self.n_active, ops.PDL)
            gin = self.gx
        ops.launches.add(2)
        na = min(E, rows * k)
        K.moe_mixed_gemv(0, t.descs, L.idx["eg"], L.idx["eu"], F, H, k, self.counts, self.offsets, self.sorted,
                         self.active, self.n_active, na, gin.q, gin.d, gin.s, self.hx.q, self.hx.d,
                         self.hx.s, None, None, ops.PDL, rows * k, fused)
        K.moe_mixed_gemv(1, t.descs, L.idx["ed"], L.idx["ed"], H, F, k, self.counts, self.offsets, self.sorted,
                         self.active, self.n_active, na, self.hx.q, self.hx.d, self.hx.s, None, None, None,
                         self.x[:rows], self.rw[:rows].reshape(-1), ops.PDL)
        hs = self.hs.view(rows)
        mixed_gemv_swiglu(t, L.idx["sg"], L.idx["su"], xa, hs)
        mixed_gemv(t, L.idx["sd"], hs, self.x[:rows], residual=True, gate_logit=self.sglog[:rows])

    def forward(self, rows: int, sample: str = "greedy", advance: bool = False, n_logits: int = 0):
        """``n_logits`` (engine): > 0 moves the logits / greedy ids of ``logit_rows[:n_logits]`` to
        the first rows. Rows must belong to distinct sequences (``serial_rows``)."""
        from .deepseek import compact_logit_rows
        if self.tp is not None and rows > 8:
            self._forward_tp_wide(rows, sample, advance, n_logits)
        elif self.tp is not None:
            self._forward_tp(rows, sample, advance)
            compact_logit_rows(self, n_logits)
        else:
            self._forward(rows, sample, advance, n_logits)

    def _forward_tp_wide(self, rows: int, sample: str, advance: bool, n_logits: int):
        """Tensor / expert-parallel prefill forward of more than 8 rows: this rank's heads and
        experts as tensor-core GEMMs into a zeroed partial, summed over the ranks by an NCCL
        all-reduce after each mixer and each MoE block (the push sites hold 8 rows); the LM head
        runs on the sampled rows only."""
        import torch.distributed as dist
        cfg, w, inp, tp = self.cfg, self.w, self.inp, self.tp
        nl = n_logits if n_logits > 0 else (0 if n_logits < 0 else rows)
        if nl > self.max_logit_rows:
            raise ValueError(f"forward: logits for {nl} rows requested, at most {self.max_logit_rows}")
        ops.tp_begin(tp)
        x, xa, p = self.x[:rows], self.xa.view(rows), self.partial[:rows]
        ops.embed(w.embed, inp.ids[:rows], x)
        for l, L in enumerate(w.layers):
            ops.rmsnorm_q8(x, L.attn_norm, cfg.eps, xa)
            p.zero_()
            if L.full:
                self._full(l, L, rows, resid=p)
            else:
                self._linear(l, L, rows, resid=p)
            dist.all_reduce(p, group=tp.group)
            x.add_(p)
            ops.rmsnorm_q8(x, L.post_norm, cfg.eps, xa)
            p.zero_()
            self._moe(L, rows, resid=p)
            dist.all_reduce(p, group=tp.group)
            x.add_(p)
        if nl:
            ops.rmsnorm_q8(x, w.out_norm, cfg.eps, xa)
            xh = xa
            if n_logits > 0:
                idx = self.logit_rows[:nl].long()
                for src, dst in ((self.xa.q, self.xh.q), (self.xa.d, self.xh.d), (self.xa.s, self.xh.s)):
                    torch.index_select(src, 0, idx, out=dst[:nl])
                xh = self.xh.view(nl)
            head = w.table.weights[w.lm_head]
            if sample == "greedy" and nl <= 8:
                mixed_gemv(w.table, w.lm_head, xh, self.logits[:nl], argmax_slots=self.argmax_slots[:nl],
                           argmax_offset=tp.rank * head.N)
                ops.tp_argmax(tp, self.argmax_slots, nl, self.next_ids)
            else:  # logits only (this rank's vocabulary slice)
                mixed_gemv(w.table, w.lm_head, xh, self.logits[:nl])
        if advance:
            ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)

    def _forward_tp(self, rows: int, sample: str, advance: bool):
        cfg, w, inp, tp = self.cfg, self.w, self.inp, self.tp
        ops.tp_begin(tp)
        xa_res, xb_res = self.x[:rows], self.x2[:rows]
        ops.embed(w.embed, inp.ids[:rows], xa_res)
        ops.rmsnorm_q8(xa_res, w.layers[0].attn_norm, cfg.eps, self.xa.view(rows))
        for l, L in enumerate(w.layers):
            if L.full:
                self._full(l, L, rows, site=2 * l)
            else:
                self._linear(l, L, rows, site=2 * l)
            ops.tp_allreduce_rmsnorm_q8(tp, 2 * l, xa_res, xb_res, L.post_norm, cfg.eps, self.xa.view(rows))
            self._moe_tp(L, rows, 2 * l + 1)
            nxt = w.layers[l + 1].attn_norm if l + 1 < len(w.layers) else w.out_norm
            ops.tp_allreduce_rmsnorm_q8(tp, 2 * l + 1, xb_res, xa_res, nxt, cfg.eps, self.xa.view(rows))
        head = w.table.weights[w.lm_head]
        if sample == "greedy":
            mixed_gemv(w.table, w.lm_head, self.xa.view(rows), self.logits[:rows],
                       argmax_slots=self.argmax_slots[:rows], argmax_offset=tp.rank * head.N)
            ops.tp_argmax(tp, self.argmax_slots, rows, self.next_ids)
        elif sample == "none":
            mixed_gemv(w.table, w.lm_head, self.xa.view(rows), self.logits[:rows])
        else:  # vocabulary-parallel logits, gathered; every rank draws the same token
            mixed_gemv(w.table, w.lm_head, self.xa.view(rows), self.logits[:rows])
            ops.sample(self.gathered_logits(rows), self.temperature[:rows], self.top_k[:rows], self.top_p[:rows],
                       self.rep_penalty[:rows], None, self.uniforms[:rows], self.next_ids[:rows])
        if advance:
            ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)

    def gathered_logits(self, nl: int) -> torch.Tensor:
        """Logits of the first ``nl`` rows over the whole vocabulary (the ranks' slices gathered
        under tensor parallelism; a collective every rank calls for the same rows)."""
        if self.tp is None:
            return self.logits[:nl]
        from ..parallel.tp import gather_vocab_logits
        if getattr(self, "_tp_full", None) is None:
            self._tp_full = torch.zeros(self.logits.shape[0], self.logits.shape[1] * self.tp.world, device=self.dev)
        return gather_vocab_logits(self.tp, self.logits[:nl], self._tp_full)

    def _forward(self, rows: int, sample: str = "greedy", advance: bool = False, n_logits: int = 0):
        cfg, w, inp = self.cfg, self.w, self.inp
        nl = n_logits or rows
        if nl > self.max_logit_rows:
            raise ValueError(f"forward: logits for {nl} rows requested, at most {self.max_logit_rows}")
        ops.embed(w.embed, inp.ids[:rows], self.x[:rows])
        for l, L in enumerate(w.layers):
            ops.rmsnorm_q8(self.x[:rows], L.attn_norm, cfg.eps, self.xa.view(rows))
            if L.full:
                self._full(l, L, rows)
            else:
                self._linear(l, L, rows)
            ops.rmsnorm_q8(self.x[:rows], L.post_norm, cfg.eps, self.xa.view(rows))
            self._moe(L, rows)
        if n_logits < 0:  # no row of this forward is sampled
            if advance:
                ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)
            return
        ops.rmsnorm_q8(self.x[:rows], w.out_norm, cfg.eps, self.xa.view(rows))
        xh = self.xa.view(rows)
        if n_logits:  # only the requested rows go through the LM head, in request order
            idx = self.logit_rows[:nl].long()
            for src, dst in ((self.xa.q, self.xh.q), (self.xa.d, self.xh.d), (self.xa.s, self.xh.s)):
                torch.index_select(src, 0, idx, out=dst[:nl])
            xh = self.xh.view(nl)
        mixed_gemv(w.table, w.lm_head, xh, self.logits[:nl])
        if sample == "greedy":
            ops.argmax(self.logits[:nl], self.next_ids[:nl])
        if advance:
            ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)

    def forward_tokens(self, tokens, seq_id: int = 0, start_pos: int = 0) -> torch.Tensor:
        """Teacher-forced forward of one sequence in chunks of up to ``max_rows`` tokens (the
        DeltaNet kernels run each chunk's recurrence token by token); fp32 logits [n, vocab]."""
        kv = self.kv
        n = len(tokens)
        if not kv.bm.reserve(seq_id, start_pos + n):
            raise RuntimeError("KV pool exhausted")
        kv.sync_tables([seq_id])
        r = kv.row(seq_id)
        if start_pos == 0:
            self.reset_state(r)
        out = torch.empty(n, self.logits.shape[1], device=self.dev)  # this rank's vocabulary slice under TP
        step = min(self.max_rows, self.max_logit_rows)
        for c0 in range(0, n, step):
            c1 = min(n, c0 + step)
            p0 = start_pos + c0
            slots = kv.bm.slots(seq_id, p0, start_pos + c1)
            pos = list(range(p0, start_pos + c1))
            self.inp.upload([int(t) for t in tokens[c0:c1]], pos, slots, [r] * (c1 - c0), [p + 1 for p in pos])
            self.forward(c1 - c0, "greedy")
            out[c0:c1] = self.logits[: c1 - c0]
        return out

    def graph_forward(self, rows: int, sample: str = "greedy", advance: bool = False):
        key = (rows, sample, advance)
        g = self._graphs.get(key)
        if g is None:
            # the warm-up forward (lazy set-up outside the capture) advances the recurrent state:
            # keep a copy and put it back, so the step's replay is its only update
            saved = (self.conv_state.clone(), self.ssm_state.clone())
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(s):
                self.forward(rows, "none")
            torch.cuda.current_stream(self.dev).wait_stream(s)
            self.conv_state.copy_(saved[0])
            self.ssm_state.copy_(saved[1])
            del saved
            g = torch.cuda.CUDAGraph()
            n0 = ops.launches.n
            with torch.cuda.graph(g):
                self.forward(rows, sample, advance)
            self.launches_per_graph = ops.launches.n - n0
            self._graphs[key] = g
        g.replay()

    def release_graphs(self):
        self._graphs.clear()


# ---- fp32 PyTorch reference (test oracle) -----------------------------------------------------
class TorchRefQwenNext:
    """Token-serial fp32 restatement of the same decoder (dequantised weights, exact softmax and
    recurrence), used to check the device forward."""

    def __init__(self, cfg: ModelConfig, w: QNWeights, act_q8: bool = True, bf16_kv: bool = True):
        """``act_q8`` rounds every projection input to int8 blocks of 32 (d = amax / 127) and
        ``bf16_kv`` stores the attention cache in bf16, as the device does; the remaining
        difference is summation order."""
        self.cfg, self.w = cfg, w
        self.act_q8, self.bf16_kv = act_q8, bf16_kv
        self.W = [mw.dequantize() for mw in w.table.weights]
        self.E = w.embed.dequantize()
        self.reset()

    def reset(self):
        cfg, dm = self.cfg, dims(self.cfg)
        dev = self.E.device
        self.kcache = {l: [] for l in range(cfg.layers) if cfg.layer_is_full_attention(l)}
        self.vcache = {l: [] for l in self.kcache}
        self.conv = {l: torch.zeros(dm["conv_ch"], cfg.conv_kernel - 1, device=dev)
                     for l in range(cfg.layers) if not cfg.layer_is_full_attention(l)}
        self.S = {l: torch.zeros(dm["vh"], dm["dk"], dm["dv"], device=dev) for l in self.conv}

    @staticmethod
    def _rms(x, w, eps):
        return x * torch.rsqrt((x * x).mean() + eps) * w

    def _q(self, v):
        if not self.act_q8:
            return v
        b = v.reshape(-1, 32)
        d = b.abs().amax(1, keepdim=True) / 127.0
        q = torch.where(d > 0, torch.round(b / torch.where(d > 0, d, torch.ones_like(d))), torch.zeros_like(b))
        return (q * d).reshape(v.shape)

    def _rope(self, x, pos):  # neox halves over the first rot dims of each head
        cfg = self.cfg
        rd = cfg.rope_dim
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, rd, 2, device=x.device, dtype=torch.float64) / rd))
        ang = (pos * inv).float()
        c, s = torch.cos(ang), torch.sin(ang)
        a, b = x[..., : rd // 2], x[..., rd // 2: rd]
        out = x.clone()
        out[..., : rd // 2] = a * c - b * s
        out[..., rd // 2: rd] = b * c + a * s
        return out

    def step(self, token: int, pos: int) -> torch.Tensor:
        cfg, w, W, dm = self.cfg, self.w, self.W, dims(self.cfg)
        nh, nkv, hd = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        x = self.E[token].clone()
        for l, L in enumerate(w.layers):
            h = self._q(self._rms(x, L.attn_norm, cfg.eps))
            if L.full:
                q = (W[L.idx["q"]] @ h).view(nh, hd)
                gte = W[L.idx["g"]] @ h
                k = (W[L.idx["k"]] @ h).view(nkv, hd)
                v = (W[L.idx["v"]] @ h).view(nkv, hd)
                q = torch.stack([self._rms(q[i], L.q_norm, cfg.eps) for i in range(nh)])
                k = torch.stack([self._rms(k[i], L.k_norm, cfg.eps) for i in range(nkv)])
                q, k = self._rope(q, pos), self._rope(k, pos)
                if self.bf16_kv:
                    k, v = k.bfloat16().float(), v.bfloat16().float()
                self.kcache[l].append(k)
                self.vcache[l].append(v)
                K = torch.stack(self.kcache[l])  # [T, nkv, hd]
                V = torch.stack(self.vcache[l])
                G = nh // nkv
                o = torch.empty(nh, hd, device=x.device)
                for i in range(nh):
                    sc = (K[:, i // G] @ q[i]) / math.sqrt(hd)
                    o[i] = torch.softmax(sc, 0) @ V[:, i // G]
                o = self._q(o.reshape(-1) * torch.sigmoid(gte))
                x = x + W[L.idx["o"]] @ o
            else:
                kh, vh, dk, dv, r = dm["kh"], dm["vh"], dm["dk"], dm["dv"], dm["r"]
                p = W[L.idx["qkvz"]] @ h
                ba = W[L.idx["ba"]] @ h
                per = 2 * dk + 2 * r * dv
                qs, ks, vs, zs = [], [], [], []
                for i in range(kh):
                    blk = p[i * per:(i + 1) * per]
                    qs.append(blk[:dk]); ks.append(blk[dk:2 * dk])
                    vs.append(blk[2 * dk:2 * dk + r * dv]); zs.append(blk[2 * dk + r * dv:])
                ch_in = torch.cat(qs + ks + vs)
                st = self.conv[l]
                full = torch.cat([st, ch_in[:, None]], 1)  # [ch, kc]
                conv = (full * L.conv_w).sum(1)
                conv = conv / (1 + torch.exp(-conv))
                self.conv[l] = full[:, 1:].clone()
                qc = conv[:kh * dk].view(kh, dk)
                kc = conv[kh * dk:2 * kh * dk].view(kh, dk)
                vc = conv[2 * kh * dk:].view(vh, dv)
                z = torch.cat(zs).view(vh, dv)
                qn = qc * torch.rsqrt((qc * qc).sum(1, keepdim=True) + cfg.eps) / math.sqrt(dk)
                kn = kc * torch.rsqrt((kc * kc).sum(1, keepdim=True) + cfg.eps)
                out = torch.empty(vh, dv, device=x.device)
                for j in range(vh):
                    i = j // r
                    bb = ba[i * 2 * r + j % r]
                    aa = ba[i * 2 * r + r + j % r]
                    sp = torch.nn.functional.softplus(aa + L.dt_bias[j])
                    decay = torch.exp(-torch.exp(L.a_log[j]) * sp)
                    beta = torch.sigmoid(bb)
                    S = self.S[l][j] * decay
                    kv = S.t() @ kn[i]
                    delta = (vc[j] - kv) * beta
                    S = S + torch.outer(kn[i], delta)
                    self.S[l][j] = S
                    o = S.t() @ qn[i]
                    o = o * torch.rsqrt((o * o).mean() + cfg.eps) * L.ssm_norm * (z[j] / (1 + torch.exp(-z[j])))
                    out[j] = o
                x = x + W[L.idx["out"]] @ self._q(out.reshape(-1))
            h = self._q(self._rms(x, L.post_norm, cfg.eps))
            logits = L.router @ h
            p = torch.softmax(logits, 0)
            top = torch.topk(p, cfg.top_k)
            wts = top.values / top.values.sum() if cfg.norm_topk else top.values
            for e, wt in zip(top.indices.tolist(), wts):
                gt = W[L.idx["eg"] + e] @ h
                up = W[L.idx["eu"] + e] @ h
                x = x + wt * (W[L.idx["ed"] + e] @ self._q(gt / (1 + torch.exp(-gt)) * up))
            gt = W[L.idx["sg"]] @ h
            up = W[L.idx["su"]] @ h
            sgate = torch.sigmoid(L.shared_gate[0] @ h)
            x = x + sgate * (W[L.idx["sd"]] @ self._q(gt / (1 + torch.exp(-gt)) * up))
        h = self._q(self._rms(x, w.out_norm, cfg.eps))
        return W[w.lm_head] @ h
