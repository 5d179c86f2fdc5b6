"""DeepSeek-V3-style MLA + MoE decoder with fp8 e4m3 block-scaled weights.

Attention is multi-head latent attention: the query goes through a low-rank q_a -> RMSNorm -> q_b;
the key/value through kv_a -> (RMSNorm'd 512-d latent, 64-d RoPE key) that is all the paged cache
holds; the key and value up-projections are absorbed into the query (q_lat = W_UK^T q_nope) and the
output (o = W_UV o_lat), so decode attends directly over the latent cache (K6 kernels). The first
``first_dense_layers`` layers have a dense SwiGLU FFN; the rest route each token to top-k of many
experts with sigmoid scores plus a learned selection bias, group-limited selection, renormalised
and scaled weights, plus one shared expert. Every projection matrix is fp8 e4m3 with 128 x 128
block scales (K1 fp8 path of the mixed GEMV kernels); W_UK / W_UV are kept in bf16.

Decode runs rows <= 8 through the GEMV path; prompts are fed through the same path in chunks of up
to 8 tokens of one sequence (the latent cache makes multi-row prefill exact).

Across the GPUs of a node (``tp`` given, weights from ``parallel.ep``): attention is tensor
parallel over heads (q_b, W_UK, W_UV and the output projection split by head; q_a / kv_a and the
latent cache replicated), the dense FFN layers split by FFN row, the routed experts expert
parallel (each rank holds E / N whole experts; the shared expert runs on rank l mod N), and the
LM head split by vocabulary row. Every row-parallel result (output projection, FFN down, the
experts' combine) is pushed from its kernel's epilogue into every rank's receive region, and the
next RMSNorm sums the ranks (``csrc/kernels/tp.cu``); greedy sampling reduces per-rank keys.

Parity: crates/hawking-core/src/model/deepseek_v2.rs:72-158 (config: q_lora, kv_lora 512, rope 64,
nope 128, v 128, routed + shared experts, first_k_dense), :2170 (forward_token), crates/hawking-core/
src/attn.rs:185 (mla_decode_step), crates/hawking-core/src/moe.rs:24 (top-k gate),
crates/hawking-core/shaders/attn.metal:18-47 (absorbed MLA decode).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .. import ops
from .._ext import kernels
from ..ops import Q8Act, QWeight
from ..ops.mixed import MixedTable, MixedWeight, mixed_gemv, mixed_gemv_push, mixed_gemv_swiglu
from .config import ModelConfig

LAT, ROPE = 512, 64


@dataclass
class DSLayer:
    dense: bool
    attn_norm: torch.Tensor
    q_a_norm: torch.Tensor
    kv_a_norm: torch.Tensor
    ffn_norm: torch.Tensor
    w_uk: torch.Tensor                  # bf16 [nh, nope, 512]
    w_uv: torch.Tensor                  # bf16 [nh, v, 512]
    idx: Dict[str, int] = field(default_factory=dict)
    router: Optional[torch.Tensor] = None
    router_bias: Optional[torch.Tensor] = None
    shared_here: bool = True            # expert parallel: this rank runs the layer's shared expert


@dataclass
class DSWeights:
    table: MixedTable
    embed: QWeight
    out_norm: torch.Tensor
    layers: List[DSLayer]
    lm_head: int
    e_lo: int = 0                       # expert parallel: this rank's routed experts are
    e_count: int = 0                    # e_lo .. e_lo + e_count - 1 (0: all of them)

    @property
    def nbytes(self) -> int:
        n = self.table.nbytes + self.embed.nbytes
        for l in self.layers:
            n += (l.w_uk.numel() + l.w_uv.numel()) * 2
            if l.router is not None:
                n += l.router.numel() * 4
        return n


def random_deepseek_weights(cfg: ModelConfig, device, seed: int = 0, std: float = 0.02,
                            materialise: bool = True) -> DSWeights:
    """Random-init fp8 weights. ``materialise`` quantises Gaussian weights tile by tile (exact
    recipe); the kernels see identical layouts either way."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    H, nh, V = cfg.hidden, cfg.n_heads, cfg.vocab
    nope, rd, vd = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
    ws: List[MixedWeight] = []

    def add(N, K):
        ws.append(MixedWeight.random_fp8(N, K, std, g, device))
        return len(ws) - 1

    def ones(n):
        return torch.ones(n, device=device)

    layers = []
    for l in range(cfg.layers):
        dense = l < cfg.first_dense_layers
        L = DSLayer(dense, ones(H), ones(cfg.q_lora_rank), ones(LAT), ones(H),
                    w_uk=(torch.randn(nh, nope, LAT, generator=g, device=device) * std).bfloat16(),
                    w_uv=(torch.randn(nh, vd, LAT, generator=g, device=device) * std).bfloat16())
        # q_a and kv_a read the same normed hidden: one [q_lora + 576, H] matrix (one GEMV), with
        # row views for each part
        qakva = MixedWeight.random_fp8(cfg.q_lora_rank + LAT + ROPE, H, std, g, device)
        L.idx["qakva"] = len(ws)
        ws.append(qakva)
        L.idx["qa"] = len(ws)
        ws.append(qakva.rows(0, cfg.q_lora_rank))
        L.idx["kva"] = len(ws)
        ws.append(qakva.rows(cfg.q_lora_rank, LAT + ROPE))
        L.idx["qb"] = add(nh * (nope + rd), cfg.q_lora_rank)
        L.idx["o"] = add(H, nh * vd)
        if dense:
            L.idx["g"] = add(cfg.ffn, H)
            L.idx["u"] = add(cfg.ffn, H)
            L.idx["d"] = add(H, cfg.ffn)
        else:
            E, F = cfg.n_experts, cfg.expert_ffn
            L.router = torch.randn(E, H, generator=g, device=device) * std
            L.router_bias = torch.randn(E, generator=g, device=device) * 0.01
            Fs = cfg.shared_ffn
            for m, sm, (n, k), (ns, ks) in (("eg", "sg", (F, H), (Fs, H)), ("eu", "su", (F, H), (Fs, H)),
                                            ("ed", "sd", (H, F), (H, Fs))):
                # all experts of one matrix drawn at once, then viewed per expert; the shared
                # expert's matrix follows as "expert E" (the MoE kernels run it with the routed ones)
                stacked = MixedWeight.random_fp8(E * n, k, std, g, device)
                L.idx[m] = len(ws)
                for e in range(E):
                    ws.append(stacked.rows(e * n, n))
                L.idx[sm] = add(ns, ks)
        layers.append(L)
    head = add(V, H)
    emb = QWeight.quantize(torch.randn(V, H, generator=g, device=device) * std, 1)  # F16 table
    torch.cuda.synchronize(device)
    return DSWeights(MixedTable(ws), emb, ones(H), layers, head)


class DeepSeekModel:
    """Decode forward over static buffers (rows <= 8)."""

    def __init__(self, cfg: ModelConfig, w: DSWeights, kv, max_rows: int = 8, device="cuda", tp=None):
        """``kv``: PagedKVCache-like object with ``latent[l]`` [num_blocks, block_size, 576] bf16
        per layer, ``block_tables``, ``bm`` (see models.deepseek.LatentCache). With ``tp``
        (parallel.tp.TPComm), ``cfg`` is this rank's shard (heads and dense FFN divided)."""
        self.cfg, self.w, self.kv, self.dev = cfg, w, kv, torch.device(device)
        self.tp = tp
        self.mla_flash = True  # latent attention on the tensor cores (mla_flash.cu)
        # decode takes up to 8 rows; on one GPU a prompt prefills in forwards of up to max_rows rows
        # (the latent cache makes multi-row prefill exact; the absorb / output kernels run in
        # 8-row slices, the experts' kernels read each expert's weights once per CTA for all of its
        # pairs); tensor-parallel forwards stay at 8 rows (push all-reduce sites)
        self.max_rows = R = max_rows
        self.max_logit_rows = min(R, 64)  # rows whose logits one forward can return
        dev = self.dev
        H, nh = cfg.hidden, cfg.n_heads
        nope, rd, vd = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
        E, k = max(cfg.n_experts, 1), max(cfg.top_k, 1)
        F, Fs = max(cfg.expert_ffn, 32), max(cfg.shared_ffn, 32)
        from .llama import StepInputs
        self.inp = StepInputs(R, dev)
        self.x = torch.zeros(R, H, device=dev)
        self.xa = Q8Act(R, H, dev)
        self.qakva = torch.zeros(R, cfg.q_lora_rank + LAT + ROPE, device=dev)
        self.qa = self.qakva[:, :cfg.q_lora_rank]
        self.qaq = Q8Act(R, cfg.q_lora_rank, dev) if cfg.q_lora_rank else None
        self.q = torch.zeros(R, nh * (nope + rd), device=dev)
        self.kva = self.qakva[:, cfg.q_lora_rank:]
        self.q_lat = torch.zeros(R, nh, LAT, device=dev)
        self.q_pe = torch.zeros(R, nh, ROPE, device=dev)
        self.o_lat = torch.zeros(R, nh, LAT, device=dev)
        self.attq = Q8Act(R, nh * vd, dev)
        self.h = Q8Act(R, max(cfg.ffn, 32), dev)
        self.rlog = torch.zeros(R, E, device=dev)
        self.ids = torch.zeros(R, k, dtype=torch.int32, device=dev)
        self.rw = torch.zeros(R, k, device=dev)
        # the shared expert runs as expert E inside the routed launches when its shape matches
        self.fold_shared = cfg.n_experts > 0 and cfg.shared_ffn == cfg.expert_ffn
        self.counts = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        self.offsets = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        self.sorted = torch.zeros(R * k + R, dtype=torch.int32, device=dev)
        self.active = torch.zeros(E + 1, dtype=torch.int32, device=dev)
        self.n_active = torch.zeros(1, dtype=torch.int32, device=dev)
        self.route_counter = torch.zeros(1, dtype=torch.int32, device=dev)
        self.fused_route = cfg.hidden % 512 == 0 and E + 1 <= 1024
        self.gx = Q8Act(R * k + R, H, dev)
        self.hx = Q8Act(R * k + R, F, dev)
        self.hs = Q8Act(R, Fs, dev)
        self.logits = torch.zeros(self.max_logit_rows, cfg.vocab, device=dev)
        self.xh = Q8Act(self.max_logit_rows, H, dev)  # normed rows of the requested logits
        self.next_ids = torch.zeros(R, dtype=torch.int32, device=dev)
        from .deepseek_gguf import yarn_attention_scale, yarn_freq_factors
        self.rope = ops.rope_table(cfg.max_ctx, ROPE, cfg.rope_theta, yarn_freq_factors(cfg), dev)
        self.scale = yarn_attention_scale(cfg)
        self.scoring = 1 if cfg.router == "sigmoid_bias" else 0  # router: sigmoid + bias, or softmax
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.prefill = None  # ops/prefill.py MoePrefill, made at the first forward of more than 8 rows
        self.wide = None     # ops/prefill.py WideLinear (dense projections of wide forwards)
        self.xb = self.qab = self.attb = self.hb = None
        if R > 8:  # bf16 rows of the wide forwards' tensor-core GEMMs
            bf = dict(dtype=torch.bfloat16, device=dev)
            self.xb = torch.zeros(R, H, **bf)
            self.qab = torch.zeros(R, max(cfg.q_lora_rank, 32), **bf)
            self.attb = torch.zeros(R, nh * vd, **bf)
            self.hb = torch.zeros(R, max(cfg.ffn, 32), **bf)
        if tp is not None:
            self.x2 = torch.zeros(R, H, device=dev)  # second residual buffer of the push all-reduce
            if R > 8:
                self.partial = torch.zeros(R, H, device=dev)  # wide forwards: NCCL all-reduce partials
            self.argmax_slots = torch.zeros(R, ops.ARGMAX_SLOTS, dtype=torch.int64, device=dev)
        self._graphs = {}
        self.launches_per_graph = 0
        engine_buffers(self, R)

    row_limit = property(lambda self: self.max_rows)  # rows one forward takes (engine chunking)

    def num_splits(self, rows: int) -> int:
        """KV splits (cluster size, <= 8) so that splits x head groups x rows covers the SMs; the
        kernel groups 4, 2 or 1 heads per CTA (fewer for tensor-parallel head shards)."""
        groups = self.cfg.n_heads // kernels().mla_heads_per_cta(self.cfg.n_heads, rows)
        s = 1
        while s < 8 and rows * groups * s < 148:
            s *= 2
        return s

    def _wide(self, rows) -> bool:
        """This forward's projections run as tensor-core GEMMs over bf16 rows (prefill)."""
        if rows <= 8 or self.xb is None:
            return False
        c = self.cfg
        if any(d % 128 for d in (c.hidden, c.q_lora_rank, c.n_heads * c.v_head_dim)):
            return False  # the GEMM's K runs in 128-element stages
        if self.wide is None:
            from ..ops.prefill import WideLinear
            self.wide = WideLinear(self.w.table, self.dev, self.status)
        return True

    def _attention(self, l, L, rows, resid: Optional[torch.Tensor] = None):
        """One layer's attention; the output projection adds to ``resid`` (default: the residual
        rows; a zeroed partial under tensor parallelism for wide forwards)."""
        cfg, t, kv, inp = self.cfg, self.w.table, self.kv, self.inp
        K = kernels()
        xa = self.xa.view(rows)
        wide = self._wide(rows)
        if wide:
            W = self.wide
            ops.rmsnorm(self.x[:rows], L.attn_norm, cfg.eps, yb=self.xb[:rows])
            xb = self.xb[:rows]
            if "q" in L.idx:
                W.linear(L.idx["q"], xb, self.q[:rows])
                W.linear(L.idx["kva"], xb, self.kva[:rows])
            else:
                if "qakva" in L.idx:
                    W.linear(L.idx["qakva"], xb, self.qakva[:rows])
                else:
                    W.linear(L.idx["qa"], xb, self.qa[:rows])
                    W.linear(L.idx["kva"], xb, self.kva[:rows])
                ops.rmsnorm(self.qa[:rows], L.q_a_norm, cfg.eps, yb=self.qab[:rows, :cfg.q_lora_rank])
                W.linear(L.idx["qb"], self.qab[:rows, :cfg.q_lora_rank], self.q[:rows])
        elif "q" in L.idx:  # no query low-rank: q and kv_a straight from the normed hidden
            mixed_gemv(t, L.idx["q"], xa, self.q[:rows])
            mixed_gemv(t, L.idx["kva"], xa, self.kva[:rows])
        else:
            if "qakva" in L.idx:
                mixed_gemv(t, L.idx["qakva"], xa, self.qakva[:rows])
            else:
                mixed_gemv(t, L.idx["qa"], xa, self.qa[:rows])
                mixed_gemv(t, L.idx["kva"], xa, self.kva[:rows])
            ops.rmsnorm_q8(self.qa[:rows], L.q_a_norm, cfg.eps, self.qaq.view(rows))
            mixed_gemv(t, L.idx["qb"], self.qaq.view(rows), self.q[:rows])
        ops.launches.add(4)
        K.mla_kv_append(self.kva[:rows], L.kv_a_norm, cfg.eps, inp.positions[:rows], kv.block_tables,
                        inp.row_seq[:rows], self.rope, kv.latent[l], ops.PDL)
        if wide:
            # key absorption of every head as one batched bf16 GEMM, and the query RoPE (halves)
            nh, nope = cfg.n_heads, cfg.qk_nope_dim
            qv = self.q[:rows].view(rows, nh, nope + ROPE)
            ql = torch.bmm(qv[:, :, :nope].transpose(0, 1).to(torch.bfloat16), L.w_uk)  # [nh, rows, 512]
            self.q_lat[:rows].copy_(ql.transpose(0, 1))
            cs = self.rope[inp.positions[:rows].long()]                                 # [rows, 32, 2]
            c, sn = cs[:, None, :, 0], cs[:, None, :, 1]
            a, b = qv[:, :, nope:nope + ROPE // 2], qv[:, :, nope + ROPE // 2:]
            self.q_pe[:rows, :, :ROPE // 2] = a * c - b * sn
            self.q_pe[:rows, :, ROPE // 2:] = b * c + a * sn
        else:
            for c0 in range(0, rows, 8):  # the absorb kernel takes up to 8 rows
                c1 = min(rows, c0 + 8)
                K.mla_absorb_q(self.q[c0:c1], L.w_uk, inp.positions[c0:c1], self.rope, self.q_lat[c0:c1],
                               self.q_pe[c0:c1], ops.PDL)
        # num_splits 0: the tensor-core kernel (mla_flash.cu, picks its own splits) for 4+ rows, where it
        # measured 2.4x faster at 8 rows; fewer rows stay on the CUDA-core kernel (as fast at 64 heads,
        # faster for tensor-parallel head shards)
        flash = self.mla_flash and rows >= 4
        K.mla_decode(self.q_lat[:rows], self.q_pe[:rows], kv.latent[l], kv.block_tables, inp.row_seq[:rows],
                     inp.row_ctx[:rows], self.scale, 0 if flash else self.num_splits(rows),
                     self.o_lat[:rows], self.status, ops.PDL)
        if wide:
            # value up-projection of every head as one batched bf16 GEMM, straight to the bf16 rows
            # of the O GEMM (no int8 round trip)
            nh, vd = cfg.n_heads, cfg.v_head_dim
            o = torch.bmm(self.o_lat[:rows].transpose(0, 1).to(torch.bfloat16), L.w_uv.transpose(1, 2))
            self.attb[:rows].view(rows, nh, vd).copy_(o.transpose(0, 1))
            self.wide.linear(L.idx["o"], self.attb[:rows], resid if resid is not None else self.x[:rows],
                             residual=True)
            return
        for c0 in range(0, rows, 8):
            c1 = min(rows, c0 + 8)
            K.mla_out(self.o_lat[c0:c1], L.w_uv, self.attq.q[c0:c1], self.attq.d[c0:c1], self.attq.s[c0:c1], ops.PDL)
        if self.tp is not None:
            mixed_gemv_push(t, L.idx["o"], self.attq.view(rows), self.tp, 2 * l)
        else:
            mixed_gemv(t, L.idx["o"], self.attq.view(rows), self.x[:rows], residual=True)

    def _ffn(self, L, rows, site: int = -1, resid: Optional[torch.Tensor] = None):
        """FFN / MoE of one layer; under tensor parallelism (``site`` >= 0) the result is pushed to
        every rank's receive region of ``site`` instead of added to the residual."""
        cfg, t, tp = self.cfg, self.w.table, self.tp
        xa = self.xa.view(rows)
        if L.dense and self._wide(rows) and cfg.ffn % 64 == 0:
            ops.rmsnorm(self.x[:rows], L.ffn_norm, cfg.eps, yb=self.xb[:rows])
            self.wide.swiglu(L.idx["g"], L.idx["u"], self.xb[:rows], self.hb[:rows, :cfg.ffn])
            self.wide.linear(L.idx["d"], self.hb[:rows, :cfg.ffn], resid if resid is not None else self.x[:rows],
                             residual=True)
            return
        if L.dense:
            h = self.h.view(rows)
            mixed_gemv_swiglu(t, L.idx["g"], L.idx["u"], xa, h)
            if tp is not None:
                mixed_gemv_push(t, L.idx["d"], h, tp, site)
            else:
                mixed_gemv(t, L.idx["d"], h, self.x[:rows], residual=True)
            return
        E, k, H, F = cfg.n_experts, cfg.top_k, cfg.hidden, cfg.expert_ffn
        ne = self.w.e_count or E  # routed experts in this rank's table
        e_lo = self.w.e_lo
        if rows > 8 and F % 128 == 0 and H % 128 == 0:
            self._ffn_wide(L, rows, resid if resid is not None else self.x[:rows])
            return
        fold = self.fold_shared and L.shared_here and L.idx.get("sg") == L.idx["eg"] + ne and \
            L.idx.get("su") == L.idx["eu"] + ne and L.idx.get("sd") == L.idx["ed"] + ne
        if tp is not None and L.shared_here and not fold:
            raise NotImplementedError("expert parallel: the shared expert must have the routed experts' shape")
        K = kernels()
        fused = self.fused_route and rows <= 8
        if fused:
            # one launch: router GEMV, top-k, sort by expert, active list (this rank's experts only
            # under expert parallelism); experts read token rows
            ops.moe_route(L.router, xa, k, self.scoring, L.router_bias, cfg.n_groups, cfg.topk_groups, cfg.norm_topk,
                          cfg.routed_scale, self.rlog[:rows], self.ids[:rows], self.rw[:rows], self.counts,
                          self.offsets, self.sorted, self.active, self.n_active, fold, self.route_counter,
                          e_lo=e_lo, e_hi=e_lo + ne if self.w.e_count else 0)
            gin = xa
        else:
            if self.w.e_count:
                raise NotImplementedError("expert parallel needs the fused routing kernel")
            ops.router_logits(L.router, xa, self.rlog[:rows])
            ops.moe_topk(self.rlog[:rows], L.router_bias, k, self.scoring, cfg.n_groups, cfg.topk_groups, cfg.norm_topk,
                         cfg.routed_scale, self.ids[:rows], self.rw[:rows])
            ops.moe_align(self.ids[:rows], E, xa, self.counts, self.offsets, self.sorted, self.gx, shared=fold)
            ops.launches.add()
            K.moe_active(self.counts, self.active, self.n_active, ops.PDL)
            gin = self.gx
        ops.launches.add(2)
        na = min(ne, rows * k) + (1 if fold else 0)
        ep = dict(e_lo=e_lo, e_count=self.w.e_count)
        K.moe_mixed_gemv(0, t.descs, L.idx["eg"], L.idx["eu"], F, H, k, self.counts, self.offsets, self.sorted,
                         self.active, self.n_active, na, gin.q, gin.d, gin.s, self.hx.q, self.hx.d,
                         self.hx.s, None, None, ops.PDL, rows * k, fused, **ep)
        if tp is not None:
            # expert-parallel combine: per-token sum over this rank's experts, pushed to every rank
            K.moe_mixed_gemv(2, t.descs, L.idx["ed"], L.idx["ed"], H, F, k, self.counts, self.offsets, self.sorted,
                             self.active, self.n_active, na, self.hx.q, self.hx.d, self.hx.s, None, None, None,
                             None, self.rw[:rows].reshape(-1), ops.PDL, rows * k, T=rows,
                             push_table=tp.push_recv[site], push_epoch=tp.epoch, **ep)
            return
        K.moe_mixed_gemv(1, t.descs, L.idx["ed"], L.idx["ed"], H, F, k, self.counts, self.offsets, self.sorted,
                         self.active, self.n_active, na, self.hx.q, self.hx.d, self.hx.s, None, None, None,
                         self.x[:rows], self.rw[:rows].reshape(-1), ops.PDL, rows * k, **ep)
        if not fold and "sg" in L.idx:
            hs = self.hs.view(rows)
            mixed_gemv_swiglu(t, L.idx["sg"], L.idx["su"], xa, hs)
            mixed_gemv(t, L.idx["sd"], hs, self.x[:rows], residual=True)

    def _ffn_wide(self, L, rows, out: torch.Tensor):
        """Routed experts of a prefill forward on the tensor cores (ops/prefill.py): routing over
        the q8 rows, experts as two grouped GEMMs over the bf16 normed rows, deterministic
        combine; the shared expert folded in as one more group when it has the experts' width."""
        from ..ops.prefill import MoePrefill
        cfg, xa = self.cfg, self.xa.view(rows)
        E, k = cfg.n_experts, cfg.top_k
        if self.prefill is None:
            self.prefill = MoePrefill(self.w.table, self.dev, E, cfg.expert_ffn, cfg.hidden,
                                      self.max_rows * (k + 1), self.status)
        ops.rmsnorm(self.x[:rows], L.ffn_norm, cfg.eps, yb=self.xb[:rows])
        fold = "sg" in L.idx and cfg.shared_ffn == cfg.expert_ffn
        ops.router_logits(L.router, xa, self.rlog[:rows])
        ops.moe_topk(self.rlog[:rows], L.router_bias, k, self.scoring, cfg.n_groups, cfg.topk_groups, cfg.norm_topk,
                     cfg.routed_scale, self.ids[:rows], self.rw[:rows])
        ops.moe_align(self.ids[:rows], E, xa, self.counts, self.offsets, self.sorted, None, shared=fold)
        # under expert parallelism this rank's experts only (the shared expert where it lives)
        self.prefill.run(L.idx, rows, k, self.xb[:rows], out, self.counts, self.offsets, self.sorted,
                         self.rw[:rows], fold, pdl=ops.PDL, e_lo=self.w.e_lo, e_count=self.w.e_count,
                         ids=self.ids[:rows])
        if not fold and "sg" in L.idx:
            self.prefill.dense_shared(L.idx, cfg.shared_ffn, rows, self.xb, out, pdl=ops.PDL)

    def forward(self, rows: int, sample: str = "greedy", advance: bool = False, n_logits: int = 0):
        """``n_logits`` (engine): > 0 moves the logits / greedy ids of ``logit_rows[:n_logits]`` to
        the first rows (all rows are computed; at most 8)."""
        if self.tp is not None and rows > 8:
            self._forward_tp_wide(rows, sample, advance, n_logits)
        elif self.tp is not None:
            self._forward_tp(rows, sample, advance)
            compact_logit_rows(self, n_logits)
        else:
            self._forward_local(rows, sample, advance, n_logits)

    def _forward_tp_wide(self, rows: int, sample: str, advance: bool, n_logits: int):
        """Tensor / expert-parallel prefill forward of more than 8 rows: this rank's heads, dense
        FFN slice and experts as tensor-core GEMMs into a zeroed partial, summed over the ranks by
        an NCCL all-reduce after the attention and after the FFN (the push sites hold 8 rows); the
        LM head runs on the sampled rows only (vocabulary slices, keys reduced as in decode)."""
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
            self._attention(l, L, rows, resid=p)
            dist.all_reduce(p, group=tp.group)
            x.add_(p)
            ops.rmsnorm_q8(x, L.ffn_norm, cfg.eps, xa)
            p.zero_()
            self._ffn(L, rows, resid=p)
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

    def _forward_local(self, rows: int, sample: str = "greedy", advance: bool = False, n_logits: int = 0):
        cfg, w, inp = self.cfg, self.w, self.inp
        nl = n_logits or rows
        if nl > self.max_logit_rows:
            raise ValueError(f"forward: logits for {nl} rows requested, at most {self.max_logit_rows}")
        ops.embed(w.embed, inp.ids[:rows], self.x[:rows])
        for l, L in enumerate(w.layers):
            ops.rmsnorm_q8(self.x[:rows], L.attn_norm, cfg.eps, self.xa.view(rows))
            self._attention(l, L, rows)
            ops.rmsnorm_q8(self.x[:rows], L.ffn_norm, cfg.eps, self.xa.view(rows))
            self._ffn(L, rows)
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

    def _forward_tp(self, rows: int, sample: str, advance: bool):
        """Tensor/expert-parallel decode forward: two push all-reduce sites per layer (attention
        output, FFN / expert combine), each consumed by the next RMSNorm on every rank."""
        cfg, w, inp, tp = self.cfg, self.w, self.inp, self.tp
        if rows > 8:
            raise RuntimeError("tensor-parallel decode takes at most 8 rows")
        ops.tp_begin(tp)
        xa_res, xb_res = self.x[:rows], self.x2[:rows]
        ops.embed(w.embed, inp.ids[:rows], xa_res)
        ops.rmsnorm_q8(xa_res, w.layers[0].attn_norm, cfg.eps, self.xa.view(rows))
        for l, L in enumerate(w.layers):
            self._attention(l, L, rows)
            ops.tp_allreduce_rmsnorm_q8(tp, 2 * l, xa_res, xb_res, L.ffn_norm, cfg.eps, self.xa.view(rows))
            self._ffn(L, rows, site=2 * l + 1)
            nxt = w.layers[l + 1].attn_norm if l + 1 < len(w.layers) else w.out_norm
            ops.tp_allreduce_rmsnorm_q8(tp, 2 * l + 1, xb_res, xa_res, nxt, cfg.eps, self.xa.view(rows))
        # the last all-reduce left norm(x) in self.xa; this rank's vocabulary slice of the LM head
        head = w.table.weights[w.lm_head]
        if sample == "greedy":
            mixed_gemv(w.table, w.lm_head, self.xa.view(rows), self.logits[:rows],
                       argmax_slots=self.argmax_slots[:rows], argmax_offset=tp.rank * head.N)
            ops.tp_argmax(tp, self.argmax_slots, rows, self.next_ids)
        elif sample == "none":
            mixed_gemv(w.table, w.lm_head, self.xa.view(rows), self.logits[:rows])
        else:  # vocabulary-parallel logits, gathered; every rank draws the same token
            mixed_gemv(w.table, w.lm_head, self.xa.view(rows), self.logits[:rows])
            full = self.gathered_logits(rows)
            ops.sample(full, self.temperature[:rows], self.top_k[:rows], self.top_p[:rows], self.rep_penalty[:rows],
                       None, self.uniforms[:rows], self.next_ids[:rows])
        if advance:
            ops.advance(inp.ids, self.next_ids, inp.positions, inp.row_ctx, rows)

    def gathered_logits(self, nl: int) -> torch.Tensor:
        """Logits of the first ``nl`` rows over the whole vocabulary (under tensor parallelism the
        ranks' vocabulary slices gathered; a collective every rank calls for the same rows)."""
        if self.tp is None:
            return self.logits[:nl]
        from ..parallel.tp import gather_vocab_logits
        if getattr(self, "_tp_full", None) is None:
            head = self.w.table.weights[self.w.lm_head]
            self._tp_full = torch.zeros(self.logits.shape[0], head.N * self.tp.world, device=self.dev)
        return gather_vocab_logits(self.tp, self.logits[:nl], self._tp_full)

    def forward_tokens(self, tokens, seq_id: int = 0, start_pos: int = 0) -> torch.Tensor:
        """Teacher-forced forward of one sequence in chunks of up to 8 rows; fp32 logits [n, vocab]."""
        kv = self.kv
        n = len(tokens)
        if not kv.bm.reserve(seq_id, start_pos + n):
            raise RuntimeError("latent cache exhausted")
        kv.sync_tables([seq_id])
        r = kv.row(seq_id)
        out = torch.empty(n, self.cfg.vocab, device=self.dev)
        step = min(self.max_rows, self.max_logit_rows)
        for c0 in range(0, n, step):
            c1 = min(n, c0 + step)
            pos = list(range(start_pos + c0, start_pos + c1))
            self.inp.upload(tokens[c0:c1], pos, [0] * (c1 - c0), [r] * (c1 - c0), [p + 1 for p in pos])
            self.forward(c1 - c0, "greedy")
            out[c0:c1] = self.logits[: c1 - c0]
        return out

    def graph_forward(self, rows: int, sample: str = "greedy", advance: bool = False):
        key = (rows, sample, advance)
        g = self._graphs.get(key)
        if g is None:
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            with torch.cuda.stream(s):
                self.forward(rows, "none")
            torch.cuda.current_stream(self.dev).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            n0 = ops.launches.n
            with torch.cuda.graph(g):
                self.forward(rows, sample, advance)
            self.launches_per_graph = ops.launches.n - n0
            self._graphs[key] = g
        g.replay()


def engine_buffers(model, R: int):
    """Per-row sampling inputs and the logit-row list the engine fills (as LlamaModel)."""
    dev = model.dev
    model.logit_rows = torch.zeros(R, dtype=torch.int32, device=dev)
    model.temperature = torch.zeros(R, device=dev)
    model.top_k = torch.zeros(R, dtype=torch.int32, device=dev)
    model.top_p = torch.ones(R, device=dev)
    model.rep_penalty = torch.ones(R, device=dev)
    model.uniforms = torch.zeros(R, device=dev)


def compact_logit_rows(model, n_logits: int):
    if n_logits > 0:
        idx = model.logit_rows[:n_logits].long()
        model.logits[:n_logits] = model.logits.index_select(0, idx)
        model.next_ids[:n_logits] = model.next_ids.index_select(0, idx)


class LatentCache:
    """Paged latent cache: ``latent[l]`` [num_blocks, block_size, 576] bf16 per layer, with the
    C++ block manager and device block tables of the regular paged KV cache."""

    def __init__(self, layers: int, num_blocks: int, block_size: int, max_seqs: int, max_blocks: int, device):
        from ..engine.kv_cache import PagedKVCache
        self._kv = PagedKVCache(1, 1, 64, num_blocks, block_size, max_seqs, max_blocks, device)
        self.latent = [torch.zeros(num_blocks, block_size, LAT + ROPE, dtype=torch.bfloat16, device=device)
                       for _ in range(layers)]
        self.block_size = block_size
        self.bm = self._kv.bm
        self.block_tables = self._kv.block_tables

    def sync_tables(self, ids):
        self._kv.sync_tables(ids)

    def row(self, seq_id):
        return self._kv.row(seq_id)

    def drop(self, seq_id):
        self._kv.drop(seq_id)


# ---- fp32 PyTorch reference (test oracle) -----------------------------------------------------
class TorchRefDeepSeek:
    """Token-serial fp32 restatement with the un-absorbed MLA (keys and values reconstructed from
    the latent per head, as in the reference CPU oracle) and the device's activation rounding."""

    def __init__(self, cfg: ModelConfig, w: DSWeights, act_q8: bool = True):
        from .deepseek_gguf import yarn_attention_scale
        self.cfg, self.w, self.act_q8 = cfg, w, act_q8
        self.scale = yarn_attention_scale(cfg)
        self.W = [mw.dequantize() for mw in w.table.weights]
        self.E = w.embed.dequantize()
        self.cache = {l: [] for l in range(cfg.layers)}

    def _q(self, v):
        if not self.act_q8:
            return v
        b = v.reshape(-1, 32)
        d = b.abs().amax(1, keepdim=True) / 127.0
        q = torch.where(d > 0, torch.round(b / torch.where(d > 0, d, torch.ones_like(d))), torch.zeros_like(b))
        return (q * d).reshape(v.shape)

    @staticmethod
    def _rms(x, w, eps):
        return x * torch.rsqrt((x * x).mean() + eps) * w

    def _rope(self, x, pos):
        from .deepseek_gguf import yarn_freq_factors
        inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, ROPE, 2, device=x.device, dtype=torch.float64) / ROPE))
        ff = yarn_freq_factors(self.cfg)
        if ff is not None:
            inv = inv / ff.to(inv.device)
        ang = (pos * inv).float()
        c, s = torch.cos(ang), torch.sin(ang)
        a, b = x[..., :ROPE // 2], x[..., ROPE // 2:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    def _route(self, L, h):
        cfg = self.cfg
        logits = L.router @ h
        if cfg.router == "sigmoid_bias":
            s = torch.sigmoid(logits)
            choice = s + L.router_bias if L.router_bias is not None else s
        else:
            s = torch.softmax(logits.double(), 0).float()
            choice = s
        E, ng = cfg.n_experts, cfg.n_groups
        gs = choice.view(ng, E // ng).topk(2, dim=1).values.sum(1)
        keep = torch.zeros(ng, dtype=torch.bool, device=h.device)
        keep[gs.topk(cfg.topk_groups).indices] = True
        masked = torch.where(keep.repeat_interleave(E // ng), choice, torch.full_like(choice, -float("inf")))
        idx = masked.topk(cfg.top_k).indices
        wts = s[idx]
        if cfg.norm_topk:
            wts = wts / wts.sum()
        return idx.tolist(), wts * cfg.routed_scale

    def step(self, token: int, pos: int) -> torch.Tensor:
        cfg, w, W = self.cfg, self.w, self.W
        nh, nope, rd, vd = cfg.n_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
        x = self.E[token].clone()
        for l, L in enumerate(w.layers):
            h = self._q(self._rms(x, L.attn_norm, cfg.eps))
            if "q" in L.idx:
                q = (W[L.idx["q"]] @ h).view(nh, nope + rd)
            else:
                qa = W[L.idx["qa"]] @ h
                q = (W[L.idx["qb"]] @ self._q(self._rms(qa, L.q_a_norm, cfg.eps))).view(nh, nope + rd)
            kva = W[L.idx["kva"]] @ h
            c = self._rms(kva[:LAT], L.kv_a_norm, cfg.eps).bfloat16().float()
            kpe = self._rope(kva[LAT:], pos).bfloat16().float()
            self.cache[l].append((c, kpe))
            C = torch.stack([a for a, _ in self.cache[l]])      # [T, 512]
            KP = torch.stack([b for _, b in self.cache[l]])     # [T, 64]
            o = torch.empty(nh, vd, device=x.device)
            uk, uv = L.w_uk.float(), L.w_uv.float()
            for i in range(nh):
                k_nope = C @ uk[i].t()                          # [T, nope]
                v = C @ uv[i].t()                               # [T, vd]
                qpe = self._rope(q[i, nope:], pos)
                sc = (k_nope @ q[i, :nope] + KP @ qpe) * self.scale
                o[i] = torch.softmax(sc, 0) @ v
            x = x + W[L.idx["o"]] @ self._q(o.reshape(-1))
            h = self._q(self._rms(x, L.ffn_norm, cfg.eps))
            if L.dense:
                gt, up = W[L.idx["g"]] @ h, W[L.idx["u"]] @ h
                x = x + W[L.idx["d"]] @ self._q(gt / (1 + torch.exp(-gt)) * up)
            else:
                idx, wts = self._route(L, h)
                for e, wt in zip(idx, wts):
                    gt, up = W[L.idx["eg"] + e] @ h, W[L.idx["eu"] + e] @ h
                    x = x + wt * (W[L.idx["ed"] + e] @ self._q(gt / (1 + torch.exp(-gt)) * up))
                if "sg" in L.idx:
                    gt, up = W[L.idx["sg"]] @ h, W[L.idx["su"]] @ h
                    x = x + W[L.idx["sd"]] @ self._q(gt / (1 + torch.exp(-gt)) * up)
        h = self._q(self._rms(x, w.out_norm, cfg.eps))
        return W[w.lm_head] @ h
