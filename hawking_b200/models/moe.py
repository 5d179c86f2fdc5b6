"""Mixture-of-experts FFN on the device (Mixtral, Qwen MoE / Qwen3-Next, DeepSeek-V3 routing).

Per step: router logits (fp32 router weights over the q8-normalised input) -> top-k (softmax, or
sigmoid + learned bias with group-limited selection) -> counting sort of the (token, slot) pairs by
expert with the activations gathered in that order -> grouped gate/up GEMV with SwiGLU (each
active expert's rows stream once per chunk of <= 8 pairs) -> grouped down GEMV accumulating
route_weight * y into the fp32 residual -> optional shared expert (sigmoid-gated for Qwen).

Parity: crates/hawking-core/src/model/mixtral.rs:894 (forward_token: 8 experts, top-2),
crates/hawking-core/src/moe.rs:24-117, crates/hawking-core/shaders/moe.metal (moe_topk_gate,
moe_batched_gemm_*_indexed_gu, moe_route_accumulate), qwen80_shared_expert_wave (sigmoid-gated
shared expert), deepseek routing (sigmoid + learned bias, noaux_tc).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .. import ops
from .._ext import kernels
from ..formats.ggml import type_id
from ..ops import Q8Act, QWeight, cat_rows
from .config import ModelConfig


# forwards of more than 8 rows on one GPU run the experts as grouped tensor-core GEMMs over bf16
# copies of their weights (0: the GEMV kernels)
WIDE_MOE = __import__("os").environ.get("HK_MOE_PREFILL", "1") == "1"


@dataclass
class MoEFFN:
    cfg: ModelConfig
    router_w: torch.Tensor             # fp32 [E, H]
    w_gate: QWeight                    # [E * Fe, H]
    w_up: QWeight                      # [E * Fe, H]
    w_down: QWeight                    # [E * H, Fe]
    router_bias: Optional[torch.Tensor] = None   # [E] selection bias (sigmoid routing)
    sh_gate: Optional[QWeight] = None  # shared expert views of one fused [gate | up] weight
    sh_up: Optional[QWeight] = None
    sh_gu: Optional[QWeight] = None
    sh_down: Optional[QWeight] = None
    sh_gate_w: Optional[torch.Tensor] = None     # fp32 [1, H] sigmoid gate of the shared expert
    e_lo: int = 0                      # expert parallel: this rank stacks experts e_lo ..
    n_local: int = 0                   # .. e_lo + n_local - 1 (0: all of them)

    @property
    def nbytes(self) -> int:
        n = self.router_w.numel() * 4 + self.w_gate.nbytes + self.w_up.nbytes + self.w_down.nbytes
        if self.sh_gu is not None:
            n += self.sh_gu.nbytes + self.sh_down.nbytes
        return n

    # ---- construction ----
    @staticmethod
    def from_gguf(m, cfg: ModelConfig, l: int, device, qw, vec) -> "MoEFFN":
        p = f"blk.{l}."
        E, H = cfg.n_experts, cfg.hidden
        router = torch.from_numpy(m.dequantize(p + "ffn_gate_inp.weight").reshape(E, H).copy()).float().to(device)
        f = MoEFFN(cfg, router, qw(p + "ffn_gate_exps.weight"), qw(p + "ffn_up_exps.weight"),
                   qw(p + "ffn_down_exps.weight"))
        if m.has(p + "exp_probs_b.bias"):
            f.router_bias = vec(p + "exp_probs_b.bias")
        if m.has(p + "ffn_gate_shexp.weight"):
            g, u = qw(p + "ffn_gate_shexp.weight"), qw(p + "ffn_up_shexp.weight")
            f._set_shared(g, u, qw(p + "ffn_down_shexp.weight"))
            if m.has(p + "ffn_gate_inp_shexp.weight"):
                f.sh_gate_w = vec(p + "ffn_gate_inp_shexp.weight").reshape(1, H).contiguous()
        return f

    @staticmethod
    def random(cfg: ModelConfig, device, g: torch.Generator, std: float = 0.02) -> "MoEFFN":
        fmt = type_id(cfg.weight_type)
        E, H, Fe = cfg.n_experts, cfg.hidden, cfg.expert_ffn
        router = torch.randn(E, H, generator=g, device=device) * std
        f = MoEFFN(cfg, router, QWeight.random(fmt, E * Fe, H, std, g, device),
                   QWeight.random(fmt, E * Fe, H, std, g, device), QWeight.random(fmt, E * H, Fe, std, g, device))
        if cfg.router == "sigmoid_bias":
            f.router_bias = torch.zeros(E, device=device)
        if cfg.shared_ffn:
            Fs = cfg.shared_ffn
            f._set_shared(QWeight.random(fmt, Fs, H, std, g, device), QWeight.random(fmt, Fs, H, std, g, device),
                          QWeight.random(fmt, H, Fs, std, g, device))
            if cfg.shared_gate:
                f.sh_gate_w = torch.randn(1, H, generator=g, device=device) * std
        return f

    def _set_shared(self, g: QWeight, u: QWeight, d: QWeight):
        Fs = g.N
        if g.fmt == u.fmt:
            self.sh_gu = cat_rows([g, u])
            self.sh_gate, self.sh_up = self.sh_gu.rows(0, Fs), self.sh_gu.rows(Fs, Fs)
        else:
            self.sh_gate, self.sh_up = g, u
        self.sh_down = d

    def _wide(self, model, rows: int) -> bool:
        """This forward's experts run as grouped tensor-core GEMMs (prefill-sized, one GPU)."""
        from ..ops.prefill import GGUF_DEQUANT
        cfg = self.cfg
        return (WIDE_MOE and rows > 8 and getattr(model, "tp", None) is None and not self.n_local and
                cfg.expert_ffn % 128 == 0 and cfg.hidden % 128 == 0 and
                all(w.fmt in GGUF_DEQUANT for w in (self.w_gate, self.w_up, self.w_down)))

    # ---- buffers (per model, sized for max rows) ----
    def _buffers(self, model):
        key = "_moe_buffers"
        buf = getattr(model, key, None)
        cfg = self.cfg
        R, E, k, H = model.max_rows, cfg.n_experts, cfg.top_k, cfg.hidden
        Fe, Fs = cfg.expert_ffn, max(cfg.shared_ffn, 32)
        if buf is None:
            dev = model.dev
            buf = dict(
                logits=torch.zeros(R, E, device=dev), ids=torch.zeros(R, k, dtype=torch.int32, device=dev),
                weights=torch.zeros(R, k, device=dev), counts=torch.zeros(E, dtype=torch.int32, device=dev),
                offsets=torch.zeros(E, dtype=torch.int32, device=dev),
                sorted=torch.zeros(R * k, dtype=torch.int32, device=dev), gx=Q8Act(R * k, H, dev),
                h=Q8Act(R * k, Fe, dev), hs=Q8Act(R, Fs, dev), tmp=torch.zeros(R, H, device=dev),
                glog=torch.zeros(R, 1, device=dev))
            setattr(model, key, buf)
        return buf

    def forward_ep(self, model, rows: int, site: int):
        """Expert-parallel MoE for tensor-parallel decode: the router and top-k run on every rank
        (the normed hidden state in ``model.xa`` is replicated), this rank's experts run their
        pairs, and the down projection's epilogue pushes each token's sum over this rank's
        experts (plus this rank's slice of the shared expert) to every rank's receive region of
        ``site``; the next RMSNorm adds the ranks' contributions. No token is dispatched."""
        from .. import ops as O
        cfg, tp = self.cfg, model.tp
        b = self._buffers(model)
        E, k, H, Fe = cfg.n_experts, cfg.top_k, cfg.hidden, cfg.expert_ffn
        ne = self.n_local or E
        xa = model.xa.view(rows)
        O.router_logits(self.router_w, xa, b["logits"][:rows])
        scoring = 1 if cfg.router == "sigmoid_bias" else 0
        O.moe_topk(b["logits"][:rows], self.router_bias, k, scoring, cfg.n_groups if scoring else 1,
                   cfg.topk_groups if scoring else 1, cfg.norm_topk, cfg.routed_scale, b["ids"][:rows],
                   b["weights"][:rows])
        O.moe_align(b["ids"][:rows], E, xa, b["counts"], b["offsets"], b["sorted"], b["gx"])
        K = kernels()
        O.launches.add(2)
        K.moe_gemv(self.w_gate.fmt, 0, self.w_gate.planes, self.w_up.planes, Fe, self.w_gate.K, ne, k, b["counts"],
                   b["offsets"], b["sorted"], b["gx"].q, b["gx"].d, b["gx"].s, b["h"].q, b["h"].d, b["h"].s, None, None,
                   O.PDL, e_lo=self.e_lo)
        base = None
        if self.sh_down is not None:  # this rank's FFN slice of the shared expert, added by the push
            hs_v = model._q8_slice(b["hs"], 0, rows, self.sh_gate.N)
            O.gemv_swiglu(self.sh_gate, self.sh_up, xa, hs_v)
            base = b["tmp"][:rows]
            O.gemv(self.sh_down, hs_v, base)
            if self.sh_gate_w is not None:
                O.router_logits(self.sh_gate_w, xa, b["glog"][:rows])
                base.mul_(torch.sigmoid(b["glog"][:rows]))
        K.moe_gemv(self.w_down.fmt, 2, self.w_down.planes, [], H, self.w_down.K, ne, k, b["counts"], b["offsets"],
                   b["sorted"], b["h"].q, b["h"].d, b["h"].s, None, None, None, None, b["weights"][:rows].reshape(-1),
                   O.PDL, e_lo=self.e_lo, T=rows, push_table=tp.push_recv[site], push_epoch=tp.epoch, base=base)

    def shard(self, rank: int, world: int) -> "MoEFFN":
        """Rank ``rank``'s expert-parallel shard: experts split across ranks (whole), router
        replicated, the shared expert split by FFN row (gate / up rows, down columns)."""
        from ..parallel.tp import cols
        E, H, Fe = self.cfg.n_experts, self.cfg.hidden, self.cfg.expert_ffn
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        ne = E // world
        lo = rank * ne

        def own(w: QWeight, rows_per_expert: int) -> QWeight:
            v = w.rows(lo * rows_per_expert, ne * rows_per_expert)
            return QWeight(v.fmt, v.N, v.K, [p.contiguous() for p in v.planes])

        f = MoEFFN(self.cfg, self.router_w, own(self.w_gate, Fe), own(self.w_up, Fe), own(self.w_down, H),
                   router_bias=self.router_bias, sh_gate_w=self.sh_gate_w, e_lo=lo, n_local=ne)
        if self.sh_down is not None:
            Fs = self.sh_gate.N
            if Fs % (32 * world):
                raise ValueError(f"shared expert FFN {Fs} must split into 32-row blocks over {world} ranks")
            lF = Fs // world
            g, u = self.sh_gate.rows(rank * lF, lF), self.sh_up.rows(rank * lF, lF)
            f._set_shared(QWeight(g.fmt, g.N, g.K, [p.contiguous() for p in g.planes]),
                          QWeight(u.fmt, u.N, u.K, [p.contiguous() for p in u.planes]),
                          cols(self.sh_down, rank * lF, (rank + 1) * lF))
        return f

    @staticmethod
    def random_shard(cfg: ModelConfig, rank: int, world: int, device, g: torch.Generator, g_rep: torch.Generator,
                     std: float = 0.02) -> "MoEFFN":
        """Random-init weights generated directly in rank ``rank``'s expert-parallel shard shapes
        (``g_rep`` seeds the replicated router identically on every rank)."""
        fmt = type_id(cfg.weight_type)
        E, H, Fe = cfg.n_experts, cfg.hidden, cfg.expert_ffn
        ne = E // world
        router = torch.randn(E, H, generator=g_rep, device=device) * std
        f = MoEFFN(cfg, router, QWeight.random(fmt, ne * Fe, H, std, g, device),
                   QWeight.random(fmt, ne * Fe, H, std, g, device), QWeight.random(fmt, ne * H, Fe, std, g, device),
                   e_lo=rank * ne, n_local=ne)
        if cfg.router == "sigmoid_bias":
            f.router_bias = torch.zeros(E, device=device)
        if cfg.shared_ffn:
            lF = cfg.shared_ffn // world
            f._set_shared(QWeight.random(fmt, lF, H, std, g, device), QWeight.random(fmt, lF, H, std, g, device),
                          QWeight.random(fmt, H, lF, std, g, device))
            if cfg.shared_gate:
                f.sh_gate_w = torch.randn(1, H, generator=g_rep, device=device) * std
        return f

    def forward(self, model, rows: int):
        """x[:rows] += MoE(q8 input model.xa[:rows]) on the device."""
        cfg = self.cfg
        b = self._buffers(model)
        E, k, H, Fe = cfg.n_experts, cfg.top_k, cfg.hidden, cfg.expert_ffn
        xa = model.xa.view(rows)
        x = model.x[:rows]
        ops.router_logits(self.router_w, xa, b["logits"][:rows])
        scoring = 1 if cfg.router == "sigmoid_bias" else 0
        ops.moe_topk(b["logits"][:rows], self.router_bias, k, scoring, cfg.n_groups if scoring else 1,
                     cfg.topk_groups if scoring else 1, cfg.norm_topk, cfg.routed_scale, b["ids"][:rows],
                     b["weights"][:rows])
        if self._wide(model, rows):
            # prefill: every expert decoded once into a bf16 copy, the pairs sorted by expert, and
            # two grouped tensor-core GEMMs over them (ops/prefill.py)
            from ..ops.prefill import MoePrefill, q8_to_bf16
            ops.moe_align(b["ids"][:rows], E, xa, b["counts"], b["offsets"], b["sorted"], None)
            pf = getattr(model, "_moe_prefill", None)
            if pf is None:
                pf = model._moe_prefill = MoePrefill(None, model.dev, E, Fe, H, model.max_rows * (k + 1),
                                                     model.status)
                model._moe_xb = torch.zeros(model.max_rows, H, dtype=torch.bfloat16, device=model.dev)
            xb = model._moe_xb[:rows]
            q8_to_bf16(xa, xb)
            pf.run_gguf(self.w_gate, self.w_up, self.w_down, rows, k, xb, x, b["counts"], b["offsets"], b["sorted"],
                        b["weights"][:rows], pdl=ops.PDL)
        else:
            ops.moe_align(b["ids"][:rows], E, xa, b["counts"], b["offsets"], b["sorted"], b["gx"])
            ops.moe_gemv_swiglu(self.w_gate, self.w_up, Fe, E, k, b["counts"], b["offsets"], b["sorted"], b["gx"],
                                b["h"])
            ops.moe_gemv_down(self.w_down, H, E, k, b["counts"], b["offsets"], b["sorted"], b["h"], x,
                              b["weights"][:rows].reshape(-1))
        if self.sh_down is not None:
            hs = b["hs"].view(rows)
            hs_v = model._q8_slice(b["hs"], 0, rows, self.sh_gate.N)
            ops.gemv_swiglu(self.sh_gate, self.sh_up, xa, hs_v)
            if self.sh_gate_w is None:
                ops.gemv(self.sh_down, hs_v, x, residual=True)
            else:
                tmp = b["tmp"][:rows]
                ops.gemv(self.sh_down, hs_v, tmp)
                ops.router_logits(self.sh_gate_w, xa, b["glog"][:rows])
                x.add_(torch.sigmoid(b["glog"][:rows]) * tmp)
