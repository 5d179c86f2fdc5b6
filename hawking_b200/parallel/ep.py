"""Expert parallelism (with tensor-parallel attention) for the DeepSeek-style MLA + MoE decoder and the
Qwen3-Next hybrid.

Plan for rank r of N GPUs of one node:

* attention: the query up-projection q_b, the absorbed W_UK / W_UV and the output projection are
  split by head (n_heads / N heads per rank); q_a / kv_a and the latent cache are replicated, so
  every rank appends the same latent rows and attends over them with its own heads;
* dense FFN layers: gate / up split by FFN row, down by FFN column (row-parallel);
* routed experts: expert parallel, rank r owns experts [r E / N, (r + 1) E / N) whole; the router
  is replicated (every rank computes the same top-k from the same replicated hidden state, so no
  token is dispatched: each rank reads its pairs' rows locally);
* shared expert: whole, on rank l mod N for layer l (folded into that rank's routed launches);
* LM head: split by vocabulary row, greedy reduced over per-rank keys.

The combine of the routed experts is the all-reduce of the layer's FFN output: the expert down
projection's epilogue pushes each token's sum over this rank's experts into every rank's receive
region (``moe_mixed_combine_push_kernel``), and the next RMSNorm adds the N contributions.

Parity: the reference runs one Apple GPU and has no model parallelism; the plan follows the
north-star requirement (TP attention + EP experts across the 8 GPUs of one box) and the reference's
DeepSeek layer math (crates/hawking-core/src/model/deepseek_v2.rs:2170 forward_token).
"""
from __future__ import annotations

from typing import List

import torch

from ..models.config import ModelConfig
from ..models.deepseek import LAT, ROPE, DSLayer, DSWeights
from ..ops import QWeight
from ..ops.mixed import MixedTable, MixedWeight


def local_deepseek_config(cfg: ModelConfig, world: int) -> ModelConfig:
    """This rank's shard of the config: heads and dense FFN width divided (experts stay global:
    routing scores all of them)."""
    if cfg.n_heads % world:
        raise ValueError(f"{cfg.n_heads} heads do not split over {world} ranks")
    if cfg.first_dense_layers and cfg.ffn % (128 * world):
        raise ValueError(f"dense FFN {cfg.ffn} must split into 128-column blocks over {world} ranks")
    if cfg.n_experts % world or cfg.vocab % world:
        raise ValueError(f"{cfg.n_experts} experts and vocab {cfg.vocab} must split over {world} ranks")
    if (cfg.n_heads // world) * cfg.v_head_dim % 128:
        raise ValueError("per-rank output-projection columns must be whole 128-column blocks")
    return cfg.with_(n_heads=cfg.n_heads // world, ffn=cfg.ffn // world)


def shard_deepseek_weights(w: DSWeights, cfg: ModelConfig, rank: int, world: int) -> DSWeights:
    """Rank ``rank``'s shard of full DSWeights (``cfg``: the full config)."""
    local_deepseek_config(cfg, world)
    W = w.table.weights
    nh, lnh = cfg.n_heads, cfg.n_heads // world
    qk, vd = cfg.qk_nope_dim + cfg.qk_rope_dim, cfg.v_head_dim
    E, ne = cfg.n_experts, cfg.n_experts // world
    e_lo = rank * ne
    lF = cfg.ffn // world
    ws: List[MixedWeight] = []

    def put(mw: MixedWeight) -> int:
        ws.append(mw)
        return len(ws) - 1

    layers = []
    for l, L in enumerate(w.layers):
        h0, h1 = rank * lnh, (rank + 1) * lnh
        nl = DSLayer(L.dense, L.attn_norm, L.q_a_norm, L.kv_a_norm, L.ffn_norm,
                     w_uk=L.w_uk[h0:h1].contiguous(), w_uv=L.w_uv[h0:h1].contiguous(),
                     router=L.router, router_bias=L.router_bias)
        for key in ("qakva", "qa", "kva"):  # replicated (q_a / kv_a, or kv_a alone without q low-rank)
            if key in L.idx:
                nl.idx[key] = put(W[L.idx[key]])
        for key in ("qb", "q"):  # query heads split
            if key in L.idx:
                nl.idx[key] = put(W[L.idx[key]].rows(h0 * qk, lnh * qk).contiguous())
        nl.idx["o"] = put(W[L.idx["o"]].cols(h0 * vd, h1 * vd))
        if L.dense:
            nl.idx["g"] = put(W[L.idx["g"]].rows(rank * lF, lF).contiguous())
            nl.idx["u"] = put(W[L.idx["u"]].rows(rank * lF, lF).contiguous())
            nl.idx["d"] = put(W[L.idx["d"]].cols(rank * lF, (rank + 1) * lF))
        else:
            nl.shared_here = (l % world) == rank
            for m, sm in (("eg", "sg"), ("eu", "su"), ("ed", "sd")):
                nl.idx[m] = len(ws)
                for e in range(e_lo, e_lo + ne):
                    put(W[L.idx[m] + e])
                if nl.shared_here and sm in L.idx:  # the shared expert follows this rank's routed experts
                    nl.idx[sm] = put(W[L.idx[sm]])
        layers.append(nl)
    V = cfg.vocab // world
    head = put(W[w.lm_head].rows(rank * V, V).contiguous())
    return DSWeights(MixedTable(ws), w.embed, w.out_norm, layers, head, e_lo=e_lo, e_count=ne)


def random_deepseek_weights_ep(cfg: ModelConfig, rank: int, world: int, device, seed: int = 0,
                               std: float = 0.02) -> DSWeights:
    """Random-init fp8 weights generated directly in rank ``rank``'s shard shapes (benchmarks:
    replicated tensors come from a generator every rank seeds alike, so they agree bitwise)."""
    lcfg = local_deepseek_config(cfg, world)
    gs = torch.Generator(device=device)
    gs.manual_seed(seed)                         # replicated tensors
    gl = torch.Generator(device=device)
    gl.manual_seed(seed * 1009 + 1 + rank)       # this rank's shards
    H, lnh = cfg.hidden, lcfg.n_heads
    nope, rd, vd = cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
    E, ne = cfg.n_experts, cfg.n_experts // world
    ws: List[MixedWeight] = []

    def put(mw: MixedWeight) -> int:
        ws.append(mw)
        return len(ws) - 1

    def ones(n):
        return torch.ones(n, device=device)

    layers = []
    for l in range(cfg.layers):
        dense = l < cfg.first_dense_layers
        L = DSLayer(dense, ones(H), ones(cfg.q_lora_rank), ones(LAT), ones(H),
                    w_uk=(torch.randn(lnh, nope, LAT, generator=gl, device=device) * std).bfloat16(),
                    w_uv=(torch.randn(lnh, vd, LAT, generator=gl, device=device) * std).bfloat16())
        qakva = MixedWeight.random_fp8(cfg.q_lora_rank + LAT + ROPE, H, std, gs, device)
        L.idx["qakva"] = put(qakva)
        L.idx["qa"] = put(qakva.rows(0, cfg.q_lora_rank))
        L.idx["kva"] = put(qakva.rows(cfg.q_lora_rank, LAT + ROPE))
        L.idx["qb"] = put(MixedWeight.random_fp8(lnh * (nope + rd), cfg.q_lora_rank, std, gl, device))
        L.idx["o"] = put(MixedWeight.random_fp8(H, lnh * vd, std, gl, device))
        if dense:
            L.idx["g"] = put(MixedWeight.random_fp8(lcfg.ffn, H, std, gl, device))
            L.idx["u"] = put(MixedWeight.random_fp8(lcfg.ffn, H, std, gl, device))
            L.idx["d"] = put(MixedWeight.random_fp8(H, lcfg.ffn, std, gl, device))
        else:
            F = cfg.expert_ffn
            L.router = torch.randn(E, H, generator=gs, device=device) * std
            L.router_bias = torch.randn(E, generator=gs, device=device) * 0.01
            L.shared_here = (l % world) == rank
            for m, sm, (n, k) in (("eg", "sg", (F, H)), ("eu", "su", (F, H)), ("ed", "sd", (H, F))):
                stacked = MixedWeight.random_fp8(ne * n, k, std, gl, device)
                L.idx[m] = len(ws)
                for e in range(ne):
                    put(stacked.rows(e * n, n))
                if L.shared_here:
                    L.idx[sm] = put(MixedWeight.random_fp8(n, k, std, gl, device))
        layers.append(L)
    head = put(MixedWeight.random_fp8(cfg.vocab // world, H, std, gl, device))
    emb = QWeight.quantize(torch.randn(cfg.vocab, H, generator=gs, device=device) * std, 1)
    torch.cuda.synchronize(device)
    return DSWeights(MixedTable(ws), emb, ones(H), layers, head, e_lo=rank * ne, e_count=ne)


# ---- Qwen3-Next hybrid: tensor-parallel mixers, expert-parallel MoE --------------------------------
# Rank r of N: full-attention query / gate heads split (n_heads / N each); key / value heads split
# when N <= n_kv_heads, otherwise each rank computes the one KV head its query heads read (KV
# replicated across that head's ranks); DeltaNet key heads split (with their value heads, the
# per-head q | k | v | z rows of the fused projection, the b | a rows, the conv channels and the
# decay parameters); output projections row-parallel (column slices) pushed into the all-reduce;
# routed experts whole on their rank, the sigmoid-gated shared expert on rank l mod N (folded into
# that rank's expert launches with the gate as its pair weight); LM head split by vocabulary row.

def local_qwen_next_config(cfg: ModelConfig, world: int) -> ModelConfig:
    nh, nkv, kh = cfg.n_heads, cfg.n_kv_heads, cfg.linear_k_heads
    if nh % world or kh % world or cfg.n_experts % world or cfg.vocab % world:
        raise ValueError(f"qwen3next over {world} ranks: heads {nh}, key heads {kh}, experts {cfg.n_experts} and "
                         f"vocab {cfg.vocab} must divide")
    if cfg.shared_ffn != cfg.expert_ffn:
        raise ValueError("qwen3next expert parallelism folds the shared expert into the expert launches: "
                         "shared FFN width must equal the experts'")
    lnh = nh // world
    if world <= nkv:
        if nkv % world:
            raise ValueError(f"{nkv} KV heads do not split over {world} ranks")
        lnkv = nkv // world
    else:
        if (nh // nkv) % lnh:
            raise ValueError("a rank's query heads must read one KV head")
        lnkv = 1
    lkh = kh // world
    return cfg.with_(n_heads=lnh, n_kv_heads=lnkv, linear_k_heads=lkh,
                     linear_v_heads=cfg.linear_v_heads // world)


def _kv_head0(cfg: ModelConfig, rank: int, world: int) -> int:
    lnh = cfg.n_heads // world
    if world <= cfg.n_kv_heads:
        return rank * (cfg.n_kv_heads // world)
    return rank * lnh // (cfg.n_heads // cfg.n_kv_heads)


def shard_qwen_next_weights(w, cfg: ModelConfig, rank: int, world: int):
    """Rank ``rank``'s shard of full QNWeights (``cfg``: the full config)."""
    from ..models.qwen_next import QNLayer, QNWeights, dims
    lc = local_qwen_next_config(cfg, world)
    W = w.table.weights
    hd, lnh, lnkv = cfg.head_dim, lc.n_heads, lc.n_kv_heads
    h0, kv0 = rank * lnh, _kv_head0(cfg, rank, world)
    dm = dims(cfg)
    dk, rv, r = dm["dk"], dm["r"] * dm["dv"], dm["r"]
    grp = 2 * dk + 2 * rv
    lkh = lc.linear_k_heads
    k0 = rank * lkh
    KE = cfg.linear_k_heads * dk
    E, ne = cfg.n_experts, cfg.n_experts // world
    e_lo = rank * ne
    ws: List[MixedWeight] = []

    def put(mw: MixedWeight) -> int:
        ws.append(mw)
        return len(ws) - 1

    layers = []
    for l, L in enumerate(w.layers):
        nl = QNLayer(L.full, L.attn_norm, L.post_norm, q_norm=L.q_norm, k_norm=L.k_norm, ssm_norm=L.ssm_norm,
                     router=L.router, shared_gate=L.shared_gate)
        if L.full:
            nl.idx["q"] = put(W[L.idx["q"]].rows(h0 * hd, lnh * hd).contiguous())
            nl.idx["g"] = put(W[L.idx["g"]].rows(h0 * hd, lnh * hd).contiguous())
            nl.idx["k"] = put(W[L.idx["k"]].rows(kv0 * hd, lnkv * hd).contiguous())
            nl.idx["v"] = put(W[L.idx["v"]].rows(kv0 * hd, lnkv * hd).contiguous())
            nl.idx["o"] = put(W[L.idx["o"]].cols(h0 * hd, (h0 + lnh) * hd))
        else:
            nl.idx["qkvz"] = put(W[L.idx["qkvz"]].rows(k0 * grp, lkh * grp).contiguous())
            nl.idx["ba"] = put(W[L.idx["ba"]].rows(k0 * 2 * r, lkh * 2 * r).contiguous())
            nl.idx["out"] = put(W[L.idx["out"]].cols(k0 * rv, (k0 + lkh) * rv))
            cw = L.conv_w
            nl.conv_w = torch.cat([cw[k0 * dk:(k0 + lkh) * dk], cw[KE + k0 * dk:KE + (k0 + lkh) * dk],
                                   cw[2 * KE + k0 * rv:2 * KE + (k0 + lkh) * rv]]).contiguous()
            nl.a_log = L.a_log[k0 * r:(k0 + lkh) * r].contiguous()
            nl.dt_bias = L.dt_bias[k0 * r:(k0 + lkh) * r].contiguous()
        nl.shared_here = (l % world) == rank
        for m, sm in (("eg", "sg"), ("eu", "su"), ("ed", "sd")):
            nl.idx[m] = len(ws)
            for e in range(e_lo, e_lo + ne):
                put(W[L.idx[m] + e])
            if nl.shared_here:  # the shared expert follows this rank's routed experts
                nl.idx[sm] = put(W[L.idx[sm]])
        layers.append(nl)
    V = cfg.vocab // world
    head = put(W[w.lm_head].rows(rank * V, V).contiguous())
    return QNWeights(MixedTable(ws), w.embed, w.out_norm, layers, head, e_lo=e_lo, e_count=ne)
