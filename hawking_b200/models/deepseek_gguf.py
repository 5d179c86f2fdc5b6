"""DeepSeek-V2 / V3 (``deepseek2``) GGUF files: architecture config and weights for the MLA + MoE
engine (``models/deepseek.py``).

Config keys (``deepseek2.*``): block_count, embedding_length, attention.head_count,
attention.q_lora_rank (0: a plain ``attn_q`` projection, as in V2-Lite), attention.kv_lora_rank,
attention.key_length (nope + rope) / value_length, rope.dimension_count, feed_forward_length
(leading dense layers), expert_feed_forward_length, expert_count, expert_used_count,
expert_shared_count, leading_dense_block_count, expert_weights_scale, expert_weights_norm,
expert_gating_func (1 softmax, 2 sigmoid with the ``exp_probs_b`` selection bias),
expert_group_count / expert_group_used_count, rope.freq_base and the YaRN keys
rope.scaling.{type,factor,original_context_length,yarn_log_multiplier}.

Tensors: ``blk.{l}.attn_q_a`` / ``attn_q_a_norm`` / ``attn_q_b`` (or ``attn_q``),
``attn_kv_a_mqa`` ([kv_lora + rope, H]), ``attn_kv_a_norm``, ``attn_kv_b`` ([heads * (nope + v),
kv_lora]; split here into the absorbed W_UK / W_UV, bf16), ``attn_output``, ``ffn_norm``,
``ffn_{gate,up,down}`` (dense layers) or ``ffn_gate_inp``, ``exp_probs_b.bias``,
``ffn_{gate,up,down}_exps`` (stacked experts) and ``ffn_{gate,up,down}_shexp`` (the shared experts
as one wider FFN).

Projection weights become table entries of the mixed GEMV kernels (``MixedWeight.from_gguf``):
Q4_K, Q8_0 and Q4_0 keep the file's values bit for bit; other formats are re-encoded as 8-bit
group-32 codes. The file's RoPE rotates adjacent pairs of the 64 rope dims; the MLA kernels rotate
halves, so the rope rows of ``attn_kv_a_mqa`` and of every head of ``attn_q_b`` are permuted at
load (pair i = dims 2i, 2i+1 moves to i, 32 + i): q_pe . k_pe and the rotation are unchanged.

Parity: crates/hawking-core/src/model/deepseek_v2.rs:97-158 (DeepSeekConfig::from_gguf), :545-660
(per-layer tensor names, fused-expert 3-D tensors, shared experts as one FFN),
crates/hawking-core/src/model/mod.rs:152-155 (arch dispatch of ``deepseek2``).
"""
from __future__ import annotations

import math
from typing import List, Optional

import numpy as np
import torch

from ..formats.gguf import GgufModel
from ..ops import QWeight
from ..ops.mixed import MixedTable, MixedWeight
from .config import ModelConfig
from .deepseek import LAT, ROPE, DSLayer, DSWeights


def deepseek_config_from_gguf(m: GgufModel) -> ModelConfig:
    a = m.architecture
    if a != "deepseek2":
        raise ValueError(f"not a deepseek2 GGUF (architecture {a!r})")
    g = lambda k, d=None: m.get(f"{a}.{k}", d)  # noqa: E731
    H = int(g("embedding_length"))
    nh = int(g("attention.head_count"))
    rd = int(g("rope.dimension_count", g("attention.qk_rope_head_dim", 64)))
    kl = g("attention.key_length")
    nope = int(kl) - rd if kl is not None else int(g("attention.qk_nope_head_dim", 128))
    vd = int(g("attention.value_length", g("attention.v_head_dim", 128)))
    kv_lora = int(g("attention.kv_lora_rank", 512))
    if kv_lora != LAT or rd != ROPE:
        raise ValueError(f"deepseek2: the MLA kernels take a {LAT}-d latent and {ROPE} rope dims "
                         f"(file: {kv_lora}, {rd})")
    E = int(g("expert_count", 0) or 0)
    Fe = int(g("expert_feed_forward_length", 0) or 0)
    n_shared = int(g("expert_shared_count", 0) or 0)
    gating = int(g("expert_gating_func", 0) or 0)
    sigmoid = gating == 2 or (gating == 0 and m.has("blk.%d.exp_probs_b.bias" % int(g("leading_dense_block_count", 1))))
    vocab = int(g("vocab_size", m.tensors["token_embd.weight"].dims[1]))
    cfg = ModelConfig(
        arch="deepseek2", vocab=vocab, hidden=H, layers=int(g("block_count")), n_heads=nh,
        n_kv_heads=int(g("attention.head_count_kv", nh)), head_dim=nope + rd,
        ffn=int(g("feed_forward_length", 0) or 0), eps=float(g("attention.layer_norm_rms_epsilon", 1e-6)),
        rope_theta=float(g("rope.freq_base", 10000.0)), rope_style=1,
        n_experts=E, top_k=int(g("expert_used_count", 0) or 0), expert_ffn=Fe, n_shared_experts=n_shared,
        shared_ffn=n_shared * Fe, norm_topk=bool(g("expert_weights_norm", False)),
        router="sigmoid_bias" if sigmoid else "softmax", n_groups=int(g("expert_group_count", 1) or 1),
        topk_groups=int(g("expert_group_used_count", 1) or 1),
        routed_scale=float(g("expert_weights_scale", 1.0) or 1.0),
        first_dense_layers=int(g("leading_dense_block_count", 1)),
        q_lora_rank=int(g("attention.q_lora_rank", 0) or 0), kv_lora_rank=kv_lora, qk_nope_dim=nope,
        qk_rope_dim=rd, v_head_dim=vd, weight_type=m.tensors["blk.0.attn_output.weight"].type_name,
        max_ctx=int(g("context_length", 4096)))
    if str(g("rope.scaling.type", "")) == "yarn":
        cfg.rope_yarn_factor = float(g("rope.scaling.factor", 1.0))
        cfg.rope_yarn_orig_ctx = int(g("rope.scaling.original_context_length", cfg.max_ctx))
        cfg.rope_yarn_log_mul = float(g("rope.scaling.yarn_log_multiplier", 0.0))
    return cfg


def _rope_pairs_to_halves(n: int) -> torch.Tensor:
    """Row order that turns ``n`` adjacent-pair rope rows into halves (new i <- old perm[i])."""
    return torch.cat([torch.arange(0, n, 2), torch.arange(1, n, 2)])


def _permute_rows(w: MixedWeight, order: torch.Tensor) -> MixedWeight:
    idx = order.to(w.codes.device)
    return MixedWeight(w.kind, w.bits, w.group, w.N, w.K, w.codes.index_select(0, idx).contiguous(),
                       w.scales.index_select(0, idx).contiguous(), w.zero)


def q_row_order(nh: int, nope: int, rd: int) -> torch.Tensor:
    """Rows of a [heads * (nope + rope), K] query projection with each head's rope rows in halves."""
    per = nope + rd
    p = _rope_pairs_to_halves(rd)
    return torch.cat([torch.cat([torch.arange(h * per, h * per + nope), h * per + nope + p]) for h in range(nh)])


def kva_row_order(rd: int) -> torch.Tensor:
    return torch.cat([torch.arange(LAT), LAT + _rope_pairs_to_halves(rd)])


def load_deepseek_weights(m: GgufModel, cfg: ModelConfig, device) -> DSWeights:
    """Every tensor of the file once onto the device, mapped to the MLA + MoE engine's layout."""
    nh, nope, rd, vd, H = cfg.n_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.hidden
    ws: List[MixedWeight] = []

    def raw(name):
        return torch.from_numpy(np.ascontiguousarray(m.raw(name))).to(device, non_blocking=True)

    def mixed(name, order: Optional[torch.Tensor] = None) -> MixedWeight:
        t = m.tensors[name]
        K = t.dims[0]
        N = t.n_elements // K
        w = MixedWeight.from_gguf(raw(name), t.type, N, K, device)
        return _permute_rows(w, order) if order is not None else w

    def add(w: MixedWeight) -> int:
        ws.append(w)
        return len(ws) - 1

    def vec(name):
        return torch.from_numpy(m.dequantize(name).reshape(-1).copy()).float().to(device)

    layers = []
    for l in range(cfg.layers):
        p = f"blk.{l}."
        dense = not cfg.layer_is_moe(l)
        kvb = torch.from_numpy(m.dequantize(p + "attn_kv_b.weight").reshape(nh, nope + vd, LAT).copy())
        L = DSLayer(dense, vec(p + "attn_norm.weight"),
                    vec(p + "attn_q_a_norm.weight") if cfg.q_lora_rank else None,
                    vec(p + "attn_kv_a_norm.weight"), vec(p + "ffn_norm.weight"),
                    w_uk=kvb[:, :nope].contiguous().to(device).bfloat16(),
                    w_uv=kvb[:, nope:].contiguous().to(device).bfloat16())
        kva = mixed(p + "attn_kv_a_mqa.weight", kva_row_order(rd))
        qord = q_row_order(nh, nope, rd)
        if cfg.q_lora_rank:
            qa = mixed(p + "attn_q_a.weight")
            if qa.kind == kva.kind and qa.bits == kva.bits and qa.group == kva.group and qa.zero == kva.zero:
                # q_a and kv_a read the same normed hidden: one GEMV over both, with row views
                both = MixedWeight(qa.kind, qa.bits, qa.group, qa.N + kva.N, H, torch.cat([qa.codes, kva.codes]),
                                   torch.cat([qa.scales, kva.scales]), qa.zero)
                L.idx["qakva"] = add(both)
                L.idx["qa"] = add(both.rows(0, qa.N))
                L.idx["kva"] = add(both.rows(qa.N, kva.N))
            else:
                L.idx["qa"] = add(qa)
                L.idx["kva"] = add(kva)
            L.idx["qb"] = add(mixed(p + "attn_q_b.weight", qord))
        else:
            L.idx["kva"] = add(kva)
            L.idx["q"] = add(mixed(p + "attn_q.weight", qord))
        L.idx["o"] = add(mixed(p + "attn_output.weight"))
        if dense:
            L.idx["g"] = add(mixed(p + "ffn_gate.weight"))
            L.idx["u"] = add(mixed(p + "ffn_up.weight"))
            L.idx["d"] = add(mixed(p + "ffn_down.weight"))
        else:
            E = cfg.n_experts
            L.router = vec(p + "ffn_gate_inp.weight").reshape(E, H)
            if m.has(p + "exp_probs_b.bias"):
                L.router_bias = vec(p + "exp_probs_b.bias")
            for key, skey, name in (("eg", "sg", "gate"), ("eu", "su", "up"), ("ed", "sd", "down")):
                stacked = mixed(p + f"ffn_{name}_exps.weight")
                n = stacked.N // E
                L.idx[key] = len(ws)
                for e in range(E):
                    ws.append(stacked.rows(e * n, n))
                if cfg.n_shared_experts:
                    L.idx[skey] = add(mixed(p + f"ffn_{name}_shexp.weight"))
        layers.append(L)
    te = m.tensors["token_embd.weight"]
    embed = QWeight.from_raw(raw("token_embd.weight"), te.type, cfg.vocab, H)
    head = add(mixed("output.weight" if m.has("output.weight") else "token_embd.weight"))
    torch.cuda.synchronize(device)
    return DSWeights(MixedTable(ws), embed, vec("output_norm.weight"), layers, head)


def yarn_freq_factors(cfg: ModelConfig, beta_fast: float = 32.0, beta_slow: float = 1.0) -> Optional[torch.Tensor]:
    """Per-frequency divisors (original inverse frequency / YaRN inverse frequency) of the rope
    dims, or None without YaRN scaling. YaRN (Peng et al., 2023): dims whose wavelength fits the
    original context many times keep their frequency, long-wavelength dims are interpolated by
    the scale factor, with a linear ramp between the two correction dims."""
    s = getattr(cfg, "rope_yarn_factor", 0.0)
    if not s or s == 1.0:
        return None
    d, base, L0 = cfg.qk_rope_dim, cfg.rope_theta, cfg.rope_yarn_orig_ctx or cfg.max_ctx

    def corr_dim(rot):
        return d * math.log(L0 / (rot * 2 * math.pi)) / (2 * math.log(base))

    lo = max(math.floor(corr_dim(beta_fast)), 0)
    hi = min(math.ceil(corr_dim(beta_slow)), d - 1)
    i = torch.arange(d // 2, dtype=torch.float64)
    ramp = ((i - lo) / max(hi - lo, 1e-3)).clamp(0, 1)
    extrap = 1.0 - ramp                                  # 1: keep the original frequency
    inv = base ** (-2.0 * i / d)
    yarn = inv / s * (1 - extrap) + inv * extrap
    return inv / yarn


def yarn_attention_scale(cfg: ModelConfig) -> float:
    """Softmax scale of the MLA attention: 1/sqrt(nope + rope), times mscale^2 under YaRN with
    mscale = 1 + log_multiplier * ln(factor)."""
    base = 1.0 / math.sqrt(cfg.qk_nope_dim + cfg.qk_rope_dim)
    s, mul = getattr(cfg, "rope_yarn_factor", 0.0), getattr(cfg, "rope_yarn_log_mul", 0.0)
    if not s or s <= 1.0 or not mul:
        return base
    ms = 1.0 + mul * math.log(s)
    return base * ms * ms
