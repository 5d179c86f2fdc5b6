"""Seeded synthetic model writers (random-init weights of a named architecture).

The engine is benchmarked on random-init weights; these writers produce byte-faithful GGUF
files for the llama family (llama / qwen2 / mixtral / qwen3moe) so every loader path is the
same one a real checkpoint takes. Weights are N(0, std) from ``seed``; RMSNorm weights are 1.
"""
from __future__ import annotations

import numpy as np

from ..models.config import ModelConfig
from .ggml import GgmlType, type_id
from .gguf import GgufBuilder


def _gguf_arch(cfg: ModelConfig) -> str:
    return "llama" if cfg.arch in ("llama", "mixtral") else cfg.arch


SPECIAL_TOKENS = ["<|begin_of_text|>", "<|end_of_text|>", "<|start_header_id|>", "<|end_header_id|>", "<|eot_id|>"]


def gpt2_byte_alphabet() -> list:
    """GPT-2 printable-byte alphabet: printable Latin-1 bytes keep their code point, the other
    68 map to U+0100.. in byte order."""
    keep = set(range(33, 127)) | set(range(161, 173)) | set(range(174, 256))
    out, extra = [], 0
    for b in range(256):
        if b in keep:
            out.append(chr(b))
        else:
            out.append(chr(256 + extra))
            extra += 1
    return out


def synthetic_bpe_vocab(vocab: int):
    """A deterministic byte-level BPE vocabulary of exactly ``vocab`` tokens: the 256 byte
    tokens, merges over lowercase letters (space-prefixed letters, letter pairs, space-prefixed
    pairs, letter triples, ...) and the Llama-3 control tokens at the end. Returns
    (tokens, merges, bos_id, eos_id)."""
    tokens = gpt2_byte_alphabet()
    n_merge = vocab - len(tokens) - len(SPECIAL_TOKENS)
    if n_merge < 0:
        raise ValueError("vocab too small for a byte-level vocabulary")
    az = [chr(c) for c in range(ord("a"), ord("z") + 1)]
    merges = []

    def gen():
        for c in az:
            yield ("Ġ", c)
        for a in az:
            for b in az:
                yield (a, b)
        for a in az:
            for b in az:
                yield ("Ġ" + a, b)
        for a in az:
            for b in az:
                for c in az:
                    yield (a + b, c)
        for a in az:
            for b in az:
                for c in az:
                    yield ("Ġ" + a + b, c)

    for left, right in gen():
        if len(merges) >= n_merge:
            break
        merges.append(f"{left} {right}")
        tokens.append(left + right)
    while len(tokens) < vocab - len(SPECIAL_TOKENS):  # pad (never produced by merges)
        tokens.append(f"<|reserved_{len(tokens)}|>")
    bos = len(tokens)
    tokens += SPECIAL_TOKENS
    return tokens, merges, bos, bos + 4


def write_llama_family_gguf(path: str, cfg: ModelConfig, seed: int = 0, std: float = 0.02,
                            threads: int = 8) -> str:
    arch = _gguf_arch(cfg)
    rng = np.random.default_rng(seed)
    wt = type_id(cfg.weight_type)
    et = type_id(cfg.embed_type or cfg.weight_type)
    b = GgufBuilder(arch)
    b.set("general.name", f"synthetic-{cfg.arch}")
    toks, merges, bos, eos = synthetic_bpe_vocab(cfg.vocab)
    b.set("tokenizer.ggml.model", "gpt2")
    b.set("tokenizer.ggml.pre", "llama-bpe")
    b.set("tokenizer.ggml.tokens", toks)
    b.set("tokenizer.ggml.merges", merges)
    b.set("tokenizer.ggml.bos_token_id", bos, 4)
    b.set("tokenizer.ggml.eos_token_id", eos, 4)
    b.arch_set("vocab_size", cfg.vocab)
    b.arch_set("context_length", cfg.max_ctx)
    b.arch_set("embedding_length", cfg.hidden)
    b.arch_set("block_count", cfg.layers)
    b.arch_set("feed_forward_length", cfg.ffn)
    b.arch_set("attention.head_count", cfg.n_heads)
    b.arch_set("attention.head_count_kv", cfg.n_kv_heads)
    b.arch_set("rope.dimension_count", cfg.rope_dim)
    b.set_f32(f"{arch}.rope.freq_base", cfg.rope_theta)
    b.set_f32(f"{arch}.attention.layer_norm_rms_epsilon", cfg.eps)
    if cfg.head_dim * cfg.n_heads != cfg.hidden:
        b.arch_set("attention.key_length", cfg.head_dim)
        b.arch_set("attention.value_length", cfg.head_dim)
    if cfg.is_moe:
        b.arch_set("expert_count", cfg.n_experts)
        b.arch_set("expert_used_count", cfg.top_k)
        if cfg.expert_ffn != cfg.ffn:
            b.arch_set("expert_feed_forward_length", cfg.expert_ffn)
        if cfg.shared_ffn:
            b.arch_set("expert_shared_feed_forward_length", cfg.shared_ffn)

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32)

    H, hd, F = cfg.hidden, cfg.head_dim, cfg.ffn
    b.add("token_embd.weight", w(cfg.vocab, H), et, threads)
    for l in range(cfg.layers):
        p = f"blk.{l}."
        b.add(p + "attn_norm.weight", np.ones(H, np.float32), GgmlType.F32)
        b.add(p + "attn_q.weight", w(cfg.n_heads * hd, H), wt, threads)
        b.add(p + "attn_k.weight", w(cfg.n_kv_heads * hd, H), wt, threads)
        b.add(p + "attn_v.weight", w(cfg.n_kv_heads * hd, H), wt, threads)
        if cfg.qkv_bias:
            b.add(p + "attn_q.bias", w(cfg.n_heads * hd), GgmlType.F32)
            b.add(p + "attn_k.bias", w(cfg.n_kv_heads * hd), GgmlType.F32)
            b.add(p + "attn_v.bias", w(cfg.n_kv_heads * hd), GgmlType.F32)
        if cfg.qk_norm:
            b.add(p + "attn_q_norm.weight", np.ones(hd, np.float32), GgmlType.F32)
            b.add(p + "attn_k_norm.weight", np.ones(hd, np.float32), GgmlType.F32)
        b.add(p + "attn_output.weight", w(H, cfg.n_heads * hd), wt, threads)
        b.add(p + "ffn_norm.weight", np.ones(H, np.float32), GgmlType.F32)
        if cfg.is_moe:
            E, Fe = cfg.n_experts, cfg.expert_ffn
            b.add(p + "ffn_gate_inp.weight", w(E, H), GgmlType.F32)
            b.add(p + "ffn_gate_exps.weight", w(E, Fe, H), wt, threads)
            b.add(p + "ffn_up_exps.weight", w(E, Fe, H), wt, threads)
            b.add(p + "ffn_down_exps.weight", w(E, H, Fe), wt, threads)
            if cfg.shared_ffn:
                Fs = cfg.shared_ffn
                b.add(p + "ffn_gate_shexp.weight", w(Fs, H), wt, threads)
                b.add(p + "ffn_up_shexp.weight", w(Fs, H), wt, threads)
                b.add(p + "ffn_down_shexp.weight", w(H, Fs), wt, threads)
                if cfg.shared_gate:
                    b.add(p + "ffn_gate_inp_shexp.weight", w(1, H), GgmlType.F32)
        else:
            b.add(p + "ffn_gate.weight", w(F, H), wt, threads)
            b.add(p + "ffn_up.weight", w(F, H), wt, threads)
            b.add(p + "ffn_down.weight", w(H, F), wt, threads)
    b.add("output_norm.weight", np.ones(H, np.float32), GgmlType.F32)
    if not cfg.tie_embeddings:
        b.add("output.weight", w(cfg.vocab, H), wt, threads)
    return b.write(path)


def write_deepseek2_gguf(path: str, cfg: ModelConfig, seed: int = 0, std: float = 0.02, mix: bool = True,
                         yarn: float = 0.0, threads: int = 8) -> str:
    """A ``deepseek2`` GGUF (MLA + MoE, llama.cpp tensor names) of random N(0, std) weights. The
    projections take ``cfg.weight_type``; with ``mix`` the routed experts' down projections and
    the LM head are Q6_K, the shared experts Q8_0 and the dense FFN Q4_0 (every loader mapping is
    exercised). ``yarn`` > 1 writes YaRN rope-scaling keys with that factor."""
    rng = np.random.default_rng(seed)
    wt = type_id(cfg.weight_type)
    b = GgufBuilder("deepseek2")
    b.set("general.name", "synthetic-deepseek2")
    toks, merges, bos, eos = synthetic_bpe_vocab(cfg.vocab)
    b.set("tokenizer.ggml.model", "gpt2")
    b.set("tokenizer.ggml.pre", "llama-bpe")
    b.set("tokenizer.ggml.tokens", toks)
    b.set("tokenizer.ggml.merges", merges)
    b.set("tokenizer.ggml.bos_token_id", bos, 4)
    b.set("tokenizer.ggml.eos_token_id", eos, 4)
    H, nh, nope, rd, vd = cfg.hidden, cfg.n_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim
    E, Fe, ns = cfg.n_experts, cfg.expert_ffn, cfg.n_shared_experts
    for k, v in (("vocab_size", cfg.vocab), ("context_length", cfg.max_ctx), ("embedding_length", H),
                 ("block_count", cfg.layers), ("feed_forward_length", cfg.ffn), ("attention.head_count", nh),
                 ("attention.head_count_kv", nh), ("attention.key_length", nope + rd),
                 ("attention.value_length", vd), ("rope.dimension_count", rd),
                 ("attention.kv_lora_rank", cfg.kv_lora_rank), ("leading_dense_block_count", cfg.first_dense_layers),
                 ("expert_count", E), ("expert_used_count", cfg.top_k), ("expert_shared_count", ns),
                 ("expert_feed_forward_length", Fe), ("expert_group_count", cfg.n_groups),
                 ("expert_group_used_count", cfg.topk_groups),
                 ("expert_gating_func", 2 if cfg.router == "sigmoid_bias" else 1)):
        b.arch_set(k, v)
    if cfg.q_lora_rank:
        b.arch_set("attention.q_lora_rank", cfg.q_lora_rank)
    b.arch_set("expert_weights_norm", bool(cfg.norm_topk))
    b.set_f32("deepseek2.expert_weights_scale", cfg.routed_scale)
    b.set_f32("deepseek2.rope.freq_base", cfg.rope_theta)
    b.set_f32("deepseek2.attention.layer_norm_rms_epsilon", cfg.eps)
    if yarn > 1.0:
        b.set("deepseek2.rope.scaling.type", "yarn")
        b.set_f32("deepseek2.rope.scaling.factor", yarn)
        b.arch_set("rope.scaling.original_context_length", max(cfg.max_ctx // 4, 64))
        b.set_f32("deepseek2.rope.scaling.yarn_log_multiplier", 0.1)

    def w(*shape):
        return (rng.standard_normal(shape, dtype=np.float32) * std).astype(np.float32)

    def norm(n):
        return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)

    t6 = GgmlType.Q6_K if mix else wt
    t8 = GgmlType.Q8_0 if mix else wt
    t40 = GgmlType.Q4_0 if mix else wt
    b.add("token_embd.weight", w(cfg.vocab, H), GgmlType.F16)
    for l in range(cfg.layers):
        p = f"blk.{l}."
        b.add(p + "attn_norm.weight", norm(H), GgmlType.F32)
        if cfg.q_lora_rank:
            b.add(p + "attn_q_a.weight", w(cfg.q_lora_rank, H), wt, threads)
            b.add(p + "attn_q_a_norm.weight", norm(cfg.q_lora_rank), GgmlType.F32)
            b.add(p + "attn_q_b.weight", w(nh * (nope + rd), cfg.q_lora_rank), wt, threads)
        else:
            b.add(p + "attn_q.weight", w(nh * (nope + rd), H), wt, threads)
        b.add(p + "attn_kv_a_mqa.weight", w(cfg.kv_lora_rank + rd, H), wt, threads)
        b.add(p + "attn_kv_a_norm.weight", norm(cfg.kv_lora_rank), GgmlType.F32)
        b.add(p + "attn_kv_b.weight", w(nh * (nope + vd), cfg.kv_lora_rank), wt, threads)
        b.add(p + "attn_output.weight", w(H, nh * vd), wt, threads)
        b.add(p + "ffn_norm.weight", norm(H), GgmlType.F32)
        if l < cfg.first_dense_layers:
            b.add(p + "ffn_gate.weight", w(cfg.ffn, H), t40, threads)
            b.add(p + "ffn_up.weight", w(cfg.ffn, H), t40, threads)
            b.add(p + "ffn_down.weight", w(H, cfg.ffn), t40, threads)
            continue
        # softmax routers get a wide logit spread (decisive top-k); sigmoid scores would saturate
        b.add(p + "ffn_gate_inp.weight", w(E, H) * (1 if cfg.router == "sigmoid_bias" else 5), GgmlType.F32)
        if cfg.router == "sigmoid_bias":
            b.add(p + "exp_probs_b.bias", (0.01 * rng.standard_normal(E)).astype(np.float32), GgmlType.F32)
        b.add(p + "ffn_gate_exps.weight", w(E, Fe, H), wt, threads)
        b.add(p + "ffn_up_exps.weight", w(E, Fe, H), wt, threads)
        b.add(p + "ffn_down_exps.weight", w(E, H, Fe), t6, threads)
        if ns:
            b.add(p + "ffn_gate_shexp.weight", w(ns * Fe, H), t8, threads)
            b.add(p + "ffn_up_shexp.weight", w(ns * Fe, H), t8, threads)
            b.add(p + "ffn_down_shexp.weight", w(H, ns * Fe), t8, threads)
    b.add("output_norm.weight", norm(H), GgmlType.F32)
    b.add("output.weight", w(cfg.vocab, H), t6, threads)
    return b.write(path)


def write_tokenizer_gguf(path: str, vocab: int, arch: str = "llama") -> str:
    """A GGUF file holding only the synthetic byte-level BPE tokenizer of ``vocab`` tokens (no
    tensors): the tokenizer for models built from random weights without a GGUF of their own."""
    toks, merges, bos, eos = synthetic_bpe_vocab(vocab)
    b = GgufBuilder(arch)
    b.set("general.name", "synthetic-tokenizer")
    b.set("tokenizer.ggml.model", "gpt2")
    b.set("tokenizer.ggml.pre", "llama-bpe")
    b.set("tokenizer.ggml.tokens", toks)
    b.set("tokenizer.ggml.merges", merges)
    b.set("tokenizer.ggml.bos_token_id", bos, 4)
    b.set("tokenizer.ggml.eos_token_id", eos, 4)
    b.arch_set("vocab_size", vocab)
    b.write(path)
    return path


def random_prompt(n: int, vocab: int, seed: int = 1) -> list:
    """Uniform-random token ids (the benchmark prompts)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n).tolist()
