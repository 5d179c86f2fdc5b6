"""Model configurations: the architecture description every loader produces and every forward
consumes, plus the named presets of the benchmark configurations.

Parity: GGUF metadata keys follow crates/hawking-core/src/model/arch_config.rs:77-126 (prefix
relative reads of ``<arch>.block_count`` etc.); presets follow the workload list the engine is
benchmarked on (tiny Llama Q4_0, Llama-3-8B Q4_K, Mixtral-8x7B Q8_0, Qwen3-Next hybrid .gravity,
DeepSeek-V3-style MLA+MoE fp8).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field, replace
from typing import List, Optional


@dataclass
class ModelConfig:
    arch: str = "llama"              # llama | qwen2 | mixtral | qwen3moe | qwen3next | deepseek2
    vocab: int = 32000
    hidden: int = 512
    layers: int = 4
    n_heads: int = 8
    n_kv_heads: int = 2
    head_dim: int = 64
    ffn: int = 1408
    eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_style: int = 0              # 0 adjacent pairs (llama GGUF), 1 neox halves (qwen)
    rot_dim: int = 0                 # 0 = head_dim
    qkv_bias: bool = False
    qk_norm: bool = False
    tie_embeddings: bool = False
    # MoE
    n_experts: int = 0
    top_k: int = 0
    expert_ffn: int = 0
    n_shared_experts: int = 0
    shared_ffn: int = 0
    shared_gate: bool = False        # sigmoid-gated shared expert (Qwen MoE)
    norm_topk: bool = True
    router: str = "softmax"          # softmax | sigmoid_bias (DeepSeek-V3 noaux_tc)
    n_groups: int = 1
    topk_groups: int = 1
    routed_scale: float = 1.0
    first_dense_layers: int = 0
    # hybrid linear attention (Qwen3-Next)
    full_attn_interval: int = 0      # every Nth layer (1-based) is full attention; 0 = all full
    linear_k_heads: int = 0
    linear_v_heads: int = 0
    linear_head_dim: int = 0
    conv_kernel: int = 4
    attn_output_gate: bool = False
    # MLA (DeepSeek)
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_nope_dim: int = 0
    qk_rope_dim: int = 0
    v_head_dim: int = 0
    # YaRN rope scaling (0: none): scale factor, original context, attention-scale log multiplier
    rope_yarn_factor: float = 0.0
    rope_yarn_orig_ctx: int = 0
    rope_yarn_log_mul: float = 0.0
    # storage
    weight_type: str = "Q4_K"
    embed_type: str = ""             # "" = same as weight_type
    max_ctx: int = 4096

    @property
    def rope_dim(self) -> int:
        return self.rot_dim or self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.n_experts > 0

    def layer_is_full_attention(self, layer: int) -> bool:
        if self.full_attn_interval <= 0:
            return True
        return (layer + 1) % self.full_attn_interval == 0

    def layer_is_moe(self, layer: int) -> bool:
        return self.is_moe and layer >= self.first_dense_layers

    def to_dict(self) -> dict:
        return asdict(self)

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)


PRESETS = {
    # tiny Llama-arch, GGUF Q4_0, embeddings/norms f16.
    "tiny-llama": ModelConfig(arch="llama", vocab=32000, hidden=512, layers=4, n_heads=8, n_kv_heads=2,
                              head_dim=64, ffn=1408, eps=1e-5, rope_theta=10000.0, weight_type="Q4_0",
                              embed_type="F16", max_ctx=2048),
    # Llama-3-8B-arch, GGUF Q4_K.
    "llama3-8b": ModelConfig(arch="llama", vocab=128256, hidden=4096, layers=32, n_heads=32, n_kv_heads=8,
                             head_dim=128, ffn=14336, eps=1e-5, rope_theta=500000.0, weight_type="Q4_K",
                             max_ctx=8192),
    # Mixtral-8x7B-arch, GGUF Q8_0.
    "mixtral-8x7b": ModelConfig(arch="mixtral", vocab=32000, hidden=4096, layers=32, n_heads=32, n_kv_heads=8,
                                head_dim=128, ffn=14336, eps=1e-5, rope_theta=1e6, n_experts=8, top_k=2,
                                expert_ffn=14336, weight_type="Q8_0", max_ctx=4096),
    # Qwen3-Next-style hybrid (DeltaNet + gated full attention), .gravity mixed.
    "qwen3-next": ModelConfig(arch="qwen3next", vocab=151936, hidden=2048, layers=48, n_heads=16, n_kv_heads=2,
                              head_dim=256, rot_dim=64, ffn=512, eps=1e-6, rope_theta=1e7, rope_style=1,
                              qk_norm=True, n_experts=512, top_k=10, expert_ffn=512, n_shared_experts=1,
                              shared_ffn=512, shared_gate=True, norm_topk=True, full_attn_interval=4,
                              linear_k_heads=16, linear_v_heads=32, linear_head_dim=128, conv_kernel=4,
                              attn_output_gate=True, weight_type="MIXED", max_ctx=8192),
    # DeepSeek-V3-style MLA + MoE, fp8 e4m3 128x128 block scales.
    "deepseek-v3": ModelConfig(arch="deepseek2", vocab=129280, hidden=4096, layers=43, n_heads=64, n_kv_heads=64,
                               head_dim=192, ffn=11264, eps=1e-6, rope_theta=10000.0, n_experts=256, top_k=8,
                               expert_ffn=1024, n_shared_experts=1, shared_ffn=1024, router="sigmoid_bias",
                               n_groups=8, topk_groups=4, routed_scale=2.5, first_dense_layers=3,
                               q_lora_rank=1024, kv_lora_rank=512, qk_nope_dim=128, qk_rope_dim=64,
                               v_head_dim=128, weight_type="FP8", max_ctx=16384),
}


def preset(name: str, **overrides) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[name].with_(**overrides)
