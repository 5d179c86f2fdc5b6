"""Engine configuration: one typed set of engine / serving knobs, plus the few ``HK_*``
environment overrides the runtime reads (documented here with their defaults).

Parity: crates/hawking-core/src/engine.rs:33-101 (EngineConfig), crates/hawking-serve/src/lib.rs:
359-450 (ServeOptions), :34-200 (RuntimeProfile -> LeverPlan, profile contracts), crates/hawking-core/src/lib.rs:198-226 (env helpers); the reference's
284-flag sprawl (workspace/docs/reference/env_flags.md) is deliberately not reproduced.
"""
from __future__ import annotations

import os
from dataclasses import asdict, dataclass, field
from typing import Dict, Optional

# name -> (default, meaning)
ENV_FLAGS = {
    "HK_PDL": ("1", "programmatic dependent launch between consecutive kernels (0 disables)"),
    "HK_PREFETCH": ("0", "decode GEMVs prefetch the next projection's weights into L2 (measured slower; A/B only)"),
    "HK_TRACE": ("0", "NVTX ranges around engine phases (engine.step > schedule / forward / sample)"),
    "HK_LEDGER": ("0", "per-step host cost ledger kept on the engine (Engine.ledger_json())"),
    "HK_GEMM_PAIR": ("0", "1: prefill GEMMs of whole 256-row weight pair tiles run on CTA pairs (cta_group::2)"),
    "HK_GEMM_SERIALIZE": ("unset", "debug: tensor-core GEMM issues each stage only after the previous one retired"),
    "HK_BOUNDS": ("0", "build time: compile index guards into the kernels (setup.py)"),
    "HK_SKIP_CUDA": ("0", "build time: build only the host (C++) module"),
    "HK_STARTUP_TIMING": ("0", "Engine.from_gguf prints its load phases (open, config, weights, engine) as JSON"),
    "HK_SMALL_BATCH": ("w4a16", "decode GEMVs of <= 8 rows: w4a16 (bf16 activations, tensor cores) or w4a8 (int8 blocks, dp4a)"),
    "HK_MG_MATH": ("int", "W4A16 GEMV math: int (two int8 limbs per activation) or bf16"),
    "HK_MG_PER_SM": ("max", "W4A16 GEMV CTAs per SM (1..3; fewer leave room for the next kernel's programmatic launch)"),
    "HK_ROPE_EPI": ("1", "RoPE and the paged K/V append in the QKV GEMV epilogue (0: separate kernel)"),
    "HK_DSTEP": ("0", "1: the persistent one-launch decode step for <= 4 rows (measured slower; opt-in)"),
    "HK_DS_WAIT_NS": ("0", "persistent decode step: nanosleep between polls of a grid-barrier flag"),
    "HK_ATTN_TC": ("1", "decode attention on the tensor cores (0: the CUDA-core cluster kernel)"),
    "HK_ATTN_STAGES": ("4", "tensor-core decode attention ring stages for one-wave launches (2 or 4)"),
    "HK_ATTN_PREFETCH_MB": ("48", "L2 prefetch budget of one decode-attention launch, split evenly over its CTAs"),
    "HK_STREAM_K": ("1", "decode-batch Q4_K GEMMs with more weight tiles than SMs run stream-K (0: one-tile split-K)"),
    "HK_FUSED_SWIGLU_PREFILL": ("0", "prefill FFN gate/up with the SwiGLU in the GEMM epilogue (0: plain GEMM + SwiGLU kernel)"),
    "HK_WIDE_GGUF": ("1", "MoE GGUF models: attention projections of forwards above 32 rows as tensor-core GEMMs"),
    "HK_MOE_PREFILL": ("1", "MoE layers of prefill-sized forwards run grouped tensor-core expert GEMMs"),
    "HK_TP_WAIT_NS": ("0", "tensor-parallel push all-reduce: nanosleep between polls of a peer flag"),
    "NCCL_NVLS_ENABLE": ("library default", "NCCL NVLink SHARP; the multi-GPU tests set 0"),
}


def env_flag(name: str) -> str:
    """The value of a documented HK_* flag (its default when unset)."""
    if name not in ENV_FLAGS:
        raise KeyError(f"undocumented flag {name}")
    return os.environ.get(name, ENV_FLAGS[name][0])


@dataclass
class EngineConfig:
    """Sizing and policy of one engine (the arguments of Engine.build and its variants)."""
    max_batch: int = 8                 # sequences decoded together
    max_ctx: Optional[int] = None      # context window (default: the model's)
    block_size: int = 64               # tokens per paged KV block
    num_blocks: Optional[int] = None   # KV pool size (default: kv_fraction of free memory)
    max_rows: int = 64                 # rows one forward holds
    max_prefill_tokens: int = 512      # prompt tokens per scheduler step (chunked prefill)
    kv_fraction: float = 0.5           # share of free device memory for the KV pool
    policy: int = 0                    # 0 default, 1 greedy-first, 2 prefix-grouped

    def build_kwargs(self) -> dict:
        return asdict(self)


@dataclass(frozen=True)
class LeverPlan:
    """What a runtime profile changes. ``engine`` overrides EngineConfig fields, ``model`` sets
    attributes on the built model (only those it has), ``serve`` sets ServeLoop options."""
    engine: Dict[str, object] = field(default_factory=dict)
    model: Dict[str, object] = field(default_factory=dict)
    serve: Dict[str, object] = field(default_factory=dict)
    contract: str = ""


# The levers this engine has: batch width and prefill budget (EngineConfig), the scheduler policy,
# the row count from which dense Q4_K projections leave the W4A8 dp4a GEMV for the W4A16 tensor-core
# GEMM (``tc_min_rows``; 1 = no int8 activation rounding at any batch), and the serving loop's
# gather window (``gather_ms``: a step with free batch slots first waits this long for arrivals).
RUNTIME_PROFILES: Dict[str, LeverPlan] = {
    "default": LeverPlan(contract="profile=default: the configured engine, no profile-level trade."),
    "fast": LeverPlan(engine={"max_prefill_tokens": 2048}, serve={"gather_ms": 0.0},
                      contract="profile=fast: whole 2k prompts in one tensor-core forward; decode rows at "
                               "batch <= 8 on the W4A8 GEMV (int8 activation blocks of 32)."),
    "race": LeverPlan(engine={"max_prefill_tokens": 2048, "max_batch": 64, "policy": 1}, serve={"gather_ms": 0.0},
                      contract="profile=race: fast + 64-wide decode batches, greedy-first scheduling; goal: "
                               "aggregate tokens/s."),
    "efficient": LeverPlan(engine={"max_prefill_tokens": 2048, "max_batch": 64}, serve={"gather_ms": 5.0},
                           contract="profile=efficient: fast + a 5 ms gather window before a step with free "
                                    "slots, so steps run wider (fewer weight passes per token: lower J/token) "
                                    "at some inter-token latency."),
    "exact": LeverPlan(model={"tc_min_rows": 1},
                       contract="profile=exact: every dense Q4_K projection on the W4A16 tensor-core path "
                                "(bf16 activations, fp32 accumulation): no int8 activation rounding; "
                                "slower decode."),
}


def runtime_profile(name: str) -> LeverPlan:
    """The lever plan of a named profile (default / fast / race / efficient / exact)."""
    try:
        return RUNTIME_PROFILES[name]
    except KeyError:
        raise ValueError(f"unknown runtime profile {name!r}; one of {sorted(RUNTIME_PROFILES)}") from None


def apply_profile(config: EngineConfig, name: str) -> EngineConfig:
    """``config`` with the profile's engine overrides applied (a new object)."""
    plan = runtime_profile(name)
    return EngineConfig(**{**asdict(config), **plan.engine})


class MemoryBudgetError(MemoryError):
    """A model or KV pool that does not fit the device is refused before anything is allocated."""


def check_memory_budget(need_bytes: int, free_bytes: int, what: str, reserve_bytes: int = 1 << 30) -> None:
    """Refuse ``what`` when ``need_bytes`` plus a working reserve exceeds ``free_bytes``.

    Parity: crates/hawking-core/src/model/mod.rs:96-115 (memory budget refusal)."""
    if need_bytes + reserve_bytes > free_bytes:
        raise MemoryBudgetError(f"{what}: needs {need_bytes / 2**30:.2f} GiB + {reserve_bytes / 2**30:.2f} GiB "
                                f"reserve, {free_bytes / 2**30:.2f} GiB free on the device")
