"""Engine configuration: one typed set of engine / serving knobs, plus the few ``HK_*``
environment overrides the runtime reads (documented here with their defaults).

Parity: crates/hawking-core/src/engine.rs:33-101 (EngineConfig), crates/hawking-serve/src/lib.rs:
359-450 (ServeOptions), crates/hawking-core/src/lib.rs:198-226 (env helpers); the reference's
284-flag sprawl (workspace/docs/reference/env_flags.md) is deliberately not reproduced.
"""
from __future__ import annotations

import os
from dataclasses import asdict, dataclass
from typing import Optional

# name -> (default, meaning)
ENV_FLAGS = {
    "HK_PDL": ("1", "programmatic dependent launch between consecutive kernels (0 disables)"),
    "HK_PREFETCH": ("0", "decode GEMVs prefetch the next projection's weights into L2 (measured slower; A/B only)"),
    "HK_TRACE": ("0", "NVTX ranges around engine phases (engine.step > schedule / forward / sample)"),
    "HK_LEDGER": ("0", "per-step host cost ledger kept on the engine (Engine.ledger_json())"),
    "HK_GEMM_SERIALIZE": ("unset", "debug: tensor-core GEMM issues each stage only after the previous one retired"),
    "HK_BOUNDS": ("0", "build time: compile index guards into the kernels (setup.py)"),
    "HK_SKIP_CUDA": ("0", "build time: build only the host (C++) module"),
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
