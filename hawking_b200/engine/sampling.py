"""Sampling parameters and per-request random streams.

Parity: crates/hawking-core/src/engine.rs:150 (SamplingParams) and crates/hawking-core/src/sample.rs
(order: repetition penalty -> temperature (0 = greedy) -> softmax -> top-k -> top-p -> draw).
The device sampler consumes one uniform per row, drawn from the request's own PCG64 stream, so a
seeded request reproduces regardless of how it was batched.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

from .._ext import native


@dataclass
class SamplingParams:
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    repetition_penalty: float = 1.0
    seed: int = 42
    max_tokens: int = 16
    stop_ids: List[int] = field(default_factory=list)
    json_mode: bool = False  # only tokens that keep the output a prefix of one JSON object

    @property
    def greedy(self) -> bool:
        """Served by the fused on-device argmax lane (JSON mode needs the logits on the host)."""
        return self.temperature <= 0.0 and self.repetition_penalty == 1.0 and not self.json_mode


class RequestRng:
    def __init__(self, seed: int):
        self._g = native().Pcg64(seed)

    def uniform(self) -> float:
        return self._g.next_f32()
