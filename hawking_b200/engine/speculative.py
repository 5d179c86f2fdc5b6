"""Lossless speculative decoding: online n-gram drafts verified by one batched forward.

Each cycle feeds the last emitted token plus up to k drafted tokens as consecutive rows of one
sequence (k + 1 <= 8, the small-batch GEMV path) and takes the device argmax of every row; the
longest draft prefix that matches the argmaxes is accepted together with the argmax after it, the
KV written for rejected drafts is truncated away, and the drafter learns the emitted tokens. The
verify rows use the same kernels and attention splits as single-row greedy decode, so the output
is bitwise the greedy output. A governor turns drafting off when acceptance stays low.

Parity: crates/hawking-speculate/src/user_ngram.rs (draft), crates/hawking-speculate/src/shared.rs:66
(verify until mismatch), crates/hawking-speculate/src/governor.rs (hysteresis),
crates/hawking-core/src/model/qwen_dense.rs:9384 (forward_tokens_verify), spec/src/metrics_sep.rs
(base vs accelerated token counts kept apart).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from .._ext import native


@dataclass
class SpecStats:
    cycles: int = 0
    drafted: int = 0
    accepted: int = 0
    emitted: int = 0
    forward_rows: int = 0
    seconds: float = 0.0

    @property
    def accept_rate(self) -> float:
        return self.accepted / self.drafted if self.drafted else 0.0

    @property
    def tokens_per_cycle(self) -> float:
        return self.emitted / self.cycles if self.cycles else 0.0


class SpeculativeDecoder:
    def __init__(self, engine, k: int = 4, governor=None, min_accept_rate: float = 0.2):
        n = native()
        self.engine = engine
        self.k = max(0, min(k, n.MAX_VERIFY_BATCH - 1))
        self.draft = n.NgramDraft()
        self.gov = governor or n.SpecGovernor(16, min_accept_rate)
        self.stats = SpecStats()

    def _forward_rows(self, sid: int, tokens: Sequence[int], p0: int, logits_row: Optional[int]) -> List[int]:
        """Run ``tokens`` at positions p0.. of sequence ``sid``; returns the greedy id of every row
        (logits_row=None), of the single row ``logits_row``, or nothing (logits_row=-1)."""
        eng, m, kv = self.engine, self.engine.model, self.engine.kv
        n = len(tokens)
        if not kv.bm.reserve(sid, p0 + n):
            raise RuntimeError("KV pool exhausted")
        kv.sync_tables([sid])
        r = kv.row(sid)
        slots = kv.bm.slots(sid, p0, p0 + n)
        pos = list(range(p0, p0 + n))
        eng.stats.h2d_bytes += m.inp.upload(list(tokens), pos, slots, [r] * n, [p + 1 for p in pos])
        m.long_runs = n >= 16  # the engine's rule: same kernels, same logits as plain decode
        if logits_row == -1:
            m.forward(n, "none", n_logits=-1)
            m.long_runs = False
            self.stats.forward_rows += n
            return []
        if logits_row is None:
            m.forward(n, "greedy")
            k = n
        else:
            m.logit_rows[:1].copy_(torch.tensor([logits_row], dtype=torch.int32), non_blocking=True)
            m.forward(n, "greedy", n_logits=1)
            k = 1
        m.long_runs = False
        ids = m.next_ids[:k].cpu().tolist()
        eng.stats.d2h_bytes += 4 * k
        self.stats.forward_rows += n
        return ids

    def generate(self, prompt: Sequence[int], max_tokens: int, stop_ids: Sequence[int] = ()) -> List[int]:
        eng, m, kv = self.engine, self.engine.model, self.engine.kv
        stop = set(int(t) for t in stop_ids)
        sid = -next(eng._ids)
        t0 = time.perf_counter()
        old_force = m.force_splits
        m.force_splits = m.num_splits(1)
        try:
            prompt = [int(t) for t in prompt]
            R = min(getattr(m, "row_limit", m.max_rows), eng.max_prefill_tokens)
            tok = None
            for c0 in range(0, len(prompt), R):  # prefill in the same chunks as the engine
                c1 = min(len(prompt), c0 + R)
                last = c1 == len(prompt)
                ids = self._forward_rows(sid, prompt[c0:c1], c0, (c1 - c0 - 1) if last else -1)
                tok = ids[0] if last else None
            history = prompt + [tok]
            out = [tok]
            self.draft.warm_start(prompt)
            self.draft.note_token(history[-2] if len(history) >= 2 else tok)
            self.draft.note_token(tok)
            while len(out) < max_tokens and out[-1] not in stop:
                room = max_tokens - len(out)
                k = min(self.k, room - 1) if self.gov.enabled else 0
                draft = list(self.draft.propose(history[-2:], k)) if k > 0 else []
                p = len(history) - 1
                verifier = self._forward_rows(sid, [history[-1]] + draft, p, None)
                emit, a = native().accept_draft(draft, verifier)
                kv.bm.truncate(sid, p + 1 + a)
                kv.sync_tables([sid])
                for i, t in enumerate(emit):  # stop tokens and max_tokens cut the emitted run
                    if t in stop or len(out) + i + 1 >= max_tokens:
                        emit = emit[: i + 1]
                        break
                history += emit
                out += emit
                for t in emit:
                    self.draft.note_token(t)
                st = self.stats
                st.cycles += 1
                st.drafted += len(draft)
                st.accepted += a
                st.emitted += len(emit)
                if draft:
                    self.gov.step(a > 0)
                else:
                    self.gov.tick_disabled()
            return out
        finally:
            m.force_splits = old_force
            kv.drop(sid)
            self.stats.seconds += time.perf_counter() - t0
