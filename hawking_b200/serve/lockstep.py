"""Multi-rank serving: rank 0 serves HTTP, every rank steps the same engine schedule.

Under tensor / expert parallelism every rank must run the same forwards in the same order (their
collectives pair up). Rank 0 owns the HTTP server and the scheduler's inputs; ``LeaderEngine``
wraps its engine and records every call that changes the engine's state (request admission,
abort). Before each call that runs device collectives (``step``, ``embed``) it broadcasts the
recorded calls plus that call over a CPU (gloo) group; ``follow`` on the other ranks replays them
on its own engine, so the schedulers (deterministic, C++) make identical plans and request ids
agree. Sampling is identical on every rank: the sampler's uniforms come from each request's seeded
stream and tensor-parallel logits are gathered before the draw.

Every step ends with an all-reduce of a success flag: a step that failed on any rank (a device
status word set, a collective that timed out) fails on the leader too, whose serve loop then
answers its requests with 503 and sends their aborts, which the followers replay. ``stop`` ends
the followers.

Parity: crates/hawking-serve/src/lib.rs:525-1121 (one serve loop driving the engine; the
reference runs one process on one device, so the broadcast of the step's inputs is this build's).
"""
from __future__ import annotations

from typing import Any, List, Optional, Tuple

import torch.distributed as dist

from ..engine.sampling import SamplingParams

Op = Tuple[str, Any]


def _params_to_dict(p: SamplingParams) -> dict:
    return dict(temperature=p.temperature, top_k=p.top_k, top_p=p.top_p, repetition_penalty=p.repetition_penalty,
                seed=p.seed, max_tokens=p.max_tokens, stop_ids=list(p.stop_ids), json_mode=p.json_mode)


class LeaderEngine:
    """Rank 0's engine proxy: every state change is recorded and broadcast before the next
    collective-bearing call. Attribute reads pass through to the wrapped engine."""

    def __init__(self, engine, group: Optional[dist.ProcessGroup] = None):
        object.__setattr__(self, "_engine", engine)
        object.__setattr__(self, "_group", group)
        object.__setattr__(self, "_pending", [])

    def __getattr__(self, name):
        return getattr(self._engine, name)

    def __setattr__(self, name, value):  # e.g. the serve loop handing the tokenizer to the engine
        setattr(self._engine, name, value)

    def _flush(self, action: Op) -> None:
        msg = [self._pending + [action]]
        dist.broadcast_object_list(msg, src=0, group=self._group)
        self._pending.clear()

    def add_request(self, prompt, params: SamplingParams):
        rid = self._engine.add_request(list(prompt), params)
        self._pending.append(("add", (list(prompt), _params_to_dict(params), rid)))
        return rid

    def abort(self, rid):
        self._engine.abort(rid)
        self._pending.append(("abort", rid))

    def step(self):
        self._flush(("step", None))
        err = None
        try:
            events = self._engine.step()
        except Exception as e:  # noqa: BLE001 - agreed with the other ranks below
            err, events = e, None
        if not _all_ok(err is None, self._group):
            raise err if err is not None else RuntimeError("engine step failed on another rank")
        return events

    def embed(self, ids):
        self._flush(("embed", list(ids)))
        return self._engine.embed(list(ids))

    def stop(self) -> None:
        """Ends every follower's loop (call once, after the last step)."""
        self._flush(("stop", None))


def _all_ok(ok: bool, group) -> bool:
    """Whether the step succeeded on every rank (one small all-reduce on the CPU group)."""
    import torch
    t = torch.tensor([1 if ok else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


def follow(engine, group: Optional[dist.ProcessGroup] = None) -> int:
    """Non-zero ranks: replay the leader's calls until it stops. Returns the number of steps run."""
    steps = 0
    while True:
        msg = [None]
        dist.broadcast_object_list(msg, src=0, group=group)
        for kind, arg in msg[0]:
            if kind == "add":
                prompt, params, rid = arg
                got = engine.add_request(prompt, SamplingParams(**params))
                if got != rid:
                    raise RuntimeError(f"lockstep: request id {got} on this rank, {rid} on rank 0")
            elif kind == "abort":
                engine.abort(arg)
            elif kind == "step":
                ok = True
                try:
                    engine.step()
                except Exception:  # noqa: BLE001 - the leader fails its requests and sends the aborts
                    ok = False
                _all_ok(ok, group)
                steps += 1
            elif kind == "embed":
                engine.embed(arg)
            elif kind == "stop":
                return steps
            else:
                raise RuntimeError(f"lockstep: unknown call {kind!r}")
