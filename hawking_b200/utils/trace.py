"""Named ranges on the profiler timeline (NVTX, from the native module) around engine phases.

Enabled with ``HK_TRACE=1`` (or ``trace.enable()``); otherwise ``trace(name)`` is a no-op context
manager. Ranges nest: ``engine.step`` > ``schedule`` / ``upload`` / ``forward`` / ``sample`` /
``commit``.

Parity: crates/hawking-core/src/metal/mod.rs:177-231 (PhysicalTraceGuard: os_signpost phase
intervals), crates/hawking-core/src/metal/physical_signpost.c.
"""
from __future__ import annotations

import os
from contextlib import contextmanager

_enabled = os.environ.get("HK_TRACE", "0") == "1"


def enable(on: bool = True) -> None:
    global _enabled
    _enabled = on


def enabled() -> bool:
    return _enabled


@contextmanager
def trace(name: str):
    if not _enabled:
        yield
        return
    from .._ext import native
    n = native()
    n.trace_push(name)
    try:
        yield
    finally:
        n.trace_pop()
