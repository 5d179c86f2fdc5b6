"""Rank-failure detection for a multi-GPU serving group (host side).

Every rank publishes a heartbeat (step number and wall time) in the process group's key-value
store after each step; ``PeerMonitor.dead_peers`` lists ranks whose heartbeat is older than the
timeout (or that never published one). Device-side, every fused-collective wait is bounded and
reports ``HK_ERR_PEER_TIMEOUT`` in the status word; ``check_device_status`` turns that into a
``PeerFailure`` on the host after a step. A failed step makes the serving loop report unhealthy
(503 on /healthz) and stop admitting work until the group is rebuilt.

Parity: crates/hawking-core/src/engine.rs:171-190 (abort flag, per-token stall watchdog),
crates/hawking-serve/src/lib.rs:995-1060 (fallback on error), crates/hawking-serve/src/http.rs:871-888
(bounded queue, slot_exhausted).
"""
from __future__ import annotations

import time
from typing import List, Optional

HK_ERR_PEER_TIMEOUT = 2
HK_ERR_MBAR_TIMEOUT = 3


class PeerFailure(RuntimeError):
    def __init__(self, message: str, ranks: Optional[List[int]] = None):
        super().__init__(message)
        self.ranks = ranks or []


class PeerMonitor:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "hk/heartbeat/"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix = timeout_s, prefix
        self.started = time.time()

    def beat(self, step: int):
        self.store.set(f"{self.prefix}{self.rank}", f"{step}:{time.time():.6f}")

    def last_beat(self, rank: int):
        key = f"{self.prefix}{rank}"
        if not self.store.check([key]):
            return None
        step, t = self.store.get(key).decode().split(":")
        return int(step), float(t)

    def dead_peers(self) -> List[int]:
        now = time.time()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            lb = self.last_beat(r)
            ref = lb[1] if lb else self.started
            if now - ref > self.timeout_s:
                dead.append(r)
        return dead

    def check(self):
        dead = self.dead_peers()
        if dead:
            raise PeerFailure(f"ranks {dead} stopped reporting for more than {self.timeout_s} s", dead)


def check_device_status(status_tensor, what: str = "collective") -> None:
    """Raise PeerFailure if a kernel reported a bounded-wait timeout in its status word."""
    st = int(status_tensor.item())
    if st == HK_ERR_PEER_TIMEOUT:
        raise PeerFailure(f"{what}: a peer did not arrive within the bounded wait")
    if st:
        raise RuntimeError(f"{what}: device error {st}")
