"""Failure detection without a GPU fault: host-side gloo ranks that stop, raise or never join.

Parity: crates/hawking-core/src/engine.rs:171-190 (stall watchdog); the multi-GPU design adds
heartbeat / bounded-wait detection (no reference counterpart)."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout=10):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout))


def _heartbeat_worker(rank, world, port, out):
    from hawking_b200.parallel.health import PeerFailure, PeerMonitor
    _init(rank, world, port)
    store = dist.distributed_c10d._get_default_store()
    mon = PeerMonitor(store, rank, world, timeout_s=1.0)
    for step in range(3):
        mon.beat(step)
        dist.barrier()
    if rank == 1:
        time.sleep(4.0)  # stops beating (a stalled rank), joins nothing
        return
    t0 = time.time()
    detected = None
    while time.time() - t0 < 10:
        try:
            mon.check()
        except PeerFailure as e:
            detected = e.ranks
            break
        mon.beat(99)
        time.sleep(0.1)
    torch.save({"dead": detected, "after": time.time() - t0}, out)


def test_heartbeat_detects_stalled_rank(tmp_path):
    out = str(tmp_path / "hb.pt")
    mp.spawn(_heartbeat_worker, args=(2, _port(), out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["dead"] == [1]
    assert r["after"] < 5.0


def _raise_worker(rank, world, port, out):
    _init(rank, world, port, timeout=5)
    t = torch.ones(4)
    dist.all_reduce(t)
    if rank == 1:
        os._exit(3)  # a rank that dies between steps, with nothing in flight
    err = None
    t0 = time.time()
    try:
        dist.all_reduce(t)
    except Exception as e:  # noqa: BLE001 - the peer is gone: the collective must fail, not hang
        err = type(e).__name__
    torch.save({"err": err, "after": time.time() - t0}, out)


def test_collective_fails_when_peer_exits(tmp_path):
    out = str(tmp_path / "x.pt")
    ctx = mp.spawn(_raise_worker, args=(2, _port(), out), nprocs=2, join=False)
    ctx.processes[0].join(60)
    ctx.processes[1].join(60)
    r = torch.load(out)
    assert r["err"] is not None and r["after"] < 30


def test_rank_that_never_joins_times_out():
    port = _port()
    t0 = time.time()
    with pytest.raises(Exception):
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=2))
    assert time.time() - t0 < 60
    if dist.is_initialized():
        dist.destroy_process_group()


def test_device_status_maps_to_peer_failure():
    from hawking_b200.parallel.health import PeerFailure, check_device_status
    check_device_status(torch.zeros(1, dtype=torch.int32))
    with pytest.raises(PeerFailure):
        check_device_status(torch.tensor([2], dtype=torch.int32))
