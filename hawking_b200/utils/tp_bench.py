"""Microbenchmark of one tensor-parallel all-reduce site at decode batch sizes (Llama-3-8B FFN-down
shape, Q4_K weights), one process per GPU.

Three ways to finish a row-parallel projection and feed the next layer, each replayed ``--iters``
times inside one CUDA graph and timed with CUDA events (max over ranks):

* ``local``  - GEMV into the residual + RMSNorm->q8, no communication (the TP=1 cost of the shard)
* ``fused``  - GEMV whose epilogue pushes partials to every rank over NVLink, then the fused
               bounded-wait all-reduce + RMSNorm->q8 kernel (what the decode step runs)
* ``nccl``   - GEMV, NCCL all-reduce of the partial, add + RMSNorm->q8 (the library baseline)

The weights cycle through copies larger than L2, as in a decode step.

``--step`` instead times whole Llama-3-8B decode steps (bs1, 2048-token context) of the
tensor-parallel model three ways, to split the cost of the fused collectives:

* ``tp``         - the real step
* ``own_slot``   - every consumer reads only this rank's own partial (no wait on a peer; the
                   producers still push to every rank)
* ``local_push`` - producers push only to this rank and consumers read only that (no NVLink)

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \
        -m hawking_b200.utils.tp_bench --rows 1
"""
from __future__ import annotations

import argparse
import datetime
import json
import os

import torch
import torch.distributed as dist

H, F = 4096, 14336


def _graph_time(fn, iters: int) -> float:
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1000.0 / iters
    del g
    return us


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--iters", type=int, default=64)
    ap.add_argument("--step", action="store_true", help="time whole decode steps (see the module docstring)")
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=60))

    if args.step:
        return step_mode(args, rank, world, dev)
    from hawking_b200 import ops
    from hawking_b200.formats.ggml import GgmlType
    from hawking_b200.ops import Q8Act, QWeight
    from hawking_b200.parallel.tp import TPComm

    rows, lF = args.rows, F // world
    g = torch.Generator(device=dev).manual_seed(rank)
    one = H * lF * 144 // 256
    reps = max(1, -(-(256 << 20) // one))
    wd = [QWeight.random(GgmlType.Q4_K, H, lF, 0.02, g, dev) for _ in range(reps)]
    h = Q8Act(rows, lF, dev)
    ops.rmsnorm_q8(torch.randn(rows, lF, device=dev), None, 1e-5, h, norm=False)
    x = torch.randn(rows, H, device=dev)
    x2 = torch.empty_like(x)
    part = torch.zeros(rows, H, device=dev)
    nw = torch.ones(H, device=dev)
    xa = Q8Act(rows, H, dev)
    tp = TPComm(rank, world, 1, 8, H, dev)

    def local_site(i):
        ops.gemv(wd[i % reps], h, x, residual=True)
        ops.rmsnorm_q8(x, nw, 1e-5, xa)

    def fused_site(i):
        ops.tp_begin(tp)
        ops.gemv_push(wd[i % reps], h, tp, 0)
        ops.tp_allreduce_rmsnorm_q8(tp, 0, x, x2, nw, 1e-5, xa)

    def nccl_site(i):
        ops.gemv(wd[i % reps], h, part)
        dist.all_reduce(part)
        x.add_(part)
        ops.rmsnorm_q8(x, nw, 1e-5, xa)

    res = {}
    for name, fn in (("local", local_site), ("fused", fused_site), ("nccl", nccl_site)):
        us = torch.tensor([_graph_time(fn, args.iters)], device=dev)
        dist.all_reduce(us, op=dist.ReduceOp.MAX)
        res[name] = round(us.item(), 2)
    tp.check()
    link_bytes = (world - 1) * rows * H * 4
    if rank == 0:
        print(json.dumps({"tp_site_us": res, "world": world, "rows": rows, "shape": [H, lF],
                          "weight_bytes": wd[0].nbytes, "nvlink_bytes_out_per_rank": link_bytes,
                          "fused_minus_local_us": round(res["fused"] - res["local"], 2)}))
    tp.close()
    dist.destroy_process_group()


class _View:
    """A TPComm seen through different peer tables (ablations of the step timing)."""

    def __init__(self, tp, consumer_own_slot: bool, push_local_only: bool):
        self._tp, self._own, self._local = tp, consumer_own_slot, push_local_only
        if push_local_only:
            self.push_recv = [t[tp.rank:tp.rank + 1].clone() for t in tp.push_recv]

    def __getattr__(self, k):
        return getattr(self._tp, k)

    @property
    def world(self):
        return 1 if self._own else self._tp.world

    def recv_local(self, site):
        base = self._tp.recv_local(site)
        return base + 8 * self._tp.rank * self._tp.rank_stride if self._own else base


def step_mode(args, rank, world, dev):
    from hawking_b200.engine.engine import Engine
    from hawking_b200.models.config import preset
    from hawking_b200.parallel.tp import TPComm, local_config, random_llama_weights_tp

    cfg = preset("llama3-8b").with_(max_ctx=4096)
    w = random_llama_weights_tp(cfg, rank, world, dev, seed=0)
    tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
    eng = Engine.build(local_config(cfg, world), w, device=dev, max_batch=1, max_ctx=4096, block_size=64,
                       max_rows=8, max_prefill_tokens=8, kv_fraction=0.3, tp=tp)
    m, kv = eng.model, eng.kv
    ctx = 2048
    for l in range(cfg.layers):
        kv.k[l].normal_()
        kv.v[l].normal_()
    if not kv.bm.reserve(7, ctx + 64):
        raise RuntimeError("KV pool too small")
    kv.sync_tables([7])
    res = {}
    for name, own, local in (("tp", False, False), ("own_slot", True, False), ("local_push", True, True)):
        m.tp = _View(tp, own, local) if (own or local) else tp
        m.inp.upload([1], [ctx], [0], [kv.row(7)], [ctx + 1])
        m.release_graphs()
        for _ in range(5):
            m.graph_forward(1, "greedy", advance=False)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            m.graph_forward(1, "greedy", advance=False)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = round(t.item(), 4)
    m.release_graphs()
    m.tp = tp
    tp.check()
    if rank == 0:
        print(json.dumps({"tp_step_ms": res, "world": world, "ctx": ctx, "model": "llama3-8b Q4_K bs1"}))
    tp.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
