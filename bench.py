#!/usr/bin/env python
"""Headline benchmark: decode tok/s at batch 1 (and batch 64) plus p50 TTFT at a 2k prompt, on the
Llama-3-8B-arch GGUF Q4_K configuration, random-init weights, synthetic token ids.

Contract (one JSON line on rank 0):
  python bench.py --gpus N --steps K --warmup W [--impl reference]
For N > 1 launch with torch.distributed.run (one rank per GPU, NCCL); the timed region is bracketed
by a barrier + synchronize on both sides and the step time is the max over ranks.

Timed ("value"): K back-to-back decode steps of B=1 sequence at context 2048, each step one CUDA
graph replay of the whole forward (embedding -> 32 layers -> LM head -> argmax -> device-side
input advance), timed with CUDA events. The 4.6 GB of weights streamed per step exceed the 126 MB
L2, so no flush is needed between steps. "e2e": the same decode through the public Engine.step()
API, including each step's pinned host->device input upload and the device->host read of the
sampled id. TTFT: wall time from Engine.add_request to the first sampled token for a 2048-token
prompt (engine prefill), p50 over runs.
"""
import argparse
import json
import math
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s bs1 & bs64 + p50 TTFT @2k prompt, 8×B200, max over ranks"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "torch"],
                    help="ours | reference (the upstream project, unavailable here) | torch (in-box PyTorch "
                         "cuBLAS + SDPA + NCCL baseline of the same Llama architecture, bf16 weights)")
    ap.add_argument("--model", default="llama3-8b")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--bs64", type=int, default=1, help="also time batch-64 decode (1/0)")
    ap.add_argument("--ttft-runs", type=int, default=3)
    ap.add_argument("--e2e-steps", type=int, default=0, help="0 = same as --steps")
    ap.add_argument("--e2e-ctx", type=int, default=256,
                    help="prompt length of the end-to-end run of the MLA / hybrid models (their prompts prefill in "
                         "8-token chunks / token by token)")
    ap.add_argument("--layers", type=int, default=0, help="override layer count (debug only; invalidates the number)")
    ap.add_argument("--parallel", default="tp", choices=["tp", "dp"],
                    help="N > 1: tensor parallel over the N GPUs (one model, strong scaling) or data-parallel replicas")
    ap.add_argument("--profile-step", action="store_true",
                    help="run one eager decode step between cudaProfilerStart/Stop (for ncu --profile-from-start off) "
                         "and exit without a result line")
    ap.add_argument("--flagships", type=int, default=1,
                    help="also run the DeepSeek-V3-style and Qwen3-Next-style models (sub-objects of the line)")
    ap.add_argument("--artifact", type=int, default=1,
                    help="Qwen3-Next: write the weights as a .gravity artifact and decode from the loaded artifact")
    ap.add_argument("--one-launch", type=int, default=1,
                    help="also time the opt-in persistent decode step (one launch per step), own key")
    ap.add_argument("--w4a8", type=int, default=1,
                    help="also time bs1 decode with the opt-in int8-activation GEMV (reported under its own key)")
    ap.add_argument("--repeats", type=int, default=3,
                    help="extra blocks of K timed steps after the first (median and spread reported beside it)")
    ap.add_argument("--tp-shard-of", type=int, default=0,
                    help="one GPU runs rank 0's shard of an N-way tensor-parallel model with its collectives looped "
                         "back to itself (profiling the shard's kernels under a single-process profiler; not a result)")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="run one --ctx-token prompt prefill through the engine between cudaProfilerStart/Stop "
                         "(after one untimed prefill) and exit without a result line")
    return ap.parse_args()


def reference_unavailable(args):
    line = {"impl": "reference",
            "unavailable": "the reference (joshuahickscorp/hawking) is a Rust+Metal workspace with no Python "
                           "package; pip install of the reference source tree fails (no setup.py/pyproject.toml) and "
                           "Metal does not exist on this box"}
    print(json.dumps(line))


def engine_e2e(eng, vocab: int, prompt_len: int, K: int, W: int, world: int, dev):
    """End-to-end decode through the public Engine API for the MLA / hybrid models: one request
    with a ``prompt_len``-token random prompt (its TTFT is returned too), then K timed
    Engine.step() calls, each uploading the step's inputs from pinned memory and reading the
    sampled id back (max over ranks)."""
    import torch
    import torch.distributed as dist
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.formats.synth import random_prompt
    prompt = random_prompt(prompt_len, vocab, seed=100)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_a = time.perf_counter()
    rid = eng.add_request(prompt, SamplingParams(max_tokens=K + W + 1))
    while not eng.requests[rid].output:
        eng.step()
    ttft = (time.perf_counter() - t_a) * 1000.0
    for _ in range(W):
        eng.step()
    st = eng.stats
    h0, d0 = st.h2d_bytes, st.d2h_bytes
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_e = time.perf_counter()
    n0 = len(eng.requests[rid].output)
    for _ in range(K):
        eng.step()
    torch.cuda.synchronize()
    dt = time.perf_counter() - t_e
    n_tok = len(eng.requests[rid].output) - n0
    if world > 1:
        t = torch.tensor([dt], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = t.item()
    while eng.has_work():
        eng.step()
    return ({"value": round(n_tok / dt, 2), "unit": "tok/s", "h2d_bytes_per_step": (st.h2d_bytes - h0) // max(1, K),
             "d2h_bytes_per_step": (st.d2h_bytes - d0) // max(1, K), "api": "Engine.step()",
             "context": prompt_len}, round(ttft, 2))


def bench_qwen_next(args, sub: bool = False):
    """Qwen3-Next-style hybrid (config 4): bs1 / bs8 device-timed decode, 80B-parameter random
    weights in the mixed <= 1.5 BPW recipe (random codes + Gaussian-statistics scales); on N > 1
    ranks the mixers are tensor parallel over heads and the 512 experts expert parallel
    (parallel/ep.py). ``sub``: return the result as a dict (a sub-object of the default bench
    line) instead of printing it."""
    import torch
    import torch.distributed as dist
    from hawking_b200.engine.kv_cache import PagedKVCache
    from hawking_b200.models.config import preset
    from hawking_b200.models.qwen_next import QwenNextModel, random_qwen_next_weights
    from hawking_b200.utils.clocks import ClockSampler
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    K, W, ctx = args.steps, args.warmup, args.ctx
    cfg = preset("qwen3-next", max_ctx=max(ctx, args.e2e_ctx) + 2 * (K + W) + 64)
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    t0 = time.time()
    tp = None
    mcfg = cfg
    if world > 1:
        from hawking_b200.parallel.ep import local_qwen_next_config
        from hawking_b200.parallel.tp import TPComm
        w = random_qwen_next_weights(cfg, dev, seed=0, shard=(rank, world))
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        mcfg = local_qwen_next_config(cfg, world)
    else:
        w = random_qwen_next_weights(cfg, dev, seed=0)
    t_load = time.time() - t0
    artifact = None
    if args.artifact and world == 1:
        # through a `.gravity` artifact: written with the repo's writer, read back (every payload's
        # sha256 verified once at admission) and decoded from the loaded planes
        import shutil
        import tempfile
        from hawking_b200.models import qwen_next_artifact as qa
        d = tempfile.mkdtemp(prefix="hk-qn-artifact-")
        try:
            t1 = time.time()
            idx = qa.save(d, cfg, w)
            t2 = time.time()
            del w
            torch.cuda.empty_cache()
            cfg2, w = qa.load(d, dev, verify=True)
            t3 = time.time()
            artifact = {"shards": len(set(idx["weight_map"].values())), "tensors": len(idx["weight_map"]),
                        "bytes": sum(os.path.getsize(os.path.join(d, f)) for f in os.listdir(d)),
                        "write_s": round(t2 - t1, 1), "load_verify_s": round(t3 - t2, 1)}
        finally:
            shutil.rmtree(d, ignore_errors=True)
    n_full = sum(cfg.layer_is_full_attention(l) for l in range(cfg.layers))
    bs, max_seqs = 64, 8
    max_blocks = -(-cfg.max_ctx // bs)
    kv = PagedKVCache(n_full, mcfg.n_kv_heads, cfg.head_dim, max_seqs * max_blocks + 8, bs, max_seqs, max_blocks, dev,
                      prefix_cache=False)
    m = QwenNextModel(mcfg, w, kv, max_rows=2048, max_seqs=max_seqs, device=dev, tp=tp)
    g = torch.Generator(device=dev).manual_seed(1 + rank)
    for l in range(n_full):
        kv.k[l].normal_(0, 1, generator=g)
        kv.v[l].normal_(0, 1, generator=g)
    m.ssm_state.normal_(0, 0.05, generator=g)
    m.conv_state.normal_(0, 0.5, generator=g)
    elements = sum(t.N * t.K for t in w.table.weights) + w.embed.N * w.embed.K
    complete_bpw = (w.table.nbytes + w.embed.nbytes) * 8.0 / elements
    expert_bytes = sum(t.nbytes for t in w.table.weights if t.N * t.K == cfg.expert_ffn * cfg.hidden)

    def timed(nseq):
        ids, pos, rseq, rctx = [], [], [], []
        for i in range(nseq):
            sid = 10 + i
            kv.bm.reserve(sid, ctx + K + W + 8)
            kv.sync_tables([sid])
            ids.append(int(torch.randint(0, cfg.vocab, (1,)).item()))
            pos.append(ctx)
            rseq.append(kv.row(sid))
            rctx.append(ctx + 1)
        if world > 1:  # every rank decodes the same token ids (the hidden state is replicated)
            t = torch.tensor(ids, dtype=torch.int32, device=dev)
            dist.broadcast(t, 0)
            ids = t.tolist()
        m.inp.upload(ids, pos, [0] * nseq, rseq, rctx)
        for _ in range(W):
            m.graph_forward(nseq, "greedy", advance=True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local, period_ms=50) as cs:
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(K):
                m.graph_forward(nseq, "greedy", advance=True)
            e1.record()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for i in range(nseq):
            kv.drop(10 + i)
        ms = e0.elapsed_time(e1) / K
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms, cs.result

    if args.profile_step:
        profile_one_step(m, kv, ctx)
        return 0
    ms1, clocks = timed(1)
    launches = m.launches_per_graph
    ms8, clocks8 = timed(8)
    from hawking_b200.engine.engine import Engine
    eng = Engine(mcfg, m, kv, max_batch=max_seqs - 1, max_prefill_tokens=m.row_limit)
    e2e, ttft = engine_e2e(eng, cfg.vocab, args.e2e_ctx, K, W, world, dev)
    if tp is not None:
        tp.check()
        m.release_graphs()
        tp.close()
    out = {
        "metric": "decode tok/s bs1 (Qwen3-Next-style hybrid MoE, .gravity mixed <= 1.5 BPW), %d GPU" % world,
        "value": round(1000.0 / ms1, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms1, 4), "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "binary/ternary experts and Q4 projections (per-64 fp16 group scales) x int8 activation blocks, "
                 "fp32 accumulate and DeltaNet state, bf16 KV",
        "data": "synthetic: random codes with Gaussian-statistics group scales (80B-parameter model), random KV "
                "and recurrent state for a %d-token context, uniform-random token ids" % ctx,
        "config": {"model": "qwen3-next (48 layers, hidden 2048, 12 gated full-attention layers 16/2 heads hd 256, "
                            "36 gated DeltaNet layers 16k/32v heads hd 128, 512 experts top-10 + shared, FFN 512, "
                            "vocab 151936)" + (f" [LAYERS OVERRIDDEN to {cfg.layers}]" if args.layers else ""),
                   "global_batch": 1, "seq_len": ctx,
                   "parallelism": "tp1" if world == 1 else "tp%d mixers + ep%d experts" % (world, world),
                   "complete_bpw": round(complete_bpw, 3),
                   "l2": "inputs larger than L2: %.1f GB of weights resident per GPU" % ((w.table.nbytes + w.embed.nbytes) / 1e9)},
        "clocks": clocks, "e2e": e2e, "ttft_ms": ttft, "ttft_prompt": args.e2e_ctx,
        "ttft_note": "prompts prefill in forwards of up to %d rows (the DeltaNet kernels walk a run token by token, state in registers; no chunked WY form)" % m.row_limit,
        "gpu_launches": launches * K,
        "bs8": {"tok_s_aggregate": round(8 * 1000.0 / ms8, 1), "ms_per_step": round(ms8, 4), "clocks": clocks8},
        "weights_gb": round((w.table.nbytes + w.embed.nbytes) / 1e9, 2),
        "expert_weights_gb": round(expert_bytes / 1e9, 2), "load_s": round(t_load, 1),
        "artifact": artifact or ("in-memory weights (--artifact 0)" if world == 1 else "in-memory shards (N > 1)"),
    }
    if sub:
        m.release_graphs()
        return out
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def profile_one_step(m, kv, ctx):
    """One eager bs1 decode step between cudaProfilerStart/Stop (after warm-up), for
    ``ncu --profile-from-start off``."""
    import torch
    kv.bm.reserve(10, ctx + 16)
    kv.sync_tables([10])
    m.inp.upload([1], [ctx], [0], [kv.row(10)], [ctx + 1])
    for _ in range(3):
        m.forward(1, "greedy")
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStart()
    m.forward(1, "greedy")
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    print(json.dumps({"profile_step": True}))


def bench_deepseek(args, sub: bool = False):
    """DeepSeek-V3-style MLA + MoE (config 5): bs1 / bs8 device-timed decode with random-init fp8
    e4m3 (128 x 128 block-scaled) weights of the full 43-layer architecture; on N > 1 ranks the
    model is tensor parallel over heads and expert parallel over the 256 experts (parallel/ep.py).
    ``sub``: run inside the default bench (process group already up; return a dict)."""
    import torch
    import torch.distributed as dist
    from hawking_b200.models.config import preset
    from hawking_b200.models.deepseek import DeepSeekModel, LatentCache, random_deepseek_weights
    from hawking_b200.utils.clocks import ClockSampler
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1 and not dist.is_initialized():
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    K, W, ctx = args.steps, args.warmup, args.ctx
    cfg = preset("deepseek-v3", max_ctx=max(ctx, args.e2e_ctx) + 2 * (K + W) + 64)
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    t0 = time.time()
    tp = None
    if world > 1:
        from hawking_b200.parallel.ep import local_deepseek_config, random_deepseek_weights_ep
        from hawking_b200.parallel.tp import TPComm
        w = random_deepseek_weights_ep(cfg, rank, world, dev, seed=0)
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        mcfg = local_deepseek_config(cfg, world)
    else:
        w = random_deepseek_weights(cfg, dev, seed=0)
        mcfg = cfg
    t_load = time.time() - t0
    bs, max_seqs = 64, 8
    max_blocks = -(-cfg.max_ctx // bs)
    kv = LatentCache(cfg.layers, max_seqs * max_blocks + 8, bs, max_seqs, max_blocks, dev)
    m = DeepSeekModel(mcfg, w, kv, max_rows=2048, device=dev, tp=tp)
    g = torch.Generator(device=dev).manual_seed(1)
    for lat in kv.latent:
        lat.normal_(0, 1, generator=g)

    def timed(nseq):
        ids, pos, rseq, rctx = [], [], [], []
        for i in range(nseq):
            sid = 10 + i
            kv.bm.reserve(sid, ctx + K + W + 8)
            kv.sync_tables([sid])
            ids.append(int(torch.randint(0, cfg.vocab, (1,)).item()))
            pos.append(ctx)
            rseq.append(kv.row(sid))
            rctx.append(ctx + 1)
        if world > 1:  # every rank decodes the same token ids (the hidden state is replicated)
            t = torch.tensor(ids, dtype=torch.int32, device=dev)
            dist.broadcast(t, 0)
            ids = t.tolist()
        m.inp.upload(ids, pos, [0] * nseq, rseq, rctx)
        for _ in range(W):
            m.graph_forward(nseq, "greedy", advance=True)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local, period_ms=50) as cs:
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(K):
                m.graph_forward(nseq, "greedy", advance=True)
            e1.record()
            torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        for i in range(nseq):
            kv.drop(10 + i)
        ms = e0.elapsed_time(e1) / K
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = t.item()
        return ms, cs.result

    if args.profile_step:
        profile_one_step(m, kv, ctx)
        return 0
    ms1, clocks = timed(1)
    launches = m.launches_per_graph
    ms8, clocks8 = timed(8)
    from hawking_b200.engine.engine import Engine
    eng = Engine(mcfg, m, kv, max_batch=8, max_prefill_tokens=m.row_limit)
    e2e, ttft = engine_e2e(eng, cfg.vocab, args.e2e_ctx, K, W, world, dev)
    if tp is not None:
        tp.check()
        m._graphs.clear()
        tp.close()
    out = {
        "metric": "decode tok/s bs1 (DeepSeek-V3-style MLA + MoE, fp8 e4m3 block-scaled), %d GPU" % world,
        "value": round(1000.0 / ms1, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms1, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp8 e4m3 weights with 128x128 fp32 block scales x int8 activation blocks, fp32 accumulate, "
                 "bf16 latent cache, bf16 W_UK/W_UV",
        "data": "synthetic: random-init N(0,0.02) weights quantised to fp8 on device, random latent cache for a "
                "%d-token context, uniform-random token ids" % ctx,
        "config": {"model": "deepseek-v3-style (%d layers, hidden 4096, 64 heads, q_lora 1024, kv_lora 512, rope 64, "
                            "nope 128, v 128, 256 experts top-8 sigmoid+bias group-limited, 1 shared, expert FFN 1024, "
                            "3 dense layers FFN 11264, vocab 129280)" % cfg.layers,
                   "global_batch": 1, "seq_len": ctx,
                   "parallelism": "tp1" if world == 1 else "tp%d attention + ep%d experts" % (world, world),
                   "l2": "inputs larger than L2: %.1f GB of weights resident per GPU" % (w.nbytes / 1e9)},
        "clocks": clocks, "e2e": e2e,
        "ttft_ms": ttft, "ttft_prompt": args.e2e_ctx,
        "gpu_launches": launches * K,
        "bs8": {"tok_s_aggregate": round(8 * 1000.0 / ms8, 1), "ms_per_step": round(ms8, 4), "clocks": clocks8},
        "weights_gb": round(w.nbytes / 1e9, 2), "load_s": round(t_load, 1),
    }
    if sub:
        m._graphs.clear()
        return out
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def bench_torch(args):
    """In-box library baseline (``--impl torch``): the same Llama-3-8B architecture and workload in
    plain PyTorch (bf16 weights, cuBLAS, SDPA, NCCL tensor parallelism), CUDA-graph decode."""
    import datetime
    import statistics

    import torch
    import torch.distributed as dist
    from hawking_b200.models.config import preset
    from hawking_b200.utils.clocks import ClockSampler
    from hawking_b200.utils.torch_baseline import TorchLlamaTP

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    cfg = preset(args.model)
    B, ctx, K, W = args.batch, args.ctx, args.steps, args.warmup
    cap = ctx + W + 2 * K + 16  # warm-up, timed and end-to-end steps each advance every position

    def barrier():
        if world > 1:
            dist.barrier()

    def max_ranks(v):
        if world > 1:
            t = torch.tensor([v], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return t.item()
        return v

    def timed(nb):
        m = TorchLlamaTP(cfg, rank, world, dev, nb, cap)
        g = torch.Generator(device=dev).manual_seed(1)
        for t in m.k + m.v:
            t.normal_(0, 1, generator=g)
        m.pos.fill_(ctx)
        m.ids.random_(0, cfg.vocab, generator=g)
        for _ in range(W):
            m.decode_step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local, period_ms=50) as cs:
            barrier()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(K):
                m.decode_step()
            e1.record()
            torch.cuda.synchronize()
        ms = max_ranks(e0.elapsed_time(e1) / K)
        # end to end: per step the ids go up from pinned memory and the next ids come back
        host_in = torch.zeros(nb, dtype=torch.long).pin_memory()
        host_out = torch.zeros(nb, dtype=torch.long).pin_memory()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(K):
            m.ids.copy_(host_in, non_blocking=True)
            m.decode_step()
            host_out.copy_(m.next_ids, non_blocking=True)
            torch.cuda.current_stream().synchronize()
            host_in.copy_(host_out)
        dt = max_ranks(time.perf_counter() - t0)
        nbytes = m.nbytes
        m.release()
        del m
        torch.cuda.empty_cache()
        return ms, cs.result, nb * K / dt, nbytes

    ms1, clocks, e2e1, wbytes = timed(B)
    ms64, clocks64, _, _ = timed(64) if args.bs64 and B != 64 else (None, None, None, None)
    # TTFT: eager prefill of a ctx-token prompt, next id read back to the host
    m = TorchLlamaTP(cfg, rank, world, dev, 1, ctx + 8)
    ttfts = []
    for run in range(max(1, args.ttft_runs) + 1):
        prompt = torch.randint(0, cfg.vocab, (1, ctx), generator=torch.Generator().manual_seed(100 + run))
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        nxt = m.prefill(prompt.to(dev, non_blocking=True))
        int(nxt[0].item())
        dt = max_ranks(time.perf_counter() - t0)
        if run:  # the first run warms up the kernels
            ttfts.append(dt * 1000.0)
    out = {
        "impl": "torch",
        "metric": METRIC,
        "value": round(B * 1000.0 / ms1, 2), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(ms1, 4), "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16 weights and activations, fp32 softmax",
        "data": "synthetic: random-init N(0,0.02) bf16 weights, random bf16 KV for a %d-token context, "
                "uniform-random token ids" % ctx,
        "config": {"model": "llama3-8b architecture, bf16 weights (no Q4_K kernel in PyTorch)",
                   "global_batch": B, "seq_len": ctx, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2: %.2f GB of weights per step per GPU" % (wbytes / 1e9),
                   "attention": "decode: masked grouped-query batched GEMMs over a %d-slot cache; prefill: "
                                "SDPA causal" % cap},
        "clocks": clocks,
        "e2e": {"value": round(e2e1, 2), "unit": "tok/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 8 * B,
                "api": "TorchLlamaTP.decode_step()"},
        "gpu_launches": None,
        "bs64": {"tok_s_aggregate": round(64 * 1000.0 / ms64, 1), "ms_per_step": round(ms64, 4),
                 "clocks": clocks64} if ms64 else None,
        "ttft_p50_ms": round(statistics.median(ttfts), 2),
        "ttft_runs_ms": [round(t, 2) for t in ttfts],
    }
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            reference_unavailable(args)
        return 0
    if args.impl == "torch":
        return bench_torch(args)
    if args.model == "qwen3-next":
        return bench_qwen_next(args)
    if args.model == "deepseek-v3":
        return bench_deepseek(args)

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)

    from hawking_b200 import ops
    from hawking_b200.engine.engine import Engine
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.formats.synth import random_prompt
    from hawking_b200.models.config import preset
    from hawking_b200.models.llama import random_llama_weights
    from hawking_b200.utils.clocks import ClockSampler

    cfg = preset(args.model)
    if args.layers:
        cfg = cfg.with_(layers=args.layers)
    B, ctx, K, W = args.batch, args.ctx, args.steps, args.warmup
    max_ctx = ctx + 2 * (K + W) + 256
    cfg = cfg.with_(max_ctx=max_ctx)
    use_tp = world > 1 and args.parallel == "tp"
    t0 = time.time()
    tp = None
    if use_tp or args.tp_shard_of > 1:
        from hawking_b200.parallel.tp import TPComm, local_config, random_llama_weights_tp
        shards = args.tp_shard_of if world == 1 else world
        w = random_llama_weights_tp(cfg, rank, shards, dev, seed=0)
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        mcfg = local_config(cfg, shards)
    else:
        w = random_llama_weights(cfg, dev, seed=0)
        mcfg = cfg
    t_load = time.time() - t0
    max_batch = max(B, 64 if args.bs64 else B)
    eng = Engine.build(mcfg, w, device=dev, max_batch=max_batch, max_ctx=max_ctx, block_size=64, max_rows=64,
                       max_prefill_tokens=2048, kv_fraction=0.6, tp=tp)
    # aggregate over the job: data-parallel replicas each decode their own batch; a tensor-parallel
    # group decodes one batch together
    replicas = 1 if use_tp else world
    m, kv = eng.model, eng.kv

    def barrier():
        if world > 1:
            dist.barrier()

    def setup_decode(nseq, first_id):
        """nseq sequences holding `ctx` tokens of (random) KV, positioned for decode."""
        ids, pos, rseq, rctx = [], [], [], []
        for i in range(nseq):
            sid = first_id + i
            if not kv.bm.reserve(sid, ctx + K + W + 8):
                raise RuntimeError("KV pool too small for the benchmark")
            kv.sync_tables([sid])
            ids.append(int(torch.randint(0, cfg.vocab, (1,)).item()))
            pos.append(ctx)
            rseq.append(kv.row(sid))
            rctx.append(ctx + 1)
        m.inp.upload(ids, pos, [0] * nseq, rseq, rctx)
        return [first_id + i for i in range(nseq)]

    def timed_decode(nseq, repeats=0):
        """W warm-up steps, then the timed block of exactly K steps (barrier + synchronize on both
        sides, CUDA events, max over ranks); then ``repeats`` more blocks of K steps, reported
        separately. Clocks are sampled across all blocks."""
        for _ in range(W):
            m.graph_forward(nseq, "greedy", advance=True)
        torch.cuda.synchronize()
        blocks = []
        with ClockSampler(local, period_ms=50) as cs:
            for _b in range(1 + repeats):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                # the barrier comes after every rank's sampler is up, so all ranks start together
                barrier()
                torch.cuda.synchronize()
                e0.record()
                for _ in range(K):
                    m.graph_forward(nseq, "greedy", advance=True)
                e1.record()
                torch.cuda.synchronize()
                barrier()
                ms = e0.elapsed_time(e1) / K
                if world > 1:
                    t = torch.tensor([ms], device=dev)
                    dist.all_reduce(t, op=dist.ReduceOp.MAX)
                    ms = t.item()
                blocks.append(ms)
        return blocks[0], cs.result, blocks[1:]

    # Random KV content for the context (decode work does not depend on the values).
    g = torch.Generator(device=dev).manual_seed(1)
    for l in range(cfg.layers):
        kv.k[l].normal_(0, 1, generator=g)
        kv.v[l].normal_(0, 1, generator=g)

    if args.profile_prefill:
        for run in range(2):
            prompt = random_prompt(ctx, cfg.vocab, seed=100 + run)
            torch.cuda.synchronize()
            if run:
                torch.cuda.cudart().cudaProfilerStart()
            rid = eng.add_request(prompt, SamplingParams(max_tokens=1))
            while eng.has_work():
                eng.step()
            torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        print(json.dumps({"profile_prefill": True, "prompt": ctx}))
        return 0

    # ---- bs1 (or --batch) device-timed decode ----
    seqs = setup_decode(B, 1_000_000)
    if args.profile_step:
        for _ in range(W):
            m.forward(B, "greedy")
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStart()
        m.forward(B, "greedy")
        torch.cuda.synchronize()
        torch.cuda.cudart().cudaProfilerStop()
        print(json.dumps({"profile_step": True, "launches": m.launches_per_forward}))
        return 0
    ms1, clocks, rep1 = timed_decode(B, args.repeats)
    launches = m.launches_per_graph
    for s in seqs:
        kv.drop(s)
    result_w4a8 = None
    if args.w4a8 and m.small_batch == "w4a16":
        # the opt-in int8-activation GEMV, same workload, reported under its own key
        m.release_graphs()
        m.small_batch = "w4a8"
        seqs = setup_decode(B, 3_000_000)
        ms8a, clocks8a, _ = timed_decode(B)
        result_w4a8 = {"tok_s": round(B * 1000.0 / ms8a, 2), "ms_per_step": round(ms8a, 4), "clocks": clocks8a,
                       "dtype": "q4_k weights x int8 activation blocks of 32 (dp4a), fp32 accumulate (opt-in: "
                                "HK_SMALL_BATCH=w4a8)"}
        for s in seqs:
            kv.drop(s)
        m.release_graphs()
        m.small_batch = "w4a16"
    result_one_launch = None
    if args.one_launch and getattr(m, "dstep", None) is None and m.tp is None and B <= 4:
        # the opt-in persistent decode step (every layer + LM head in one launch), same workload,
        # reported under its own key
        from hawking_b200.ops.dstep import DecodeStep
        ds = DecodeStep.build(m)
        if ds is None:
            result_one_launch = {"unavailable": "model or shapes outside the persistent decode step"}
        else:
            m.release_graphs()
            m.dstep = ds
            seqs = setup_decode(B, 4_000_000)
            msd, clocksd, _ = timed_decode(B)
            result_one_launch = {"tok_s": round(B * 1000.0 / msd, 2), "ms_per_step": round(msd, 4),
                                 "clocks": clocksd, "launches_per_step": m.launches_per_graph,
                                 "note": "opt-in (HK_DSTEP=1): slower than the default per-kernel path so far"}
            for s_ in seqs:
                kv.drop(s_)
            m.release_graphs()
            m.dstep = None
    result_bs64 = None
    if args.bs64 and B != 64 and m.row_limit < 64:
        # tensor parallel without the tensor-core path (MoE layers): the push all-reduce sites
        # hold 8 rows per forward
        result_bs64 = {"unavailable": "batch 64 under tensor/expert parallelism needs the tensor-core path, "
                                      "which MoE layers do not have yet (forwards of <= 8 rows only)"}
    elif args.bs64 and B != 64:
        seqs = setup_decode(64, 2_000_000)
        ms64, clocks64, _ = timed_decode(64)
        result_bs64 = {"tok_s_aggregate": round(64 * 1000.0 / ms64 * replicas, 1), "ms_per_step": round(ms64, 4),
                       "clocks": clocks64}
        for s in seqs:
            kv.drop(s)
    m.release_graphs()

    # ---- TTFT @ctx prompt and e2e decode through the public API ----
    ttfts = []
    e2e = None
    KE = args.e2e_steps or K
    for run in range(max(1, args.ttft_runs)):
        prompt = random_prompt(ctx, cfg.vocab, seed=100 + run)
        torch.cuda.synchronize()
        barrier()
        t_a = time.perf_counter()
        rid = eng.add_request(prompt, SamplingParams(max_tokens=KE + W + 1 if run == 0 else 1))
        while not eng.requests[rid].output:
            eng.step()
        ttfts.append((time.perf_counter() - t_a) * 1000.0)
        if run == 0:
            for _ in range(W):
                eng.step()
            st = eng.stats
            h0, d0 = st.h2d_bytes, st.d2h_bytes
            torch.cuda.synchronize()
            barrier()
            t_e = time.perf_counter()
            n0 = len(eng.requests[rid].output)
            for _ in range(KE):
                eng.step()
            torch.cuda.synchronize()
            dt = time.perf_counter() - t_e
            n_tok = len(eng.requests[rid].output) - n0
            if world > 1:
                t = torch.tensor([dt], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                dt = t.item()
            e2e = {"value": round(n_tok * replicas / dt, 2), "unit": "tok/s",
                   "h2d_bytes_per_step": (st.h2d_bytes - h0) // max(1, KE),
                   "d2h_bytes_per_step": (st.d2h_bytes - d0) // max(1, KE),
                   "api": "Engine.step()"}
        while eng.has_work():
            eng.step()
    ttft_p50 = statistics.median(ttfts)

    value = B * 1000.0 / ms1 * replicas
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms1, 4),
        "higher_is_better": True,
        "scaling": "strong" if args.parallel == "tp" else "weak",
        "vs_baseline": None,
        "dtype": (f"{cfg.weight_type.lower()} weights, bf16 activations (W4A16 tensor-core GEMV), fp32 accumulate, "
                  "bf16 KV" if m.small_batch == "w4a16" and args.model == "llama3-8b" else
                  f"{cfg.weight_type.lower()} weights, int8 activation blocks (dp4a GEMV), fp32 accumulate, bf16 KV"),
        "data": f"synthetic: random-init N(0,0.02) weights quantised to GGUF {cfg.weight_type} on device; "
                "uniform-random token ids; device-timed decode runs over a 2048-token KV context filled with "
                "random bf16",
        "config": {"model": (("llama3-8b (Llama-3-8B-arch: 32 layers, hidden 4096, 32/8 GQA heads, head_dim 128, "
                              "FFN 14336, vocab 128256, rope theta 5e5, GGUF Q4_K)") if args.model == "llama3-8b" else
                             f"{args.model} ({cfg.layers} layers, hidden {cfg.hidden}, {cfg.n_heads}/{cfg.n_kv_heads} "
                             f"GQA heads, {cfg.n_experts} experts top-{cfg.top_k}, expert FFN {cfg.expert_ffn}, "
                             f"vocab {cfg.vocab}, GGUF {cfg.weight_type})") + (
                                f" [LAYERS OVERRIDDEN to {cfg.layers}]" if args.layers else ""),
                   "global_batch": B * replicas, "seq_len": ctx,
                   "parallelism": f"tp{world}" if use_tp else (f"dp{world}" if world > 1 else "tp1"),
                   "l2": "inputs larger than L2: %.2f GB of weights streamed per step per GPU" % (w.nbytes / 1e9),
                   "kv_block_size": 64},
        "clocks": clocks,
        "e2e": e2e,
        "gpu_launches": launches * K,
        "bs64": result_bs64,
        "repeat_blocks_ms_per_step": [round(v, 4) for v in rep1],
        "w4a8_opt_in": result_w4a8,
        "one_launch_step": result_one_launch,
        "ttft_p50_ms": round(ttft_p50, 2),
        "ttft_runs_ms": [round(t, 2) for t in ttfts],
        "weights_gb": round(w.nbytes / 1e9, 3),
        "weight_bw_gbs": round(w.nbytes / (ms1 * 1e-3) / 1e9, 1),
        "load_s": round(t_load, 1),
    }
    if args.tp_shard_of > 1 and world == 1:
        out["invalid"] = f"one GPU ran rank 0's shard of a {args.tp_shard_of}-way TP model, collectives looped back"
    if tp is not None:
        tp.check()
        out["tp_collectives"] = "decode (<= 8 rows): GEMV epilogue pushes partials over NVLink + fused " \
                                "all-reduce/RMSNorm; prefill and bs64 (tensor-core path): NCCL all-reduce"
    # free the Llama model before the checks and flagship models below
    m.release_graphs()
    if tp is not None:
        tp.close()
    del eng, m, kv, w
    import gc
    gc.collect()
    torch.cuda.empty_cache()
    barrier()
    if use_tp and not args.layers:
        out["tokens_match_tp1"], out["tokens_agree_prefix"] = tp_token_check(args, world, rank, dev)
    if args.flagships and not args.layers and args.tp_shard_of <= 1:
        import copy
        fa = copy.copy(args)
        fa.e2e_ctx = 2048  # TTFT at a 2k prompt
        out["deepseek_v3"] = bench_deepseek(fa, sub=True)
        gc.collect()
        torch.cuda.empty_cache()
        barrier()
        out["qwen3_next"] = bench_qwen_next(fa, sub=True)
        gc.collect()
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def tp_token_check(args, world, rank, dev):
    """The first 16 greedy ids of a 2-layer model of the bench's architecture (same seed) under
    N-way tensor parallelism against a one-GPU run on rank 0. Returns (match, agreeing prefix)."""
    import torch
    import torch.distributed as dist
    from hawking_b200.engine.engine import Engine
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.formats.synth import random_prompt
    from hawking_b200.models.config import preset
    from hawking_b200.models.llama import random_llama_weights
    from hawking_b200.parallel.tp import TPComm, local_config, shard_llama_weights
    cfg = preset(args.model).with_(layers=2, max_ctx=512)
    w = random_llama_weights(cfg, dev, seed=11)  # identical on every rank
    prompt = random_prompt(24, cfg.vocab, seed=12)
    sp = SamplingParams(max_tokens=16)
    ref = []
    if rank == 0:
        e1 = Engine.build(cfg, w, device=dev, max_batch=1, max_ctx=512, block_size=64, max_rows=8,
                          max_prefill_tokens=64, num_blocks=16)
        ref = e1.generate([prompt], sp)[0]
        e1.model.release_graphs()
        del e1
    dist.barrier()
    tpc = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
    e2 = Engine.build(local_config(cfg, world), shard_llama_weights(w, cfg, rank, world), device=dev, max_batch=1,
                      max_ctx=512, block_size=64, max_rows=8, max_prefill_tokens=64, num_blocks=16, tp=tpc)
    got = e2.generate([prompt], sp)[0]
    tpc.check()
    e2.model.release_graphs()
    tpc.close()
    del e2, w
    torch.cuda.empty_cache()
    dist.barrier()
    n = 0
    while n < min(len(got), len(ref)) and got[n] == ref[n]:
        n += 1
    return (got == ref) if rank == 0 else None, n if rank == 0 else None


if __name__ == "__main__":
    sys.exit(main())
