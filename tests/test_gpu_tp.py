"""Tensor parallelism on 2 GPUs (one process per GPU, NCCL plumbing): the fused push all-reduce
and vocabulary-parallel greedy give the TP=1 logits and tokens.

Runs only where at least two GPUs are visible."""
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, gguf, out_path):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from hawking_b200.engine.engine import Engine
        from hawking_b200.engine.sampling import SamplingParams
        from hawking_b200.formats.gguf import GgufModel
        from hawking_b200.models.llama import load_llama_weights
        from hawking_b200.models.torch_ref import config_from_gguf
        from hawking_b200.parallel.tp import TPComm, local_config, shard_llama_weights
        m = GgufModel(gguf)
        cfg = config_from_gguf(m).with_(max_ctx=128)
        w = load_llama_weights(m, cfg, dev)
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        eng = Engine.build(local_config(cfg, world), shard_llama_weights(w, cfg, rank, world), device=dev,
                           max_batch=2, max_ctx=128, block_size=16, num_blocks=64, max_rows=8, tp=tp)
        toks = list(range(10, 22))
        local = eng.model.forward_tokens(toks, seq_id=1)
        eng.kv.drop(1)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        full = torch.cat(parts, 1)
        gen = eng.generate([list(range(30, 40))], SamplingParams(max_tokens=6))[0]
        gens = [None] * world
        dist.all_gather_object(gens, gen)
        tp.check()
        if rank == 0:
            ref = Engine.build(cfg, w, device=dev, max_batch=2, max_ctx=128, block_size=16, num_blocks=64, max_rows=8)
            ref_logits = ref.model.forward_tokens(toks, seq_id=1)
            ref_gen = ref.generate([list(range(30, 40))], SamplingParams(max_tokens=6))[0]
            err = float((full - ref_logits).abs().max() / ref_logits.abs().max())
            agree = float((full.argmax(1) == ref_logits.argmax(1)).float().mean())
            torch.save({"err": err, "agree": agree, "gens": gens, "ref_gen": ref_gen}, out_path)
        torch.cuda.synchronize()
        tp.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_tp1(tiny_gguf, tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "tp.pt")
    mp.spawn(_worker, args=(2, _free_port(), tiny_gguf, out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["err"] < 0.03, r
    assert r["agree"] >= 0.9, r
    assert r["gens"][0] == r["gens"][1]  # every rank decodes the same tokens
    assert r["gens"][0][0] == r["ref_gen"][0]


def _moe_worker(rank, world, port, shared, out_path):
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from hawking_b200.engine.engine import Engine
        from hawking_b200.models.config import ModelConfig
        from hawking_b200.models.llama import random_llama_weights
        from hawking_b200.parallel.tp import TPComm, local_config, shard_llama_weights
        cfg = ModelConfig(arch="mixtral", vocab=1024, hidden=512, layers=2, n_heads=8, n_kv_heads=2, head_dim=64,
                          ffn=1024, n_experts=4, top_k=2, expert_ffn=512, weight_type="Q8_0", max_ctx=128)
        if shared:  # Qwen-MoE style: a sigmoid-gated shared expert next to the routed ones
            cfg = cfg.with_(shared_ffn=256, shared_gate=True, n_shared_experts=1, norm_topk=True)
        w = random_llama_weights(cfg, dev, seed=4, std=0.05)  # same seed: identical on every rank
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        eng = Engine.build(local_config(cfg, world), shard_llama_weights(w, cfg, rank, world), device=dev,
                           max_batch=2, max_ctx=128, block_size=16, num_blocks=64, max_rows=8, tp=tp)
        toks = list(range(10, 22))
        local = eng.model.forward_tokens(toks, seq_id=1)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        full = torch.cat(parts, 1)
        tp.check()
        if rank == 0:
            ref = Engine.build(cfg, w, device=dev, max_batch=2, max_ctx=128, block_size=16, num_blocks=64, max_rows=8)
            ref.model.long_runs = False
            ref_logits = torch.cat([ref.model.forward_tokens(toks[:8], seq_id=1),
                                    ref.model.forward_tokens(toks[8:], seq_id=1, start_pos=8)])
            err = float((full - ref_logits).abs().max() / ref_logits.abs().max())
            torch.save({"err": err}, out_path)
        torch.cuda.synchronize()
        tp.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("shared", [False, True])
def test_tp2_expert_parallel_moe_matches_tp1(shared, tmp_path):
    """Mixtral-style MoE (and a gated shared expert) with TP attention and experts split 2 + 2."""
    import torch.multiprocessing as mp
    out = str(tmp_path / "moe.pt")
    mp.spawn(_moe_worker, args=(2, _free_port(), shared, out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["err"] < 0.03, r


def _dense_q4k_worker(rank, world, port, math, out_path):
    """Q4_K dense Llama shape: the decode path runs the W4A16 GEMV with its push epilogue."""
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["HK_MG_MATH"] = math
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from hawking_b200.engine.engine import Engine
        from hawking_b200.engine.sampling import SamplingParams
        from hawking_b200.models.config import preset
        from hawking_b200.models.llama import random_llama_weights
        from hawking_b200.parallel.tp import TPComm, local_config, shard_llama_weights
        cfg = preset("llama3-8b", layers=2, hidden=1024, n_heads=8, n_kv_heads=2, ffn=2048, vocab=2048, max_ctx=128)
        w = random_llama_weights(cfg, dev, seed=5, std=0.05)  # same seed: identical on every rank
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        eng = Engine.build(local_config(cfg, world), shard_llama_weights(w, cfg, rank, world), device=dev,
                           max_batch=4, max_ctx=128, block_size=16, num_blocks=64, max_rows=8, tp=tp)
        assert eng.model._mg_layer(eng.model.w.layers[0])
        toks = list(range(10, 16))  # <= 8 rows: the GEMV path with the push all-reduce
        local = eng.model.forward_tokens(toks, seq_id=1)
        eng.kv.drop(1)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        full = torch.cat(parts, 1)
        gen = eng.generate([list(range(30, 40)), list(range(50, 53))], SamplingParams(max_tokens=5))
        gens = [None] * world
        dist.all_gather_object(gens, gen)
        tp.check()
        if rank == 0:
            ref = Engine.build(cfg, w, device=dev, max_batch=4, max_ctx=128, block_size=16, num_blocks=64,
                               max_rows=8)
            ref_logits = ref.model.forward_tokens(toks, seq_id=1)
            ref.kv.drop(1)
            ref_gen = ref.generate([list(range(30, 40)), list(range(50, 53))], SamplingParams(max_tokens=5))
            err = float((full - ref_logits).abs().max() / ref_logits.abs().max())
            torch.save({"err": err, "gens": gens, "ref_gen": ref_gen}, out_path)
        torch.cuda.synchronize()
        tp.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("math", ["int", "bf16"])
def test_tp2_q4k_w4a16_push_matches_tp1(math, tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "dense.pt")
    mp.spawn(_dense_q4k_worker, args=(2, _free_port(), math, out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["err"] < 0.01, r
    assert r["gens"][0] == r["gens"][1]  # every rank decodes the same tokens
    assert [g[0] for g in r["gens"][0]] == [g[0] for g in r["ref_gen"]], r


def _sampling_worker(rank, world, port, out_path):
    """Non-greedy decode under tensor parallelism: gathered vocabulary slices, same uniforms."""
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from hawking_b200.engine.engine import Engine
        from hawking_b200.engine.sampling import SamplingParams
        from hawking_b200.models.config import preset
        from hawking_b200.models.llama import random_llama_weights
        from hawking_b200.parallel.tp import TPComm, local_config, shard_llama_weights
        cfg = preset("llama3-8b", layers=2, hidden=1024, n_heads=8, n_kv_heads=2, ffn=2048, vocab=2048, max_ctx=128)
        w = random_llama_weights(cfg, dev, seed=6, std=0.02)  # flat logits: sampling departs from greedy
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        eng = Engine.build(local_config(cfg, world), shard_llama_weights(w, cfg, rank, world), device=dev,
                           max_batch=4, max_ctx=128, block_size=16, num_blocks=64, max_rows=8, tp=tp)
        sp = SamplingParams(max_tokens=12, temperature=1.2, top_k=200, top_p=0.98, seed=123)
        gen = eng.generate([list(range(30, 40))], sp)
        gens = [None] * world
        dist.all_gather_object(gens, gen)
        tp.check()
        if rank == 0:
            ref = Engine.build(cfg, w, device=dev, max_batch=4, max_ctx=128, block_size=16, num_blocks=64,
                               max_rows=8)
            ref_gen = ref.generate([list(range(30, 40))], sp)
            greedy = ref.generate([list(range(30, 40))], SamplingParams(max_tokens=12))
            torch.save({"gens": gens, "ref_gen": ref_gen, "greedy": greedy}, out_path)
        torch.cuda.synchronize()
        tp.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_sampling_matches_tp1(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "sample.pt")
    mp.spawn(_sampling_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["gens"][0] == r["gens"][1], r  # every rank draws the same tokens
    # the one-GPU engine draws the same tokens from the same seed until a draw lands within the
    # logits' rounding difference of a CDF boundary (the two sum the layers in different orders),
    # after which the sequences are different samples: the leading tokens must agree
    tp_seq, ref_seq = r["gens"][0][0], r["ref_gen"][0]
    assert tp_seq[:3] == ref_seq[:3], r
    assert r["ref_gen"] != r["greedy"] and r["gens"][0] != r["greedy"], r  # it really sampled


def _tc_wide_worker(rank, world, port, out_path):
    """Tensor-core path at up to 64 rows: row-parallel GEMM partials all-reduced by the P2P-read
    consumer (no NCCL), against one GPU on the same path."""
    import datetime

    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from hawking_b200.engine.engine import Engine
        from hawking_b200.engine.sampling import SamplingParams
        from hawking_b200.models.config import preset
        from hawking_b200.models.llama import random_llama_weights
        from hawking_b200.parallel.tp import TPComm, local_config, shard_llama_weights
        cfg = preset("llama3-8b", layers=2, hidden=1024, n_heads=8, n_kv_heads=2, ffn=2048, vocab=2048, max_ctx=128)
        w = random_llama_weights(cfg, dev, seed=7, std=0.05)
        tp = TPComm(rank, world, 2 * cfg.layers, 8, cfg.hidden, dev)
        eng = Engine.build(local_config(cfg, world), shard_llama_weights(w, cfg, rank, world), device=dev,
                           max_batch=4, max_ctx=128, block_size=16, num_blocks=64, max_rows=64, tp=tp)
        eng.model.tc_min_rows = 1  # the tensor-core path at every row count
        toks = list(range(10, 34))  # 24 rows: one tensor-core forward through the P2P sites
        local = eng.model.forward_tokens(toks, seq_id=1)
        eng.kv.drop(1)
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous())
        full = torch.cat(parts, 1)
        gen = eng.generate([list(range(30, 40)), list(range(50, 53)), list(range(60, 70))],
                           SamplingParams(max_tokens=6))
        gens = [None] * world
        dist.all_gather_object(gens, gen)
        tp.check()
        if rank == 0:
            ref = Engine.build(cfg, w, device=dev, max_batch=4, max_ctx=128, block_size=16, num_blocks=64,
                               max_rows=64)
            ref.model.tc_min_rows = 1
            ref_logits = ref.model.forward_tokens(toks, seq_id=1)
            ref.kv.drop(1)
            ref_gen = ref.generate([list(range(30, 40)), list(range(50, 53)), list(range(60, 70))],
                                   SamplingParams(max_tokens=6))
            err = float((full - ref_logits).abs().max() / ref_logits.abs().max())
            torch.save({"err": err, "gens": gens, "ref_gen": ref_gen}, out_path)
        torch.cuda.synchronize()
        eng.model.release_graphs()
        tp.close()
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_tensor_core_p2p_allreduce_matches_tp1(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "tcwide.pt")
    mp.spawn(_tc_wide_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["err"] < 0.01, r
    assert r["gens"][0] == r["gens"][1], r
    assert [g[0] for g in r["gens"][0]] == [g[0] for g in r["ref_gen"]], r
