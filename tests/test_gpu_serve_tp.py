"""Serving on 2 GPUs: rank 0 runs HTTP and the engine loop (``LeaderEngine``), rank 1 replays the
schedule (``follow``); the tensor-parallel engine streams a non-greedy chat completion over SSE
(sampling over the gathered vocabulary slices, tested against one GPU in test_gpu_tp.py)."""
import http.client
import json
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from hawking_b200.serve.__main__ import init_ranks, preset_engine, shutdown_ranks
    from hawking_b200.serve.lockstep import LeaderEngine, follow
    from hawking_b200.serve.server import ServeLoop
    world, rank, gloo = init_ranks()
    eng, tok = preset_engine("llama3-8b", layers=2, max_batch=4, max_ctx=256, device=f"cuda:{rank}",
                             tp_rank=rank, tp_world=world)
    try:
        if rank > 0:
            eng.tokenizer = tok
            follow(eng, gloo)
            return
        leader = LeaderEngine(eng, gloo)
        loop = ServeLoop(leader, tok, port=0, model_id="tp2").start()
        th = loop.run_in_thread()
        body = {"messages": [{"role": "user", "content": "hello there"}], "max_tokens": 8, "stream": True,
                "temperature": 0.9, "top_k": 50, "top_p": 0.95, "seed": 5}
        c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=300)
        c.request("POST", "/v1/chat/completions", body=json.dumps(body))
        r = c.getresponse()
        status, text = r.status, r.read().decode()
        c.close()
        loop.stop()
        th.join(timeout=30)
        leader.stop()
        torch.save({"status": status, "sse": text}, out_path)
    finally:
        shutdown_ranks(eng)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_serve_streams_sampled_completion(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "serve.pt")
    mp.spawn(_worker, args=(2, _port(), out), nprocs=2, join=True)
    r = torch.load(out)
    assert r["status"] == 200, r
    events = [ln[len("data: "):] for ln in r["sse"].splitlines() if ln.startswith("data: ")]
    assert events and events[-1] == "[DONE]", r["sse"][-400:]
    chunks = [json.loads(e) for e in events[:-1]]
    assert any(ch["choices"][0]["delta"].get("content") for ch in chunks if ch.get("choices")), r["sse"][-400:]
