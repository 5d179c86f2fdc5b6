"""Multi-rank serving lockstep (serve/lockstep.py) on CPU ranks over gloo: the follower replays the
leader's admissions, aborts, steps and embeddings in order with matching request ids, a step that
fails on a follower fails on the leader, and ``stop`` ends the follower."""
import os
import socket

import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402


class FakeEngine:
    def __init__(self, fail_step=-1):
        self.log, self.next_id, self.steps, self.fail_step = [], 0, 0, fail_step
        self.max_batch = 4

    def add_request(self, prompt, params):
        rid = self.next_id
        self.next_id += 1
        self.log.append(("add", rid, tuple(prompt), params.temperature, params.seed))
        return rid

    def abort(self, rid):
        self.log.append(("abort", rid))

    def step(self):
        self.steps += 1
        self.log.append(("step", self.steps))
        if self.steps == self.fail_step:
            raise RuntimeError("device status word set")
        return [(0, 7, 0)]

    def embed(self, ids):
        self.log.append(("embed", tuple(ids)))
        return [0.0]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.serve.lockstep import LeaderEngine, follow
    try:
        if rank == 0:
            eng = LeaderEngine(FakeEngine())
            eng.tokenizer = "tok"  # attribute writes reach the wrapped engine
            a = eng.add_request([1, 2, 3], SamplingParams(temperature=0.7, seed=9))
            b = eng.add_request([4], SamplingParams())
            eng.step()
            eng.abort(a)
            eng.embed([5, 6])
            eng.step()
            failed = False
            try:
                eng.step()  # the follower fails this one
            except RuntimeError:
                failed = True
            eng.abort(b)
            eng.stop()
            q.put(("leader", eng._engine.log, eng._engine.tokenizer, failed))
        else:
            e = FakeEngine(fail_step=3)
            n = follow(e)
            q.put(("follower", e.log, n))
    finally:
        dist.destroy_process_group()


def test_lockstep_replays_the_leader():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict()
    for _ in range(2):
        item = q.get(timeout=60)
        out[item[0]] = item[1:]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    leader_log, tok, failed = out["leader"]
    follower_log, steps = out["follower"]
    assert tok == "tok"
    assert failed  # a step that failed on the follower failed on the leader
    assert follower_log == leader_log
    assert steps == 3
    assert [e[0] for e in leader_log] == ["add", "add", "step", "abort", "embed", "step", "step", "abort"]
