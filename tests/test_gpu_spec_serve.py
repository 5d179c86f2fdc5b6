"""Speculative decoding inside the engine step (``Engine.enable_speculative``) and disk prefix-KV
reuse at admission (``Engine.enable_prefix_disk``), on the tiny Llama-arch model: both lossless
against the plain engine, both reachable from the HTTP serving loop."""
import http.client
import json

import pytest

pytestmark = pytest.mark.gpu

from hawking_b200.engine.engine import Engine  # noqa: E402
from hawking_b200.engine.sampling import SamplingParams  # noqa: E402
from hawking_b200.formats.gguf import GgufModel  # noqa: E402
from hawking_b200.models.llama import load_llama_weights  # noqa: E402
from hawking_b200.models.torch_ref import config_from_gguf  # noqa: E402


@pytest.fixture(scope="module")
def parts(tiny_gguf):
    m = GgufModel(tiny_gguf)
    cfg = config_from_gguf(m).with_(max_ctx=512)
    return cfg, load_llama_weights(m, cfg, "cuda")


def _engine(cfg, w):
    return Engine.build(cfg, w, device="cuda", max_batch=4, max_ctx=512, block_size=16, num_blocks=192, max_rows=16)


def test_speculative_step_is_lossless(parts):
    cfg, w = parts
    prompt = [5, 6, 7, 8, 9] * 6  # repetitive: the n-gram drafter finds continuations
    sp = SamplingParams(max_tokens=40)
    plain = _engine(cfg, w)
    plain.model.force_splits = plain.model.num_splits(1)
    ref = plain.generate([prompt], sp)[0]
    eng = _engine(cfg, w)
    eng.enable_speculative(4)
    got = eng.generate([prompt], sp)[0]
    st = eng.spec_stats()
    assert got == ref
    assert st["cycles"] > 0 and st["emitted"] == len(got) - 1  # the first token comes from the prefill
    assert st["cycles"] < st["emitted"] or st["accepted"] == 0


def test_prefix_disk_reuse_is_lossless(parts, tmp_path):
    cfg, w = parts
    shared = list(range(100, 180))  # 5 whole blocks of 16
    a, b = shared + [3, 4, 5], shared + [7, 8]
    sp = SamplingParams(max_tokens=8)
    e1 = _engine(cfg, w)
    e1.enable_prefix_disk(str(tmp_path), min_blocks=2)
    e1.generate([a], sp)
    assert e1.stats_disk["stored"] == 1
    e2 = _engine(cfg, w)  # a fresh engine: empty in-memory prefix cache
    e2.enable_prefix_disk(str(tmp_path), min_blocks=2)
    got = e2.generate([b], sp)[0]
    assert e2.stats_disk["hits"] == 1 and e2.stats_disk["hit_tokens"] == 80
    assert e2.kv.bm.prefix_hits >= 1
    ref = _engine(cfg, w).generate([b], sp)[0]
    assert got == ref


def test_serve_with_speculation(parts, tiny_gguf, native, tmp_path):
    from hawking_b200.serve import ServeLoop
    cfg, w = parts
    tok = native.Tokenizer.from_gguf(native.GgufFile.open(tiny_gguf))
    outs = []
    for spec in (0, 4):
        eng = _engine(cfg, w)
        eng.model.force_splits = eng.model.num_splits(1)
        if spec:
            eng.enable_speculative(spec)
            eng.enable_prefix_disk(str(tmp_path / "pd"), min_blocks=1)
        loop = ServeLoop(eng, tok, port=0, model_id="tiny").start()
        th = loop.run_in_thread()
        c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=120)
        c.request("POST", "/v1/completions", body=json.dumps({"prompt": "a b c a b c a b c a b c", "max_tokens": 16,
                                                              "temperature": 0}))
        r = c.getresponse()
        outs.append((r.status, json.loads(r.read().decode())["choices"][0]["text"]))
        c.close()
        loop.stop()
        th.join(timeout=10)
        if spec:
            assert eng.spec_stats()["cycles"] > 0
    assert outs[0][0] == outs[1][0] == 200
    assert outs[0][1] == outs[1][1]
