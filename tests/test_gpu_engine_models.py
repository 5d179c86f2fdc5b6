"""The serving engine (scheduler, paged caches, CUDA-graph decode) around the MLA + MoE and the
hybrid DeltaNet models: greedy generation through ``Engine.step`` equals the model's own
teacher-forced token-by-token greedy decode."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _greedy_reference(model, prompt, n, seq_id=99):
    """Greedy tokens from the model's teacher-forced forward: the prompt, then one token at a time."""
    out = []
    logits = model.forward_tokens(prompt, seq_id=seq_id)
    tok = int(logits[-1].argmax())
    pos = len(prompt)
    for _ in range(n):
        out.append(tok)
        logits = model.forward_tokens([tok], seq_id=seq_id, start_pos=pos)
        pos += 1
        tok = int(logits[-1].argmax())
    return out


def test_engine_deepseek_greedy_matches_model():
    from hawking_b200.engine.engine import Engine
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.models.deepseek import DeepSeekModel, LatentCache, random_deepseek_weights
    from test_gpu_deepseek import tiny_cfg
    cfg = tiny_cfg().with_(hidden=512)
    w = random_deepseek_weights(cfg, DEV, seed=7, std=0.05)
    eng = Engine.build_deepseek(cfg, w, device=DEV, max_batch=2, max_ctx=256, block_size=16, num_blocks=64)
    prompt = [5, 77, 300, 12, 9, 401, 256, 3, 44, 100]
    got = eng.generate([prompt], SamplingParams(max_tokens=5))[0]
    # the reference runs the prompt in forwards as wide as the engine's (same kernels, same rounding)
    ref_m = DeepSeekModel(cfg, w, LatentCache(cfg.layers, 64, 16, 2, 16, DEV), max_rows=eng.model.row_limit,
                          device=DEV)
    assert got == _greedy_reference(ref_m, prompt, 5)
    two = eng.generate([prompt, prompt[:4]], SamplingParams(max_tokens=3))
    assert [len(t) for t in two] == [3, 3]


def test_engine_qwen_next_waves_match_model():
    from hawking_b200.engine.engine import Engine
    from hawking_b200.engine.kv_cache import PagedKVCache
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.models.qwen_next import QwenNextModel, random_qwen_next_weights
    from test_gpu_qwen_next import tiny_cfg
    cfg = tiny_cfg()
    w = random_qwen_next_weights(cfg, DEV, seed=1, materialise=True, std=0.05)
    eng = Engine.build_qwen_next(cfg, w, device=DEV, max_batch=2, max_ctx=256, block_size=16, num_blocks=64)
    prompt = [5, 77, 300, 12, 9, 401, 256, 3, 44, 100, 7]
    got = eng.generate([prompt], SamplingParams(max_tokens=5))[0]
    n_full = sum(cfg.layer_is_full_attention(l) for l in range(cfg.layers))
    kv = PagedKVCache(n_full, cfg.n_kv_heads, cfg.head_dim, 64, 16, 2, 16, DEV, prefix_cache=False)
    ref_m = QwenNextModel(cfg, w, kv, max_rows=eng.model.row_limit, max_seqs=2, device=DEV)
    assert got == _greedy_reference(ref_m, prompt, 5, seq_id=1)
    # two sequences of different lengths advance in waves (one row per sequence per forward)
    two = eng.generate([prompt, prompt[:3]], SamplingParams(max_tokens=4))
    assert [len(t) for t in two] == [4, 4]
    again = eng.generate([prompt], SamplingParams(max_tokens=5))[0]
    assert again == got  # the recurrent state was reset for the new sequence


def test_serve_deepseek_preset_completion():
    """The OpenAI server on the MLA + MoE engine (random weights, synthetic tokenizer)."""
    import http.client
    import json

    from hawking_b200.serve import ServeLoop
    from hawking_b200.serve.__main__ import preset_engine
    eng, tok = preset_engine("deepseek-v3", layers=4, max_batch=2, max_ctx=512)
    loop = ServeLoop(eng, tok, port=0, model_id="ds").start()
    th = loop.run_in_thread()
    try:
        c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=300)
        c.request("POST", "/v1/completions", body=json.dumps({"prompt": "hello world", "max_tokens": 5,
                                                                "temperature": 0}))
        r = c.getresponse()
        body = r.read().decode()
        assert r.status == 200, body
        o = json.loads(body)
        assert 1 <= o["usage"]["completion_tokens"] <= 5
    finally:
        loop.stop()
        th.join(timeout=10)


def test_cli_generate_preset(capsys):
    """``python -m hawking_b200 generate`` end to end on random-weight presets."""
    import json as _json

    from hawking_b200.__main__ import main
    for preset in ("deepseek-v3", "qwen3-next"):
        assert main(["generate", "--preset", preset, "--layers", "4", "--prompt", "hello", "--max-tokens", "4",
                     "--max-ctx", "256", "--json"]) == 0
        out = _json.loads(capsys.readouterr().out.strip().splitlines()[-1])
        assert 1 <= len(out["tokens"]) <= 4
