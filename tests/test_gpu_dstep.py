"""Persistent decode step (decode_step.cu, ops/dstep.py) on a tiny Q4_K Llama: teacher-forced logits
against the C++ CPU oracle run in fp32 activations / bf16 KV, against the per-kernel W4A16 path,
batch-composition invariance, CUDA-graph replay, and the bounded grid-barrier wait."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200.engine.engine import Engine  # noqa: E402
from hawking_b200.engine.sampling import SamplingParams  # noqa: E402
from hawking_b200.formats.gguf import GgufModel  # noqa: E402
from hawking_b200.formats.synth import random_prompt  # noqa: E402
from hawking_b200.models.llama import load_llama_weights  # noqa: E402
from hawking_b200.models.torch_ref import config_from_gguf  # noqa: E402


@pytest.fixture(scope="module")
def q4k_path(tmp_path_factory):
    from hawking_b200.formats.synth import write_llama_family_gguf
    from hawking_b200.models.config import preset
    p = tmp_path_factory.mktemp("dstep") / "tiny-llama-q4_k.gguf"
    write_llama_family_gguf(str(p), preset("tiny-llama", weight_type="Q4_K", ffn=1536), seed=5)
    return str(p)


@pytest.fixture(scope="module")
def parts(q4k_path):
    m = GgufModel(q4k_path)
    cfg = config_from_gguf(m).with_(max_ctx=512)
    return cfg, load_llama_weights(m, cfg, "cuda")


def _engine(cfg, w):
    import os
    old = os.environ.get("HK_DSTEP")
    os.environ["HK_DSTEP"] = "1"  # the one-launch step is opt-in
    try:
        return Engine.build(cfg, w, device="cuda", max_batch=4, max_ctx=512, block_size=16, num_blocks=160,
                            max_rows=16)
    finally:
        if old is None:
            del os.environ["HK_DSTEP"]
        else:
            os.environ["HK_DSTEP"] = old


def _decode_tokens(model, tokens, seq_id):
    """Teacher-forced, one decode-step forward per token (the persistent kernel's path)."""
    kv = model.kv
    assert kv.bm.reserve(seq_id, len(tokens))
    kv.sync_tables([seq_id])
    r = kv.row(seq_id)
    out = []
    for i, t in enumerate(tokens):
        model.inp.upload([t], [i], [0], [r], [i + 1])
        model.forward(1, "none", n_logits=0)
        out.append(model.logits[0].clone())
    torch.cuda.synchronize()
    return torch.stack(out)


def test_decode_step_is_built(parts):
    cfg, w = parts
    eng = _engine(cfg, w)
    assert eng.model.dstep is not None


def test_decode_step_logits_match_cpu_oracle(parts, q4k_path, native):
    cfg, w = parts
    prompt = random_prompt(40, cfg.vocab, seed=4)
    cpu = native.CpuLlama(q4k_path, 128, 8, False, True)  # fp32 activations, bf16 KV
    ref = np.stack([cpu.forward(t, i) for i, t in enumerate(prompt)])
    eng = _engine(cfg, w)
    got = _decode_tokens(eng.model, prompt, seq_id=1).cpu().numpy()
    assert int(eng.model.status.item()) == 0
    scale = np.abs(ref).max()
    err = np.abs(got - ref).max()
    assert err < 2e-2 * scale, (err, scale)
    top2 = np.sort(ref, axis=1)[:, -2:]
    decided = (top2[:, 1] - top2[:, 0]) > 2 * err
    assert decided.sum() >= 4
    assert (got.argmax(1)[decided] == ref.argmax(1)[decided]).all()


def test_decode_step_matches_per_kernel_path(parts):
    cfg, w = parts
    prompt = random_prompt(24, cfg.vocab, seed=6)
    eng = _engine(cfg, w)
    a = _decode_tokens(eng.model, prompt, seq_id=1)
    ds = eng.model.dstep
    eng.model.dstep = None
    try:
        b = _decode_tokens(eng.model, prompt, seq_id=2)
    finally:
        eng.model.dstep = ds
    err = (a - b).abs().max().item()
    assert err < 1e-2 * b.abs().max().item(), err


def test_decode_step_rows_independent_of_batch(parts):
    """With the split count fixed, a row's tokens do not depend on the other rows of the step
    (per-column GEMV math, fixed fix-up order, per-row attention)."""
    cfg, w = parts
    prompts = [random_prompt(17 + 5 * i, cfg.vocab, seed=20 + i) for i in range(4)]
    sp = SamplingParams(max_tokens=10)
    outs = []
    for batched in (False, True):
        eng = _engine(cfg, w)
        eng.model.force_splits = 2
        outs.append(eng.generate(prompts, sp) if batched else [eng.generate([p], sp)[0] for p in prompts])
    assert outs[0] == outs[1]


def test_decode_step_graph_replay_matches_eager(parts):
    cfg, w = parts
    p = random_prompt(30, cfg.vocab, seed=8)
    g = _engine(cfg, w).generate([p], SamplingParams(max_tokens=12))[0]
    eng = _engine(cfg, w)
    eng.use_graphs = False
    e = eng.generate([p], SamplingParams(max_tokens=12))[0]
    assert g == e


def test_decode_step_barrier_wait_is_bounded(parts):
    """A grid barrier that can never complete (its arrival counter pre-set far past the grid size)
    ends every CTA's wait after wait_ns with status 2; the context stays usable and a reset step
    runs clean."""
    cfg, w = parts
    eng = _engine(cfg, w)
    m = eng.model
    ds = m.dstep
    kv = m.kv
    assert kv.bm.reserve(3, 8)
    kv.sync_tables([3])
    m.inp.upload([5], [0], [0], [kv.row(3)], [1])
    ds.wait_ns = 5_000_000
    ds.bar[0] = 1 << 30
    m.status.zero_()
    m.forward(1, "none", n_logits=0)
    torch.cuda.synchronize()
    assert int(m.status.item()) == 2
    ds.reset()
    m.status.zero_()
    m.forward(1, "none", n_logits=0)
    torch.cuda.synchronize()
    assert int(m.status.item()) == 0
    assert bool(torch.isfinite(m.logits[0]).all())
