"""Pruned LM head and per-layer quantisation tiers on the device.

* The pruned head's logits are the full head's logits at the kept ids (teacher-forced decode rows
  through the same W4A16 / W4A8 head kernels), and every token the engine emits, greedy or
  sampled, is an original id of the whitelist: the argmax of the kept logits.
* A tier map re-quantises the FFN weights of the listed layers (the decoded weights stay within
  the target format's rounding of the originals) and the engine then generates through the mixed
  formats."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200.engine.engine import Engine  # noqa: E402
from hawking_b200.engine.sampling import SamplingParams  # noqa: E402
from hawking_b200.engine.vocab_prune import PrunedVocab, QuantTierMap  # noqa: E402
from hawking_b200.formats.ggml import GgmlType  # noqa: E402
from hawking_b200.formats.synth import random_prompt  # noqa: E402
from hawking_b200.models.config import preset  # noqa: E402
from hawking_b200.models.llama import random_llama_weights  # noqa: E402

DEV = "cuda"


def _engine(cfg, w):
    return Engine.build(cfg, w, device=DEV, max_batch=2, max_ctx=256, block_size=16, num_blocks=64, max_rows=16)


def _decode_logits(model, tokens, seq_id):
    """Teacher-forced single-row decode forwards (the small-batch head kernels)."""
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
    kv.drop(seq_id)
    return torch.stack(out)


@pytest.mark.parametrize("name", ["tiny-llama", "llama3-8b"])
def test_pruned_head_is_the_full_head_at_kept_ids(name):
    cfg = preset(name).with_(layers=1, max_ctx=256)
    w = random_llama_weights(cfg, DEV, seed=5, std=0.02)
    prompt = random_prompt(24, cfg.vocab, seed=6)
    full = _engine(cfg, w)
    ref = _decode_logits(full.model, prompt, seq_id=1)
    g = torch.Generator().manual_seed(7)
    keep = set(torch.randperm(cfg.vocab, generator=g)[:3001].tolist())
    keep |= set(ref[::2].argmax(1).tolist())  # the full argmax is kept at half of the positions
    pv = PrunedVocab(sorted(keep), cfg.vocab)
    eng = _engine(cfg, w)
    eng.enable_vocab_prune(pv)
    assert w.lm_head.N == cfg.vocab  # the caller's weights keep the whole head
    got = _decode_logits(eng.model, prompt, seq_id=2)
    idx = torch.tensor(pv.keep, device=DEV)
    sub = ref[:, idx]
    assert got.shape == sub.shape
    assert (got - sub).abs().max().item() <= 1e-4 * sub.abs().max().item()

    # greedy generation: original ids of the whitelist, the first one the kept argmax
    out = eng.generate([prompt], SamplingParams(max_tokens=12))[0]
    assert len(out) == 12 and all(t in keep for t in out)
    last = sub[-1]
    top2 = last.topk(2).values
    if (top2[0] - top2[1]).item() > 1e-3 * last.abs().max().item():
        assert out[0] == pv.keep[int(last.argmax())]
    # the full-logits lane (device sampler, host repetition penalty) emits kept ids too
    for params in (SamplingParams(temperature=0.9, top_k=50, max_tokens=10, seed=3),
                   SamplingParams(temperature=0.7, repetition_penalty=1.3, max_tokens=6, seed=4)):
        out = eng.generate([prompt], params)[0]
        assert len(out) == params.max_tokens and all(t in keep for t in out)
    with pytest.raises(ValueError):
        eng.add_request(prompt, SamplingParams(json_mode=True))
    with pytest.raises(ValueError):
        eng.enable_vocab_prune(pv)


def test_tier_map_requantizes_ffn_layers():
    cfg = preset("llama3-8b").with_(layers=2, hidden=1024, n_heads=8, n_kv_heads=2, ffn=2816, vocab=32000,
                                    max_ctx=256)
    w = random_llama_weights(cfg, DEV, seed=8, std=0.02)
    down0 = w.layers[0].w_down.dequantize()
    gate1 = (w.layers[1].w_gu or w.layers[1].w_gate).dequantize()
    tiers = QuantTierMap({0: {"down": int(GgmlType.Q8_0)},
                          1: {"gate_up": int(GgmlType.Q6_K), "down": int(GgmlType.Q4_K)}}, n_layers=2)
    assert tiers.apply(w, cfg) >= 2
    l0, l1 = w.layers
    assert l0.w_down.fmt == GgmlType.Q8_0 and l1.w_down.fmt == GgmlType.Q4_K
    gu1 = l1.w_gu or l1.w_gate
    assert gu1.fmt == GgmlType.Q6_K and l1.w_up.fmt == GgmlType.Q6_K
    # re-quantising Q4_K values to a finer format keeps them within that format's rounding
    assert (l0.w_down.dequantize() - down0).abs().max().item() <= 1e-2 * down0.abs().max().item()
    assert (gu1.dequantize() - gate1).abs().max().item() <= 3e-2 * gate1.abs().max().item()
    eng = _engine(cfg, w)
    prompt = random_prompt(20, cfg.vocab, seed=9)
    out = eng.generate([prompt], SamplingParams(max_tokens=8))[0]
    assert len(out) == 8 and all(0 <= t < cfg.vocab for t in out)
    logits = eng.model.forward_tokens(prompt, seq_id=5)
    assert torch.isfinite(logits).all()
