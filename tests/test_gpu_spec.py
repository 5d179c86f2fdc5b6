"""Lossless speculative decoding on the GPU: n-gram drafts verified in one forward give exactly
the plain greedy output (tiny Llama-arch model)."""
import pytest

pytestmark = pytest.mark.gpu


def test_speculative_matches_greedy(tiny_gguf):
    from hawking_b200.engine.engine import Engine
    from hawking_b200.engine.sampling import SamplingParams
    from hawking_b200.engine.speculative import SpeculativeDecoder
    eng = Engine.from_gguf(tiny_gguf, max_batch=2, max_ctx=256, block_size=16, num_blocks=64, max_rows=32)
    prompts = [[3, 4, 5, 6] * 6, list(range(100, 131))]
    for prompt in prompts:
        ref = eng.generate([prompt], SamplingParams(max_tokens=40))[0]
        dec = SpeculativeDecoder(eng, k=4)
        out = dec.generate(prompt, 40)
        assert out == ref
        assert dec.stats.cycles < 40 or dec.stats.drafted == 0
    # all KV blocks of the scratch sequences were returned
    assert eng.kv.bm.num_free == eng.kv.bm.num_blocks
