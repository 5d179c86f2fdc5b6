"""Wide prefill forwards of the flagship models: a prompt run as one forward of many rows (the
expert kernels over all of the chunk's pairs, the absorb / output MLA kernels in 8-row slices, the
DeltaNet kernels walking the run) gives the logits of the 8-row forwards, position by position
(a top-k expert choice that is a near tie may flip between the two, so 90 % of the positions
must agree closely)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOKS = [5, 77, 300, 12, 9, 401, 256, 3, 44, 100, 7, 18, 250, 31, 402, 66, 1, 90, 301, 11, 420, 7, 8, 9, 10,
        123, 200, 310, 45, 46, 47, 48, 49, 50, 51, 52, 53, 54, 55, 56]


def _agree(a, b, tol):
    scale = b.abs().max()
    err = (a - b).abs().amax(1) / scale
    return (err < tol).float().mean().item(), err


def test_deepseek_wide_prefill_matches_8_row_chunks():
    from hawking_b200.models.deepseek import DeepSeekModel, LatentCache, random_deepseek_weights
    from test_gpu_deepseek import tiny_cfg
    cfg = tiny_cfg().with_(hidden=512)
    w = random_deepseek_weights(cfg, DEV, seed=5, std=0.05)
    narrow = DeepSeekModel(cfg, w, LatentCache(cfg.layers, 64, 16, 2, 16, DEV), max_rows=8, device=DEV)
    wide = DeepSeekModel(cfg, w, LatentCache(cfg.layers, 64, 16, 2, 16, DEV), max_rows=64, device=DEV)
    a = narrow.forward_tokens(TOKS, seq_id=1)
    b = wide.forward_tokens(TOKS, seq_id=1)
    frac, err = _agree(b, a, 2e-2)
    assert frac >= 0.9, err.tolist()
    assert int(wide.status.item()) == 0


def test_qwen_next_wide_prefill_matches_8_row_chunks():
    from hawking_b200.engine.kv_cache import PagedKVCache
    from hawking_b200.models.qwen_next import QwenNextModel, random_qwen_next_weights
    from test_gpu_qwen_next import tiny_cfg
    cfg = tiny_cfg().with_(hidden=512)
    w = random_qwen_next_weights(cfg, DEV, seed=6, materialise=True, std=0.05)
    n_full = sum(cfg.layer_is_full_attention(l) for l in range(cfg.layers))

    def model(rows):
        kv = PagedKVCache(n_full, cfg.n_kv_heads, cfg.head_dim, 64, 16, 2, 16, DEV, prefix_cache=False)
        return QwenNextModel(cfg, w, kv, max_rows=rows, max_seqs=2, device=DEV)

    a = model(8).forward_tokens(TOKS, seq_id=1)
    b = model(64).forward_tokens(TOKS, seq_id=1)
    frac, err = _agree(b, a, 2e-2)
    assert frac >= 0.9, err.tolist()
