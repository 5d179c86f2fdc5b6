"""Wide prefill forwards of the flagship models: a prompt run as one forward of many rows (experts
as grouped tensor-core GEMMs over bf16 rows, the MLA absorb / output kernels in 8-row slices, the
DeltaNet kernels walking the run) against the fp32 oracle without activation rounding, next to
the 8-row decode-kernel forwards (int8 activation blocks) against the oracle that rounds like
them. The wide path rounds activations to bf16 instead of int8 blocks, so a top-k expert choice
that is a near tie can go either way between the two paths: each path must match its own oracle
at 90 % of the positions."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOKS = [5, 77, 300, 12, 9, 401, 256, 3, 44, 100, 7, 18, 250, 31, 402, 66, 1, 90, 301, 11, 420, 7, 8, 9, 10,
        123, 200, 310, 45, 46, 47, 48, 49, 50, 51, 52, 53, 54, 55, 56]


def _frac(a, b, tol):
    err = (a - b).abs().amax(1) / b.abs().max()
    return (err < tol).float().mean().item(), err


def test_deepseek_wide_prefill_matches_oracle():
    from hawking_b200.models.deepseek import DeepSeekModel, LatentCache, TorchRefDeepSeek, random_deepseek_weights
    from test_gpu_deepseek import tiny_cfg
    cfg = tiny_cfg().with_(hidden=512)
    w = random_deepseek_weights(cfg, DEV, seed=5, std=0.05)
    wide = DeepSeekModel(cfg, w, LatentCache(cfg.layers, 64, 16, 2, 16, DEV), max_rows=64, device=DEV)
    got = wide.forward_tokens(TOKS, seq_id=1)
    ref_m = TorchRefDeepSeek(cfg, w, act_q8=False)
    with torch.no_grad():
        ref = torch.stack([ref_m.step(t, p) for p, t in enumerate(TOKS)])
    frac, err = _frac(got, ref, 3e-2)
    assert frac >= 0.9, err.tolist()
    assert int(wide.status.item()) == 0


def test_qwen_next_wide_prefill_matches_oracle():
    from hawking_b200.engine.kv_cache import PagedKVCache
    from hawking_b200.models.qwen_next import QwenNextModel, TorchRefQwenNext, random_qwen_next_weights
    from test_gpu_qwen_next import tiny_cfg
    cfg = tiny_cfg().with_(hidden=512)
    w = random_qwen_next_weights(cfg, DEV, seed=6, materialise=True, std=0.05)
    n_full = sum(cfg.layer_is_full_attention(l) for l in range(cfg.layers))

    def model(rows):
        kv = PagedKVCache(n_full, cfg.n_kv_heads, cfg.head_dim, 64, 16, 2, 16, DEV, prefix_cache=False)
        return QwenNextModel(cfg, w, kv, max_rows=rows, max_seqs=2, device=DEV)

    wide = model(64).forward_tokens(TOKS, seq_id=1)
    narrow = model(8).forward_tokens(TOKS, seq_id=1)
    with torch.no_grad():
        ref32 = TorchRefQwenNext(cfg, w, act_q8=False)
        r32 = torch.stack([ref32.step(t, p) for p, t in enumerate(TOKS)])
        ref8 = TorchRefQwenNext(cfg, w, act_q8=True)
        r8 = torch.stack([ref8.step(t, p) for p, t in enumerate(TOKS)])
    frac, err = _frac(wide, r32, 3e-2)
    assert frac >= 0.9, ("wide", err.tolist())
    frac, err = _frac(narrow, r8, 2e-2)
    assert frac >= 0.9, ("narrow", err.tolist())
