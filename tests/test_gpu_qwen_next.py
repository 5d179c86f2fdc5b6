"""Qwen3-Next-style hybrid decoder on the GPU vs the fp32 token-serial PyTorch oracle: gated DeltaNet
(K7), gated full attention (head_dim 64 here), routed mixed-codec experts + sigmoid-gated shared
expert (K8), on a tiny configuration with materialised (encoded) random weights."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def tiny_cfg():
    from hawking_b200.models.config import preset
    return preset("qwen3-next", vocab=512, hidden=256, layers=4, n_heads=4, n_kv_heads=2, head_dim=64, rot_dim=16,
                  n_experts=8, top_k=2, expert_ffn=128, shared_ffn=128, linear_k_heads=2, linear_v_heads=4,
                  linear_head_dim=64, max_ctx=256)


def test_mixed_weight_roundtrip_and_gemv(native):
    from hawking_b200.formats import mixed as mx
    from hawking_b200.ops import Q8Act, rmsnorm_q8
    from hawking_b200.ops.mixed import BINARY, UNIFORM, MixedTable, MixedWeight, mixed_gemv
    g = torch.Generator(device=DEV).manual_seed(3)
    w = torch.randn(96, 512, generator=g, device=DEV) * 0.05
    ws = [MixedWeight.quantize(w, BINARY, 1), MixedWeight.quantize(w, UNIFORM, 2), MixedWeight.quantize(w, UNIFORM, 4),
          MixedWeight.quantize(w, UNIFORM, 8)]
    # payloads written by the C++ encoders load to the same device planes' semantics
    wn = w.cpu().numpy()
    for payload in (mx.encode_binary(wn, 64), mx.encode_uniform(wn, 2, 64), mx.encode_uniform(wn, 4, 64)):
        mw = MixedWeight.from_payload(payload, DEV)
        ref = torch.from_numpy(mx.decode(payload)).to(DEV)
        assert torch.allclose(mw.dequantize(), ref, atol=1e-6)
        ws.append(mw)
    t = MixedTable(ws)
    x = torch.randn(3, 512, generator=g, device=DEV)
    xa = Q8Act(3, 512, DEV)
    rmsnorm_q8(x, None, 1e-5, xa, norm=False)
    xdq = xa.dequantize()
    for i, mw in enumerate(ws):
        y = torch.zeros(3, 96, device=DEV)
        mixed_gemv(t, i, xa, y)
        ref = xdq @ mw.dequantize().t()
        torch.testing.assert_close(y, ref, rtol=2e-3, atol=2e-3 * float(ref.abs().max()),
                                   msg=lambda m, i=i, mw=mw: f"tensor {i} (kind {mw.kind}, bits {mw.bits}): {m}")


def test_qwen_next_matches_torch_oracle():
    from hawking_b200.engine.kv_cache import PagedKVCache
    from hawking_b200.models.qwen_next import QwenNextModel, TorchRefQwenNext, random_qwen_next_weights
    cfg = tiny_cfg()
    w = random_qwen_next_weights(cfg, DEV, seed=1, materialise=True, std=0.05)
    n_full = sum(cfg.layer_is_full_attention(l) for l in range(cfg.layers))
    kv = PagedKVCache(n_full, cfg.n_kv_heads, cfg.head_dim, 32, 16, 2, 16, DEV)
    m = QwenNextModel(cfg, w, kv, max_rows=2, max_seqs=3, device=DEV)
    toks = [5, 77, 300, 12, 9, 401, 256, 3]
    got = m.forward_tokens(toks, seq_id=1)
    ref_model = TorchRefQwenNext(cfg, w)
    ref = torch.stack([ref_model.step(t, p) for p, t in enumerate(toks)])
    err = float((got - ref).abs().max() / ref.abs().max())
    assert err < 0.02, err
    top2 = ref.topk(2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2 * err * ref.abs().max()
    assert ((got.argmax(1) == ref.argmax(1)) | ~clear).all()
