"""Wide prefill forwards of the flagship models (experts as grouped tensor-core GEMMs over bf16
rows, projections as bf16-weight GEMMs, the MLA absorption / value projection as batched GEMMs,
the DeltaNet kernels walking the run): the DeepSeek-style model end to end against the fp32
oracle without activation rounding, the hybrid per component. The wide path rounds activations to
bf16 where the decode path uses int8 blocks, so a top-k expert choice that is a near tie can go
either way: 90 % of the positions must match closely."""
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


def test_qwen_next_wide_components_match_torch():
    """Per component on one set of inputs (the tiny random hybrid is chaotic end to end: its two
    fp32 oracles, with and without int8 activation rounding, differ by up to 25 % per position):
    every projection as a bf16-weight GEMM, and a whole MoE layer (routing, grouped experts, gated
    shared expert) against fp32 PyTorch."""
    from hawking_b200 import ops
    from hawking_b200.engine.kv_cache import PagedKVCache
    from hawking_b200.models.qwen_next import QwenNextModel, random_qwen_next_weights
    from test_gpu_qwen_next import tiny_cfg
    cfg = tiny_cfg().with_(hidden=512)
    w = random_qwen_next_weights(cfg, DEV, seed=6, materialise=True, std=0.05)
    n_full = sum(cfg.layer_is_full_attention(l) for l in range(cfg.layers))
    kv = PagedKVCache(n_full, cfg.n_kv_heads, cfg.head_dim, 64, 16, 2, 16, DEV, prefix_cache=False)
    m = QwenNextModel(cfg, w, kv, max_rows=64, max_seqs=2, device=DEV)
    rows = 40
    g = torch.Generator(device=DEV).manual_seed(3)
    assert m._wide(rows)
    for L in w.layers:
        for key in (("q", "k", "v", "g", "o") if L.full else ("qkvz", "ba", "out")):
            wt = w.table.weights[L.idx[key]]
            xb = torch.randn(rows, wt.K, generator=g, device=DEV).bfloat16()
            y = torch.zeros(rows, wt.N, device=DEV)
            m.wide.linear(L.idx[key], xb, y)
            ref = xb.float() @ wt.dequantize().T
            assert (y - ref).abs().max().item() <= 5e-3 * ref.abs().max().item(), key
    W = [mw.dequantize() for mw in w.table.weights]
    silu = torch.nn.functional.silu
    for L in w.layers:
        x0 = torch.randn(rows, cfg.hidden, generator=g, device=DEV)
        m.x[:rows] = x0
        ops.rmsnorm_q8(m.x[:rows], L.post_norm, cfg.eps, m.xa.view(rows))
        m._moe(L, rows)
        torch.cuda.synchronize()
        got = m.x[:rows] - x0
        xn = x0 * torch.rsqrt((x0 * x0).mean(1, keepdim=True) + cfg.eps) * L.post_norm
        probs = torch.softmax(xn @ L.router.T, 1)
        tv, ti = probs.topk(cfg.top_k, 1)
        tv = tv / tv.sum(1, keepdim=True)
        ref = torch.zeros_like(x0)
        for t in range(rows):
            for j in range(cfg.top_k):
                e = int(ti[t, j])
                ref[t] += tv[t, j] * (W[L.idx["ed"] + e] @ (silu(W[L.idx["eg"] + e] @ xn[t]) * (W[L.idx["eu"] + e] @ xn[t])))
            ref[t] += torch.sigmoid(L.shared_gate[0] @ xn[t]) * (
                W[L.idx["sd"]] @ (silu(W[L.idx["sg"]] @ xn[t]) * (W[L.idx["su"]] @ xn[t])))
        err = (got - ref).abs().amax(1) / ref.abs().max()
        assert (err < 2e-2).float().mean().item() >= 0.9, err.tolist()


def test_deltanet_conv_wide_matches_walk():
    """The parallel convolution of a wide forward (two runs of 13 and 20 rows, each continuing a
    sequence whose conv state holds earlier inputs) equals the token walk run in forwards of up to
    8 rows: outputs and the final conv states."""
    from hawking_b200._ext import kernels
    kh, r, dk, dv, kc = 2, 2, 64, 64, 4
    ch = 2 * kh * dk + kh * r * dv
    qkvz_w = 2 * kh * dk + 2 * kh * r * dv
    g = torch.Generator(device=DEV).manual_seed(9)
    lens = [13, 20]
    rows = sum(lens)
    qkvz = torch.randn(rows, qkvz_w, generator=g, device=DEV)
    conv_w = torch.randn(ch, kc, generator=g, device=DEV) * 0.3
    state0 = torch.randn(3, ch, kc - 1, generator=g, device=DEV)
    slot = torch.tensor([1] * lens[0] + [2] * lens[1], dtype=torch.int32, device=DEV)

    def outs(n):
        return (torch.zeros(n, kh * r, dk, device=DEV), torch.zeros(n, kh * r, dk, device=DEV),
                torch.zeros(n, kh * r * dv, device=DEV), torch.zeros(n, kh * r * dv, device=DEV))

    st_w = state0.clone()
    qw, kw, vw, zw = outs(rows)
    kernels().deltanet_conv(qkvz, conv_w, st_w, slot, kh, r, dk, dv, kc, 1e-6, qw, kw, vw, zw, False)
    st_n = state0.clone()
    qn, kn, vn, zn = outs(rows)
    c0 = 0
    for L in lens:
        for a in range(c0, c0 + L, 8):
            b = min(c0 + L, a + 8)
            q1, k1, v1, z1 = outs(b - a)
            kernels().deltanet_conv(qkvz[a:b], conv_w, st_n, slot[a:b], kh, r, dk, dv, kc, 1e-6, q1, k1, v1, z1, False)
            qn[a:b], kn[a:b], vn[a:b], zn[a:b] = q1, k1, v1, z1
        c0 += L
    torch.cuda.synchronize()
    for got, ref in ((qw, qn), (kw, kn), (vw, vn), (zw, zn), (st_w, st_n)):
        assert (got - ref).abs().max().item() <= 1e-5 * (ref.abs().max().item() + 1), (got - ref).abs().max().item()
