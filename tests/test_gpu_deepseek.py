"""DeepSeek-V3-style MLA + MoE on the GPU vs the fp32 token-serial oracle with un-absorbed MLA:
latent-cache attention (K6), fp8 e4m3 block-scaled GEMVs (K1), sigmoid + bias group-limited routing
with a shared expert (K3/K4), on a tiny configuration."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def tiny_cfg():
    from hawking_b200.models.config import preset
    return preset("deepseek-v3", vocab=512, hidden=256, layers=3, n_heads=4, n_kv_heads=4, ffn=256, n_experts=8,
                  top_k=2, expert_ffn=128, shared_ffn=128, n_groups=4, topk_groups=2, routed_scale=2.5,
                  first_dense_layers=1, q_lora_rank=128, kv_lora_rank=512, qk_nope_dim=128, qk_rope_dim=64,
                  v_head_dim=128, max_ctx=256)


def test_fp8_gemv_matches_dequantised():
    from hawking_b200.ops import Q8Act, rmsnorm_q8
    from hawking_b200.ops.mixed import MixedTable, MixedWeight, mixed_gemv
    g = torch.Generator(device=DEV).manual_seed(5)
    w = MixedWeight.random_fp8(200, 512, 0.05, g, DEV)
    t = MixedTable([w])
    x = torch.randn(2, 512, generator=g, device=DEV)
    xa = Q8Act(2, 512, DEV)
    rmsnorm_q8(x, None, 1e-5, xa, norm=False)
    y = torch.zeros(2, 200, device=DEV)
    mixed_gemv(t, 0, xa, y)
    ref = xa.dequantize() @ w.dequantize().t()
    torch.testing.assert_close(y, ref, rtol=1e-3, atol=1e-3 * float(ref.abs().max()))


def test_deepseek_matches_torch_oracle():
    from hawking_b200.models.deepseek import DeepSeekModel, LatentCache, TorchRefDeepSeek, random_deepseek_weights
    cfg = tiny_cfg()
    w = random_deepseek_weights(cfg, DEV, seed=2, std=0.05)
    kv = LatentCache(cfg.layers, 32, 16, 2, 16, DEV)
    m = DeepSeekModel(cfg, w, kv, max_rows=8, device=DEV)
    toks = [5, 77, 300, 12, 9, 401, 256, 3, 44, 100]
    got = m.forward_tokens(toks, seq_id=1)
    ref_m = TorchRefDeepSeek(cfg, w)
    ref = torch.stack([ref_m.step(t, p) for p, t in enumerate(toks)])
    err = float((got - ref).abs().max() / ref.abs().max())
    assert err < 0.03, err
    assert int(m.status.item()) == 0


@pytest.mark.parametrize("flash", [False, True])
@pytest.mark.parametrize("nh,rows", [(64, 1), (8, 1), (8, 3), (4, 2), (16, 8)])
def test_mla_decode_head_groupings(nh, rows, flash):
    """Latent-cache attention vs fp32 PyTorch: the CUDA-core kernel for every heads-per-CTA grouping
    (4, 2, 1) and the tensor-core kernel (16 heads per CTA, splits x output slices)."""
    from hawking_b200._ext import kernels
    K = kernels()
    g = torch.Generator(device=DEV).manual_seed(nh * 10 + rows)
    bs, nblk, ctx = 64, 6, 300
    cache = (torch.randn(nblk * rows, bs, 576, generator=g, device=DEV)).bfloat16()
    tables = torch.arange(nblk * rows, dtype=torch.int32, device=DEV).view(rows, nblk).contiguous()
    row_seq = torch.arange(rows, dtype=torch.int32, device=DEV)
    row_ctx = torch.tensor([ctx - 7 * r for r in range(rows)], dtype=torch.int32, device=DEV)
    q_lat = torch.randn(rows, nh, 512, generator=g, device=DEV) * 0.05
    q_pe = torch.randn(rows, nh, 64, generator=g, device=DEV) * 0.05
    o = torch.zeros(rows, nh, 512, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    scale = 192 ** -0.5
    splits = 1
    groups = nh // K.mla_heads_per_cta(nh, rows)
    while splits < 8 and rows * groups * splits < 148:
        splits *= 2
    K.mla_decode(q_lat, q_pe, cache, tables, row_seq, row_ctx, scale, 0 if flash else splits, o, st, False)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for r in range(rows):
        c = cache[tables[r].long()].reshape(-1, 576)[: int(row_ctx[r])].float()
        sc = (q_lat[r] @ c[:, :512].T + q_pe[r] @ c[:, 512:].T) * scale
        ref = torch.softmax(sc, -1) @ c[:, :512]
        tol = 1e-2 if flash else 2e-3  # bf16 query and P on the tensor cores
        torch.testing.assert_close(o[r], ref, rtol=tol, atol=tol)
