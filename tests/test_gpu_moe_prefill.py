"""Prefill kernels of the mixed-codec MoE path: table -> bf16 decode for every kind, the bf16-weight
tcgen05 GEMM (plain, split-K, SwiGLU epilogue) and its grouped form over device-built tiles, the
gather and the deterministic combine, against fp32 PyTorch."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200._ext import kernels  # noqa: E402
from hawking_b200.ops.mixed import BINARY, UNIFORM, MixedTable, MixedWeight  # noqa: E402

DEV = "cuda"


def _g(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def test_table_decode_to_bf16_every_kind():
    g = _g(1)
    w = torch.randn(64, 512, generator=g, device=DEV) * 0.05
    ws = [MixedWeight.quantize(w, BINARY, 1), MixedWeight.quantize(w, UNIFORM, 2), MixedWeight.quantize(w, UNIFORM, 4),
          MixedWeight.quantize(w, UNIFORM, 8), MixedWeight.quantize_fp8(w), MixedWeight.quantize_fp4(w)]
    t = MixedTable(ws)
    out = torch.zeros(64 * len(ws), 512, dtype=torch.bfloat16, device=DEV)
    didx = torch.arange(len(ws), dtype=torch.int32, device=DEV)
    drow = didx * 64
    kernels().mixed_dequant_bf16(t.descs, didx, drow, 64, 512, out)
    torch.cuda.synchronize()
    for i, mw in enumerate(ws):
        ref = mw.dequantize().float()
        got = out[64 * i:64 * (i + 1)].float()
        assert (got - ref).abs().max().item() <= 8e-3 * ref.abs().max().item() + 1e-7, i


@pytest.mark.parametrize("N,K,M,bn,splits", [(256, 512, 96, 64, 1), (384, 1024, 40, 32, 4), (128, 256, 300, 128, 1)])
def test_bf16_gemm_plain(N, K, M, bn, splits):
    g = _g(N + K)
    w = (torch.randn(N, K, generator=g, device=DEV) * 0.05).bfloat16()
    x = torch.randn(M, K, generator=g, device=DEV).bfloat16()
    y = torch.zeros(M, N, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels().tc_gemm_bf16(w, x, N, M, y=y, y_zeroed=True, k_splits=splits, bn=bn, status=st)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().T
    assert int(st.item()) == 0
    assert (y - ref).abs().max().item() <= 1e-3 * ref.abs().max().item()


def test_bf16_gemm_swiglu():
    g = _g(7)
    F, K, M = 256, 512, 72
    w = (torch.randn(2 * F, K, generator=g, device=DEV) * 0.05).bfloat16()
    x = torch.randn(M, K, generator=g, device=DEV).bfloat16()
    h = torch.zeros(M, F, dtype=torch.bfloat16, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels().tc_gemm_bf16(w, x, 2 * F, M, h=h, bn=64, status=st)
    torch.cuda.synchronize()
    gu = x.float() @ w.float().T
    ref = torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
    assert (h.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_grouped_experts_pipeline():
    """Routing -> tiles -> gather -> grouped gate|up (SwiGLU) -> grouped down -> combine, vs a
    per-token fp32 loop over the same bf16 weights."""
    from hawking_b200 import ops
    g = _g(11)
    E, F, H, T, k = 8, 128, 256, 37, 2
    wgu = (torch.randn(E * 2 * F, H, generator=g, device=DEV) * 0.05).bfloat16()
    wdn = (torch.randn(E * H, F, generator=g, device=DEV) * 0.05).bfloat16()
    xb = torch.randn(T, H, generator=g, device=DEV).bfloat16()
    logits = torch.randn(T, E, generator=g, device=DEV)
    ids = torch.zeros(T, k, dtype=torch.int32, device=DEV)
    rw = torch.zeros(T, k, device=DEV)
    ops.moe_topk(logits, None, k, 0, 1, 1, True, 1.0, ids, rw)
    counts = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    offsets = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    sorted_pairs = torch.zeros(T * k + T, dtype=torch.int32, device=DEV)
    xa = ops.Q8Act(T, H, DEV)
    gx = ops.Q8Act(T * k + T, H, DEV)
    ops.moe_align(ids, E, xa, counts, offsets, sorted_pairs, gx)
    K = kernels()
    BN = 64
    tiles = torch.zeros(3 * ((T * k) // BN + E + 1), dtype=torch.int32, device=DEV)
    n_tiles = torch.zeros(1, dtype=torch.int32, device=DEV)
    K.moe_tiles(counts, offsets, E, BN, tiles, n_tiles)
    P = T * k
    xg = torch.zeros(P, H, dtype=torch.bfloat16, device=DEV)
    pos = torch.zeros(P, dtype=torch.int32, device=DEV)
    K.moe_gather_bf16(sorted_pairs, P, P, k, xb, xg, pos)
    h = torch.zeros(P, F, dtype=torch.bfloat16, device=DEV)
    y = torch.zeros(P, H, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    mt = tiles.numel() // 3
    K.tc_gemm_bf16(wgu, xg, 2 * F, P, h=h, bn=BN, status=st, tiles=tiles, n_tiles=n_tiles, max_tiles=mt,
                   group_rows=2 * F)
    K.tc_gemm_bf16(wdn, h, H, P, y=y, bn=BN, status=st, tiles=tiles, n_tiles=n_tiles, max_tiles=mt, group_rows=H)
    x = torch.zeros(T, H, device=DEV)
    K.moe_combine(y, pos, rw, T, k, False, None, x)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ref = torch.zeros(T, H, device=DEV)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            gu = wgu[e * 2 * F:(e + 1) * 2 * F].float() @ xb[t].float()
            hh = (torch.nn.functional.silu(gu[:F]) * gu[F:]).bfloat16().float()
            ref[t] += rw[t, j] * (wdn[e * H:(e + 1) * H].float() @ hh)
    assert (x - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()


@pytest.mark.parametrize("fmt", [8, 2, 6, 12, 14])  # Q8_0, Q4_0, Q5_0, Q4_K, Q6_K
def test_gguf_blocks_decode_to_bf16(fmt):
    """GGUF planes of a stacked two-expert tensor -> bf16 rows in the [gate | up] per-expert layout
    (gate rows at 2F e, up rows at 2F e + F), against the PyTorch restatement of the format."""
    from hawking_b200.ops import QWeight
    g = _g(fmt)
    F, K = 64, 512
    gate = QWeight.quantize(torch.randn(2 * F, K, generator=g, device=DEV) * 0.05, fmt)
    up = QWeight.quantize(torch.randn(2 * F, K, generator=g, device=DEV) * 0.05, fmt)
    out = torch.zeros(4 * F, K, dtype=torch.bfloat16, device=DEV)
    kernels().qweight_dequant_bf16(gate.fmt, gate.planes, K, F, 2 * F, 0, out)
    kernels().qweight_dequant_bf16(up.fmt, up.planes, K, F, 2 * F, F, out)
    torch.cuda.synchronize()
    gd, ud = gate.dequantize(), up.dequantize()
    for e in range(2):
        for src, off in ((gd, 0), (ud, F)):
            ref = src[e * F:(e + 1) * F]
            got = out[2 * F * e + off:2 * F * e + off + F].float()
            assert (got - ref).abs().max().item() <= 8e-3 * ref.abs().max().item() + 1e-7, (fmt, e, off)
