"""tcgen05 dequant GEMM (Q4_K x bf16 -> fp32) against a plain-PyTorch fp32 reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200 import ops  # noqa: E402
from hawking_b200.formats.ggml import GgmlType  # noqa: E402
from hawking_b200.ops import QWeight  # noqa: E402

DEV = "cuda"


def _case(N, K, M, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = QWeight.quantize(torch.randn(N, K, device=DEV, generator=g) * 0.02, GgmlType.Q4_K)
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    ref = x.float() @ w.dequantize().T
    return w, x, ref


def _check(y, ref):
    err = (y - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= 1.5e-2 * scale, (err, scale)


@pytest.mark.parametrize("M,bn", [(1, 32), (16, 32), (64, 64), (100, 128), (130, 64), (300, 256), (256, 256)])
def test_tc_gemm_store(M, bn):
    w, x, ref = _case(256, 1024, M, M + bn)
    y = torch.zeros(M, 256, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.tc_gemm(w, x, y, st, bn=bn, k_splits=1)
    torch.cuda.synchronize()
    assert st.item() == 0
    _check(y, ref)


@pytest.mark.parametrize("splits", [2, 3, 8])
def test_tc_gemm_split_k_atomic(splits):
    w, x, ref = _case(384, 2048, 48, splits)
    y0 = torch.randn(48, 384, device=DEV)
    y = y0.clone()
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.tc_gemm(w, x, y, st, atomic=True, k_splits=splits, bn=64)
    torch.cuda.synchronize()
    assert st.item() == 0
    _check(y - y0, ref)


def test_tc_gemm_strided_output_and_swiglu():
    F, K, M = 256, 512, 8
    g = torch.Generator(device=DEV).manual_seed(9)
    wg = QWeight.quantize(torch.randn(F, K, device=DEV, generator=g) * 0.05, GgmlType.Q4_K)
    wu = QWeight.quantize(torch.randn(F, K, device=DEV, generator=g) * 0.05, GgmlType.Q4_K)
    w = ops.cat_rows([wg, wu])
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    gu = torch.zeros(M, 2 * F, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.tc_gemm(w, x, gu, st, y_zeroed=True, k_splits=2)
    h = torch.zeros(M, F, device=DEV, dtype=torch.bfloat16)
    ops.swiglu_bf16(gu, F, h)
    torch.cuda.synchronize()
    xf = x.float()
    ref = torch.nn.functional.silu(xf @ wg.dequantize().T) * (xf @ wu.dequantize().T)
    _check(h.float(), ref)
    assert gu.abs().max().item() == 0.0  # consumed and cleared


def test_tc_gemm_large_n_covers_grid():
    w, x, ref = _case(128 * 40, 4096, 64, 77)
    y = torch.zeros(64, 128 * 40, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.tc_gemm(w, x, y, st, y_zeroed=True)
    torch.cuda.synchronize()
    assert st.item() == 0
    _check(y, ref)


@pytest.mark.parametrize("M,bn", [(100, 128), (300, 256), (64, 64)])
def test_tc_gemm_swiglu_epilogue(M, bn):
    """Fused [gate | up] GEMM with the SwiGLU in the epilogue vs the fp32 reference."""
    from hawking_b200.ops import cat_rows
    F, K = 192, 512
    g = torch.Generator(device=DEV).manual_seed(M)
    wg = QWeight.quantize(torch.randn(F, K, device=DEV, generator=g) * 0.05, GgmlType.Q4_K)
    wu = QWeight.quantize(torch.randn(F, K, device=DEV, generator=g) * 0.05, GgmlType.Q4_K)
    w = cat_rows([wg, wu])
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    gt, up = x.float() @ wg.dequantize().T, x.float() @ wu.dequantize().T
    ref = gt / (1 + torch.exp(-gt)) * up
    h = torch.zeros(M, F, dtype=torch.bfloat16, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.tc_gemm_swiglu(w, x, h, st, bn=bn)
    torch.cuda.synchronize()
    assert st.item() == 0
    _check(h.float(), ref)


@pytest.mark.parametrize("pair", ["0", "1"])
@pytest.mark.parametrize("M,N,swiglu", [(300, 512, False), (1000, 384, False), (520, 384, True), (257, 256, True),
                                        (1000, 1024, False), (520, 512, True), (600, 8192, False)])
def test_tc_gemm_persistent(M, N, swiglu, pair, monkeypatch):
    """Persistent tcgen05 GEMM (tiles looped per CTA, double-buffered TMEM accumulators), plain
    store and fused SwiGLU epilogues, more tiles than CTAs and a ragged last token tile; with
    pair=1 the CTA-pair (cta_group::2) kernel takes the shapes made of whole 256-row pair tiles
    (N % 256, or F % 128 under SwiGLU), including more pair tiles than resident pairs."""
    from hawking_b200.ops import cat_rows
    monkeypatch.setenv("HK_GEMM_PAIR", pair)
    K = 512
    g = torch.Generator(device=DEV).manual_seed(M + N)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    if swiglu:
        F = N // 2
        wg = QWeight.quantize(torch.randn(F, K, device=DEV, generator=g) * 0.05, GgmlType.Q4_K)
        wu = QWeight.quantize(torch.randn(F, K, device=DEV, generator=g) * 0.05, GgmlType.Q4_K)
        gt, up = x.float() @ wg.dequantize().T, x.float() @ wu.dequantize().T
        ref = gt / (1 + torch.exp(-gt)) * up
        h = torch.zeros(M, F, dtype=torch.bfloat16, device=DEV)
        ops.tc_gemm_swiglu(cat_rows([wg, wu]), x, h, st, bn=256)
        out = h.float()
    else:
        w = QWeight.quantize(torch.randn(N, K, device=DEV, generator=g) * 0.02, GgmlType.Q4_K)
        ref = x.float() @ w.dequantize().T
        out = torch.zeros(M, N, device=DEV)
        ops.tc_gemm(w, x, out, st, bn=256)
    torch.cuda.synchronize()
    assert st.item() == 0
    _check(out, ref)


@pytest.mark.parametrize("pair", ["0", "1"])
def test_tc_gemm_persistent_repeated_multi_tile(pair, monkeypatch):
    """Many tiles per CTA, repeated launches: every run matches the reference (a slot released
    before its shared-memory loads completed once corrupted rows of a CTA's second tile in about
    one run in four)."""
    monkeypatch.setenv("HK_GEMM_PAIR", pair)
    M, N, K = 600, 8192, 512
    g = torch.Generator(device=DEV).manual_seed(7)
    x = torch.randn(M, K, device=DEV, generator=g).bfloat16()
    w = QWeight.quantize(torch.randn(N, K, device=DEV, generator=g) * 0.02, GgmlType.Q4_K)
    ref = x.float() @ w.dequantize().T
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(12):
        out = torch.zeros(M, N, device=DEV)
        ops.tc_gemm(w, x, out, st, bn=256)
        torch.cuda.synchronize()
        assert st.item() == 0
        _check(out, ref)


@pytest.mark.parametrize("M,N,K", [(64, 19200, 2304), (17, 28672, 1024), (1, 20480, 512)])
@pytest.mark.parametrize("residual", [False, True])
def test_tc_gemm_stream_k(M, N, K, residual):
    """Stream-K decode-batch GEMM: each CTA takes a balanced range of (weight tile, K stage) units
    that may start and end inside tiles (150 tiles x 18 stages over 148 CTAs, ...), the partial
    tiles accumulated with atomics into a zeroed output or onto a residual."""
    assert ops.tc_gemm_stream_k(M, N)
    w, x, ref = _case(N, K, M, N + K + M)
    y0 = torch.randn(M, N, device=DEV) if residual else torch.zeros(M, N, device=DEV)
    y = y0.clone()
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    if residual:
        ops.tc_gemm(w, x, y, st, atomic=True)
    else:
        ops.tc_gemm(w, x, y, st, y_zeroed=True)
    torch.cuda.synchronize()
    assert st.item() == 0
    _check(y - y0, ref)


@pytest.mark.parametrize("M,F,clear", [(300, 14336, False), (5, 512, True), (7, 250, True)])
def test_swiglu_bf16_kernel(M, F, clear):
    """h = silu(g) * u as bf16 from the fp32 [g | u] rows (four columns per thread when F and the
    rows are 16-byte aligned, one otherwise); ``clear`` re-zeroes the rows it read."""
    g = torch.Generator(device=DEV).manual_seed(M + F)
    gu = torch.randn(M, 2 * F, device=DEV, generator=g)
    ref = (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]).bfloat16().float()
    h = torch.zeros(M, F, dtype=torch.bfloat16, device=DEV)
    src = gu.clone()
    ops.swiglu_bf16(src, F, h, clear=clear)
    torch.cuda.synchronize()
    assert (h.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    if clear:
        assert not src.any()
    else:
        assert torch.equal(src, gu)
