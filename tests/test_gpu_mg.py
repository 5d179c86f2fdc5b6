"""Full-precision (W4A16) tensor-core GEMV against a plain-PyTorch fp64 reference of the same op:
y = dequant(W) @ x, with dequant from the independent torch restatement of the GGUF formats.

Both math modes: "bf16" (activations rounded to bf16) and "int" (activations as 16-bit fixed point
per 32-element block, at most 1/64516 of the block's largest magnitude off)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200.formats.ggml import GgmlType  # noqa: E402
from hawking_b200.ops import QWeight, cat_rows  # noqa: E402
from hawking_b200.ops import mg  # noqa: E402

DEV = "cuda"


def _w(N, K, seed, std=0.02):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return QWeight.quantize(torch.randn(N, K, device=DEV, generator=g) * std, GgmlType.Q4_K)


def _x(nb, K, seed, scale=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed + 1000)
    return torch.randn(nb, K, device=DEV, generator=g) * scale


def _ref(w: QWeight, xb: torch.Tensor) -> torch.Tensor:
    return xb.double() @ w.dequantize().double().T


MATHS = ["int", "bf16"]
TOL = {"int": 2e-4, "bf16": 2e-5}  # the int math also rounds the (already bf16) input to its grid


def _close(y, ref, tol=2e-5):
    err = (y.double() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= tol * scale + 1e-7, (err, scale)


def _status_ok():
    torch.cuda.synchronize()
    assert mg.MgScratch.get(DEV).status.item() == 0


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("N,K", [(200, 1024), (16, 256), (4096, 4096), (4096, 14336), (1000, 2560)])
@pytest.mark.parametrize("nb", [1, 2, 3, 8])
def test_mg_store_bf16_input(N, K, nb, math):
    w = _w(N, K, N + K)
    mw = mg.pack(w, math=math)
    xb = _x(nb, K, nb).bfloat16()
    y = torch.full((nb, N), float("nan"), device=DEV)
    if nb * K * 2 > 96 * 1024:  # too wide to stage in shared memory: fragment-order input
        if math == "bf16":
            xf = mg.FragAct(K, DEV)
            xf.buf.view(-1)[mg.frag_index(K, nb, xf.cstride, DEV)] = xb.reshape(-1)
        else:
            xf = mg.IntFragAct(K, DEV)
            mg.quantize(xb, nb, xf)
        mg.gemv(mw, nb, xfrag=xf, y=y)
    else:
        mg.gemv(mw, nb, xb=xb, y=y)
    _status_ok()
    _close(y, _ref(w, xb), TOL[math])


@pytest.mark.parametrize("nb", [1, 3])
def test_mg_int_math_at_least_as_accurate_as_bf16(nb):
    """Against fp64 on the unrounded fp32 activations, the integer math's error is no larger than
    the bf16 math's (16-bit fixed point per block vs bf16 per element)."""
    N, K = 2048, 4096
    w = _w(N, K, 77)
    x = _x(nb, K, 8)
    exact = x.double() @ w.dequantize().double().T
    errs = {}
    for math in MATHS:
        y = torch.zeros(nb, N, device=DEV)
        mg.gemv(mg.pack(w, math=math), nb, x_norm=(x, None, 0.0), y=y)
        _status_ok()
        xs = x * torch.rsqrt((x * x).mean(1, keepdim=True))
        ref = xs.double() @ w.dequantize().double().T
        errs[math] = (y.double() - ref).abs().max().item() / ref.abs().max().item()
    assert errs["int"] <= errs["bf16"], errs
    assert errs["int"] < 1e-4, errs
    del exact


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("nb", [1, 4, 8])
def test_mg_fused_rmsnorm_input_and_residual(nb, math):
    N, K, eps = 512, 4096, 1e-5
    w = _w(N, K, 7)
    mw = mg.pack(w, math=math)
    x = _x(nb, K, 3, scale=3.0)
    nw = torch.rand(K, device=DEV) + 0.5
    xn = x * torch.rsqrt((x * x).mean(1, keepdim=True) + eps) * nw
    y0 = torch.randn(nb, N, device=DEV)
    y = y0.clone()
    mg.gemv(mw, nb, x_norm=(x, nw, eps), y=y, residual=True)
    _status_ok()
    if math == "bf16":  # its reduction order may round a few elements to the neighbouring bf16 value
        _close(y - y0, _ref(w, xn.bfloat16()), tol=2e-3)
    else:  # the integer math quantises the fp32 normalised values
        _close(y - y0, _ref(w, xn), tol=2e-4)


@pytest.mark.parametrize("math", MATHS)
def test_mg_swiglu_then_fragment_input(math):
    F, H, nb = 512, 1024, 3
    wg, wu = _w(F, H, 11, 0.05), _w(F, H, 12, 0.05)
    wgu = cat_rows([wg, wu])
    mgu = mg.pack(wgu, swiglu=F, math=math)
    wd = _w(H, F, 13)
    md = mg.pack(wd, math=math)
    xb = _x(nb, H, 5).bfloat16()
    hf = mg.FragAct(F, DEV)
    hb = torch.zeros(nb, F, dtype=torch.bfloat16, device=DEV)
    mg.gemv(mgu, nb, xb=xb, hfrag=hf, hb=hb)
    _status_ok()
    g = _ref(wg, xb)
    u = _ref(wu, xb)
    _close(hb.float(), g / (1 + torch.exp(-g)) * u, tol=8e-3)  # bf16 output rounding
    assert torch.equal(hf.to_plain(nb), hb)  # both outputs carry the same bf16 values
    y = torch.zeros(nb, H, device=DEV)
    if math == "bf16":
        mg.gemv(md, nb, xfrag=hf, y=y)
    else:
        xi = mg.IntFragAct(F, DEV)
        mg.quantize(hb, nb, xi)
        mg.gemv(md, nb, xfrag=xi, y=y)
        y2 = torch.zeros(nb, H, device=DEV)
        mg.gemv(md, nb, xb=hb, y=y2)  # staged and quantised inside the GEMV: the same numbers
        _status_ok()
        assert torch.equal(y, y2)
    _status_ok()
    _close(y, _ref(wd, hb), TOL[math])


@pytest.mark.parametrize("math", MATHS)
def test_mg_swiglu_gpu_sized_fixup(math):
    """Llama-3-8B gate/up shape: every row group split across warps (deterministic fix-up)."""
    F, H, nb = 14336, 4096, 1
    wgu = _w(2 * F, H, 21)
    mgu = mg.pack(wgu, swiglu=F, math=math)
    xb = _x(nb, H, 6).bfloat16()
    hb = torch.zeros(nb, F, dtype=torch.bfloat16, device=DEV)
    mg.gemv(mgu, nb, xb=xb, hb=hb)
    _status_ok()
    gu = _ref(wgu, xb)
    g, u = gu[:, :F], gu[:, F:]
    _close(hb.float(), g / (1 + torch.exp(-g)) * u, tol=8e-3)


@pytest.mark.parametrize("math", MATHS)
def test_mg_deterministic_and_repeatable(math):
    N, K, nb = 4096, 14336, 2
    w = _w(N, K, 31)
    mw = mg.pack(w, math=math)
    xb = _x(nb, K, 9).bfloat16()
    outs = []
    for _ in range(4):
        y = torch.zeros(nb, N, device=DEV)
        mg.gemv(mw, nb, xb=xb, y=y)
        outs.append(y)
    _status_ok()
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert int(mg.MgScratch.get(DEV).counters.abs().sum().item()) == 0  # every counter cleared


@pytest.mark.parametrize("math", MATHS)
def test_mg_fused_argmax(math):
    from hawking_b200 import ops
    V, K, nb = 5000, 2048, 3
    w = _w(V, K, 41, 0.05)
    mw = mg.pack(w, math=math)
    xb = _x(nb, K, 2).bfloat16()
    y = torch.zeros(nb, V, device=DEV)
    slots = torch.zeros(nb, ops.ARGMAX_SLOTS, dtype=torch.int64, device=DEV)
    ids = torch.zeros(nb, dtype=torch.int32, device=DEV)
    mg.gemv(mw, nb, xb=xb, y=y, argmax_slots=slots)
    ops.argmax_finalize(slots, nb, ids)
    _status_ok()
    assert torch.equal(ids.long().cpu(), y.argmax(1).cpu())
    _close(y, _ref(w, xb), TOL[math])


@pytest.mark.parametrize("math", MATHS)
def test_mg_in_cuda_graph(math):
    N, K, nb = 1024, 4096, 1
    w = _w(N, K, 51)
    mw = mg.pack(w, math=math)
    x = _x(nb, K, 4)
    y = torch.zeros(nb, N, device=DEV)
    mg.gemv(mw, nb, x_norm=(x, None, 1e-6), y=y)  # warm-up outside the graph
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        mg.gemv(mw, nb, x_norm=(x, None, 1e-6), y=y)
    for s in range(3):
        x.copy_(_x(nb, K, 100 + s))
        g.replay()
        torch.cuda.synchronize()
        xn = (x * torch.rsqrt((x * x).mean(1, keepdim=True) + 1e-6)).bfloat16()
        _close(y, _ref(w, xn), tol=2e-3)
    _status_ok()


@pytest.mark.parametrize("math", MATHS)
@pytest.mark.parametrize("hd,rot,style,nb", [(128, 128, 0, 1), (128, 128, 1, 3), (64, 64, 0, 8), (128, 64, 1, 2)])
def test_mg_rope_epilogue_matches_store_then_rope(hd, rot, style, nb, math):
    """QKV packed in RoPE-pair order: the fused epilogue (bias, RoPE, q out, paged K/V append) equals
    the logical-order store followed by the stand-alone rope_append kernel."""
    from hawking_b200 import ops
    nh, nkv, H, bs = 8, 2, 1024, 16
    N = (nh + 2 * nkv) * hd
    w = _w(N, H, hd + rot + style)
    mw = mg.pack(w, math=math, rope=(nh + nkv, hd, rot, style))
    x = _x(nb, H, 12)
    nw = torch.rand(H, device=DEV) + 0.5
    bias = torch.randn(N, device=DEV) * 0.1
    rope = ops.rope_table(512, rot, 10000.0, None, DEV)
    positions = torch.tensor([5 + 37 * i for i in range(nb)], dtype=torch.int32, device=DEV)
    row_seq = torch.arange(nb, dtype=torch.int32, device=DEV)
    mb = 20  # table columns: 20 blocks of 16 cover the largest position (5 + 37 * 7 = 264)
    nblk = nb * mb + 4
    tables = torch.randperm(nblk, device=DEV)[: nb * mb].int().view(nb, mb).contiguous()
    outs = []
    for fused in (False, True):
        kc = torch.zeros(nblk, nkv, bs, hd, dtype=torch.bfloat16, device=DEV)
        vc = torch.zeros_like(kc)
        q = torch.zeros(nb, nh, hd, device=DEV)
        y = torch.zeros(nb, N, device=DEV)
        if fused:
            mg.gemv(mw, nb, x_norm=(x, nw, 1e-5), y=y, bias=bias,
                    rope_append=(rope, positions, row_seq, tables, kc, vc, q, nh, nkv, bs))
        else:
            mg.gemv(mw, nb, x_norm=(x, nw, 1e-5), y=y)  # logical rows (the store epilogue unpermutes)
            ops.rope_append(y, positions, None, rope, rot, style, q, kc, vc, nh, nkv, hd, bs, bias=bias,
                            block_tables=tables, row_seq=row_seq)
        _status_ok()
        outs.append((q, kc.float(), vc.float()))
    for a, b in zip(outs[0], outs[1]):
        err = (a - b).abs().max().item()
        assert err <= 1e-2 * b.abs().max().item() + 1e-6, err
