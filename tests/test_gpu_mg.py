"""Full-precision (W4A16) tensor-core GEMV against a plain-PyTorch fp64 reference of the same op:
y = dequant(W) @ bf16(x), with dequant from the independent torch restatement of the GGUF formats."""
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


def _close(y, ref, tol=2e-5):
    err = (y.double() - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= tol * scale + 1e-7, (err, scale)


def _status_ok():
    torch.cuda.synchronize()
    assert mg.MgScratch.get(DEV).status.item() == 0


@pytest.mark.parametrize("N,K", [(200, 1024), (16, 256), (4096, 4096), (4096, 14336), (1000, 2560)])
@pytest.mark.parametrize("nb", [1, 2, 3, 8])
def test_mg_store_bf16_input(N, K, nb):
    w = _w(N, K, N + K)
    mw = mg.pack(w)
    xb = _x(nb, K, nb).bfloat16()
    y = torch.full((nb, N), float("nan"), device=DEV)
    if nb * K * 2 > 96 * 1024:  # too wide to stage in shared memory: fragment-order input
        xf = mg.FragAct(K, DEV)
        xf.buf.view(-1)[mg.frag_index(K, nb, xf.cstride, DEV)] = xb.reshape(-1)
        mg.gemv(mw, nb, xfrag=xf, y=y)
    else:
        mg.gemv(mw, nb, xb=xb, y=y)
    _status_ok()
    _close(y, _ref(w, xb))


@pytest.mark.parametrize("nb", [1, 4, 8])
def test_mg_fused_rmsnorm_input_and_residual(nb):
    N, K, eps = 512, 4096, 1e-5
    w = _w(N, K, 7)
    mw = mg.pack(w)
    x = _x(nb, K, 3, scale=3.0)
    nw = torch.rand(K, device=DEV) + 0.5
    xn = (x * torch.rsqrt((x * x).mean(1, keepdim=True) + eps) * nw).bfloat16()
    y0 = torch.randn(nb, N, device=DEV)
    y = y0.clone()
    mg.gemv(mw, nb, x_norm=(x, nw, eps), y=y, residual=True)
    _status_ok()
    # the kernel's own reduction order may round a few elements of x to the neighbouring bf16 value
    _close(y - y0, _ref(w, xn), tol=2e-3)


def test_mg_swiglu_then_fragment_input():
    F, H, nb = 512, 1024, 3
    wg, wu = _w(F, H, 11, 0.05), _w(F, H, 12, 0.05)
    wgu = cat_rows([wg, wu])
    mgu = mg.pack(wgu, swiglu=F)
    wd = _w(H, F, 13)
    md = mg.pack(wd)
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
    mg.gemv(md, nb, xfrag=hf, y=y)
    _status_ok()
    _close(y, _ref(wd, hb))


def test_mg_swiglu_gpu_sized_fixup():
    """Llama-3-8B gate/up shape: every row group split across warps (deterministic fix-up)."""
    F, H, nb = 14336, 4096, 1
    wgu = _w(2 * F, H, 21)
    mgu = mg.pack(wgu, swiglu=F)
    xb = _x(nb, H, 6).bfloat16()
    hb = torch.zeros(nb, F, dtype=torch.bfloat16, device=DEV)
    mg.gemv(mgu, nb, xb=xb, hb=hb)
    _status_ok()
    gu = _ref(wgu, xb)
    g, u = gu[:, :F], gu[:, F:]
    _close(hb.float(), g / (1 + torch.exp(-g)) * u, tol=8e-3)


def test_mg_deterministic_and_repeatable():
    N, K, nb = 4096, 14336, 2
    w = _w(N, K, 31)
    mw = mg.pack(w)
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


def test_mg_fused_argmax():
    from hawking_b200 import ops
    V, K, nb = 5000, 2048, 3
    w = _w(V, K, 41, 0.05)
    mw = mg.pack(w)
    xb = _x(nb, K, 2).bfloat16()
    y = torch.zeros(nb, V, device=DEV)
    slots = torch.zeros(nb, ops.ARGMAX_SLOTS, dtype=torch.int64, device=DEV)
    ids = torch.zeros(nb, dtype=torch.int32, device=DEV)
    mg.gemv(mw, nb, xb=xb, y=y, argmax_slots=slots)
    ops.argmax_finalize(slots, nb, ids)
    _status_ok()
    assert torch.equal(ids.long().cpu(), y.argmax(1).cpu())
    _close(y, _ref(w, xb))


def test_mg_in_cuda_graph():
    N, K, nb = 1024, 4096, 1
    w = _w(N, K, 51)
    mw = mg.pack(w)
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
