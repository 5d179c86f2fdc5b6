"""fp4 e2m1 weights (power-of-two scale per 32 columns) in the mixed-table GEMV: store and residual
epilogues and the SwiGLU -> q8 epilogue, against fp64 products of the dequantised weights and the
same int8-block activations; a tensor loaded from raw e2m1 / e8m0 bytes decodes bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200 import ops  # noqa: E402
from hawking_b200.ops.mixed import MixedTable, MixedWeight, _pack_lsb, mixed_gemv, mixed_gemv_swiglu  # noqa: E402

DEV = "cuda"


def _x(nb, K, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = ops.Q8Act(nb, K, DEV)
    ops.rmsnorm_q8(torch.randn(nb, K, device=DEV, generator=g), None, 0.0, x, norm=False)
    xd = (x.q.view(nb, K // 32, 32).float() * x.d.view(nb, K // 32, 1)).view(nb, K)
    return x, xd


@pytest.mark.parametrize("N,K,nb", [(96, 512, 1), (256, 1024, 4), (40, 256, 8)])
def test_fp4_gemv(N, K, nb):
    g = torch.Generator(device=DEV).manual_seed(N + K)
    w = MixedWeight.quantize_fp4(torch.randn(N, K, device=DEV, generator=g) * 0.05)
    t = MixedTable([w])
    x, xd = _x(nb, K, N)
    y = torch.zeros(nb, N, device=DEV)
    mixed_gemv(t, 0, x, y)
    r = torch.full((nb, N), 0.5, device=DEV)
    mixed_gemv(t, 0, x, r, residual=True)
    torch.cuda.synchronize()
    ref = xd.double() @ w.dequantize().double().T
    tol = 1e-4 * ref.abs().max().item() + 1e-6
    assert (y.double() - ref).abs().max().item() <= tol
    assert (r.double() - 0.5 - ref).abs().max().item() <= tol


def test_fp4_swiglu_and_raw_bytes():
    N, K, nb = 256, 512, 3
    g = torch.Generator(device=DEV).manual_seed(7)
    codes = torch.randint(0, 16, (2 * N, K), device=DEV, generator=g, dtype=torch.uint8)
    e = torch.randint(118, 124, (2 * N, K // 32), device=DEV, generator=g, dtype=torch.uint8)
    both = MixedWeight.from_e2m1_e8m0(_pack_lsb(codes, 4), e, 2 * N, K, DEV)
    gw, uw = both.rows(0, N), both.rows(N, N)
    assert torch.equal(gw.codes, _pack_lsb(codes[:N], 4))
    t = MixedTable([gw, uw])
    x, xd = _x(nb, K, 9)
    h = ops.Q8Act(nb, N, DEV)
    mixed_gemv_swiglu(t, 0, 1, x, h)
    torch.cuda.synchronize()
    gv = xd.double() @ gw.dequantize().double().T
    uv = xd.double() @ uw.dequantize().double().T
    ref = gv / (1 + torch.exp(-gv)) * uv
    got = (h.q.view(nb, N // 32, 32).double() * h.d.view(nb, N // 32, 1).double()).view(nb, N)
    assert (got - ref).abs().max().item() <= 1.5e-2 * ref.abs().max().item()
