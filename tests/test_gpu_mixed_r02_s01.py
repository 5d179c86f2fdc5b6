"""HGRAVR02 (binary + Rice-coded outlier residual) and HGRAVS01 (low-rank) on the GPU: y = W x from
the device planes (base GEMV + CSR residual kernel; two factor GEMVs) against the C++ CPU decode of
the same payload times the same int8-block activations, in fp64."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200 import ops  # noqa: E402
from hawking_b200._ext import native  # noqa: E402
from hawking_b200.formats import mixed as mx  # noqa: E402
from hawking_b200.ops.mixed import LowRankWeight, RiceResidualWeight, mixed_linear  # noqa: E402

DEV = "cuda"


def _x(nb, K, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = ops.Q8Act(nb, K, DEV)
    ops.rmsnorm_q8(torch.randn(nb, K, device=DEV, generator=g), None, 0.0, x, norm=False)
    xd = (x.q.view(nb, K // 32, 32).float() * x.d.view(nb, K // 32, 1)).view(nb, K)
    return x, xd


@pytest.mark.parametrize("N,K,nb", [(96, 512, 1), (200, 1024, 3), (64, 2048, 8)])
def test_r02_matches_cpu_decode(N, K, nb):
    rng = np.random.default_rng(N + K)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    w[rng.random((N, K)) < 0.01] *= 12.0  # outliers for the residual
    payload = mx.encode_binary_residual(w, group=128, ratio=0.02, rice_k=5)
    dense = torch.from_numpy(mx.decode(payload)).double().to(DEV)
    rw = RiceResidualWeight.from_payload(payload, DEV)
    assert rw.cols.numel() > 0
    assert torch.allclose(rw.dequantize().double(), dense, atol=1e-6)
    x, xd = _x(nb, K, N)
    y = torch.zeros(nb, N, device=DEV)
    mixed_linear(rw, x, y)
    torch.cuda.synchronize()
    ref = xd.double() @ dense.T
    assert (y.double() - ref).abs().max().item() <= 1e-4 * ref.abs().max().item() + 1e-6


@pytest.mark.parametrize("N,K,rank,nb", [(128, 512, 64, 1), (256, 1024, 128, 4)])
def test_s01_matches_cpu_decode(N, K, rank, nb):
    rng = np.random.default_rng(N + rank)
    L = (rng.standard_normal((N, rank)) * 0.1).astype(np.float32)
    R = (rng.standard_normal((rank, K)) * 0.1).astype(np.float32)
    payload = mx.encode_low_rank(L, R, bits=4, group=64)
    dense = torch.from_numpy(mx.decode(payload)).double().to(DEV)
    lw = LowRankWeight.from_payload(payload, DEV)
    assert torch.allclose(lw.dequantize().double(), dense, rtol=1e-4, atol=1e-5)
    x, xd = _x(nb, K, rank)
    y = torch.zeros(nb, N, device=DEV)
    mixed_linear(lw, x, y)
    torch.cuda.synchronize()
    ref = xd.double() @ dense.T
    # the rank-wide intermediate is re-quantised to int8 blocks between the two GEMVs
    assert (y.double() - ref).abs().max().item() <= 2e-2 * ref.abs().max().item()
