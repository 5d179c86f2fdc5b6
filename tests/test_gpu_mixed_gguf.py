"""GGUF tensors as mixed-table weights on the GPU (``MixedWeight.from_gguf``): the dense GEMV (store
and residual epilogues) and the SwiGLU -> q8 epilogue over Q4_K planes, Q8_0 / Q4_0 as uniform
codes and re-encoded Q6_K / F16, against fp64 products of the dequantised file tensor and the
same int8-block activations."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200 import ops  # noqa: E402
from hawking_b200.formats.ggml import GgmlType  # noqa: E402
from hawking_b200.formats.gguf import GgufBuilder, GgufModel  # noqa: E402
from hawking_b200.ops.mixed import MixedTable, MixedWeight, mixed_gemv, mixed_gemv_swiglu  # noqa: E402

DEV = "cuda"
FMTS = [GgmlType.Q4_K, GgmlType.Q8_0, GgmlType.Q4_0, GgmlType.Q6_K, GgmlType.F16]


def _tensor(tmp_path, fmt, N, K, seed, name="w"):
    rng = np.random.default_rng(seed)
    a = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    b = GgufBuilder("llama")
    b.add(name, a, fmt)
    m = GgufModel(b.write(str(tmp_path / f"{name}{seed}.gguf")))
    raw = torch.from_numpy(np.array(m.raw(name)))
    return MixedWeight.from_gguf(raw, fmt, N, K, DEV), torch.from_numpy(m.dequantize(name).reshape(N, K).copy())


def _x(nb, K, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = ops.Q8Act(nb, K, DEV)
    ops.rmsnorm_q8(torch.randn(nb, K, device=DEV, generator=g), None, 0.0, x, norm=False)
    xd = (x.q.view(nb, K // 32, 32).float() * x.d.view(nb, K // 32, 1)).view(nb, K)
    return x, xd


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("N,K,nb", [(96, 512, 1), (256, 1024, 4), (40, 256, 8)])
def test_gemv_over_gguf_tensor(tmp_path, fmt, N, K, nb):
    w, dense = _tensor(tmp_path, fmt, N, K, N + K)
    if fmt in (GgmlType.Q4_K, GgmlType.Q8_0, GgmlType.Q4_0):
        assert torch.equal(w.dequantize().cpu(), dense)  # the file's values, bit for bit
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


@pytest.mark.parametrize("fmt", FMTS)
def test_swiglu_over_gguf_tensors(tmp_path, fmt):
    N, K, nb = 256, 512, 3
    g, _ = _tensor(tmp_path, fmt, N, K, 7, "g")
    u, _ = _tensor(tmp_path, fmt, N, K, 8, "u")
    t = MixedTable([g, u])
    x, xd = _x(nb, K, 9)
    h = ops.Q8Act(nb, N, DEV)
    mixed_gemv_swiglu(t, 0, 1, x, h)
    torch.cuda.synchronize()
    gv = xd.double() @ g.dequantize().double().T
    uv = xd.double() @ u.dequantize().double().T
    ref = gv / (1 + torch.exp(-gv)) * uv
    got = (h.q.view(nb, N // 32, 32).double() * h.d.view(nb, N // 32, 1).double()).view(nb, N)
    assert (got - ref).abs().max().item() <= 1.5e-2 * ref.abs().max().item()
