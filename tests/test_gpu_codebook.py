"""GPU GEMVs of the fixed-header `.gravity` codecs against the fp32 dense decode of the same
payload (C++ decoder): PQ, residual PQ, activation-aware low rank, HQ30 binary / uniform Q4 and
binary + sparse residual, with 1 and 3 activation columns."""
import numpy as np
import pytest
import torch

from hawking_b200.formats import codecs
from hawking_b200.ops import Q8Act, rmsnorm_q8
from hawking_b200.ops.codebook import gravity_weight

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _payloads(rng):
    cb = rng.standard_normal((4, 64, 2)).astype(np.float16)
    idx = rng.integers(0, 64, size=(96, 32, 4))
    yield "pq", codecs.encode_pq(cb, idx, bits=6)
    rcb = (rng.standard_normal((3, 16, 8)) * 0.5).astype(np.float16)
    ridx = rng.integers(0, 16, size=(80, 32, 3))
    yield "residual_pq", codecs.encode_residual_pq(rcb, ridx, bits=5)
    yield "aap_in", codecs.encode_aap(rng.standard_normal((72, 8)), rng.standard_normal((256, 8)), "input")
    yield "aap_out", codecs.encode_aap(rng.standard_normal((8, 256)), rng.standard_normal((72, 8)), "output")
    w = rng.standard_normal((64, 256)).astype(np.float32)
    yield "binary", codecs.encode_hq30(w, "complete_binary", 64)
    yield "uq4", codecs.encode_hq30(w, "uniform_q4", 64)
    yield "residual", codecs.encode_hq30(w, "binary_residual", 128, keep=300)


@pytest.mark.parametrize("nb", [1, 3])
def test_codebook_gemvs_match_dense(nb):
    rng = np.random.default_rng(11 + nb)
    for name, p in _payloads(rng):
        W = torch.from_numpy(codecs.decode(p).reshape(-1, 256 if name not in ("pq", "residual_pq") else
                                                      codecs.header(p)["cols"])).to(DEV)
        N, K = W.shape
        x = Q8Act(nb, K, DEV)
        rmsnorm_q8(torch.randn(nb, K, device=DEV), None, 1e-5, x, norm=False)
        dev_w = gravity_weight(p, DEV)
        y = torch.zeros(nb, N, device=DEV)
        dev_w.gemv(x, y)
        ref = x.dequantize() @ W.t()
        torch.testing.assert_close(y, ref, rtol=2e-3, atol=2e-3 * float(ref.abs().max()), msg=name)
        y2 = y.clone()
        dev_w.gemv(x, y2, accumulate=True)  # residual epilogue adds
        torch.testing.assert_close(y2, 2 * y, rtol=1e-4, atol=1e-4 * float(ref.abs().max()), msg=name)
