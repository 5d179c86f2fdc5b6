"""Chunked matrix form of the gated delta rule against the token-serial recurrence (fp64 on the
CPU): outputs and carried state agree for several chunk sizes, a partial last chunk, a nonzero
initial state and strong decays."""
import pytest
import torch

from hawking_b200.models.deltanet_ref import gated_delta_chunk, gated_delta_chunked, gated_delta_recurrent


def _inputs(T, dk, dv, seed, strong_decay=False):
    g = torch.Generator().manual_seed(seed)
    f = lambda *s: torch.randn(*s, generator=g, dtype=torch.float64)  # noqa: E731
    k = torch.nn.functional.normalize(f(T, dk), dim=-1)   # the mixer normalises q and k
    q = torch.nn.functional.normalize(f(T, dk), dim=-1) * dk ** -0.5
    v = f(T, dv)
    beta = torch.sigmoid(f(T))
    log_alpha = -torch.rand(T, generator=g, dtype=torch.float64) * (6.0 if strong_decay else 0.5)
    S0 = f(dk, dv) * 0.3
    return q, k, v, beta, log_alpha, S0


@pytest.mark.parametrize("T,chunk", [(1, 64), (63, 64), (64, 64), (150, 64), (150, 16), (37, 8)])
@pytest.mark.parametrize("strong_decay", [False, True])
def test_chunked_matches_recurrence(T, chunk, strong_decay):
    q, k, v, beta, la, S0 = _inputs(T, 32, 24, T + chunk, strong_decay)
    o_ref, S_ref = gated_delta_recurrent(q, k, v, beta, la, S0)
    o, S = gated_delta_chunked(q, k, v, beta, la, S0, chunk=chunk)
    assert torch.allclose(o, o_ref, rtol=1e-9, atol=1e-10)
    assert torch.allclose(S, S_ref, rtol=1e-9, atol=1e-10)


def test_single_chunk_from_zero_state_and_split_point_invariance():
    q, k, v, beta, la, _ = _inputs(40, 16, 16, 5)
    Z = torch.zeros(16, 16, dtype=torch.float64)
    o1, S1 = gated_delta_chunk(q, k, v, beta, la, Z)
    # the same tokens split at any point give the same outputs and state
    oa, Sa = gated_delta_chunk(q[:13], k[:13], v[:13], beta[:13], la[:13], Z)
    ob, Sb = gated_delta_chunk(q[13:], k[13:], v[13:], beta[13:], la[13:], Sa)
    assert torch.allclose(torch.cat([oa, ob]), o1, rtol=1e-10, atol=1e-12)
    assert torch.allclose(Sb, S1, rtol=1e-10, atol=1e-12)
