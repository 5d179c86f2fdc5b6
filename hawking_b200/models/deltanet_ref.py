"""Gated delta rule (the DeltaNet mixer of the Qwen3-Next-style hybrid): the token-serial recurrence
and its chunked matrix form, in plain PyTorch (fp32 or fp64, any device).

The recurrence, per value head, with state S [dk, dv], key k (already normalised), query q, value
v, gate beta in (0, 1) and decay alpha = exp(log_alpha) in (0, 1]:

    S <- alpha S ;  delta = beta (v - S^T k) ;  S <- S + k delta^T ;  o = S^T q

Chunked form over C consecutive tokens from a chunk-initial state S0 (A_t = prod_{s<=t} alpha_s
inside the chunk). Unrolling the recurrence gives, for the chunk's correction vectors Delta [C, dv]:

    (I + L) Delta = diag(beta) (V - diag(A) K S0),   L_ts = beta_t (A_t / A_s) k_t . k_s  (s < t)

so Delta = U - W S0 with T = (I + L)^-1 diag(beta), U = T V, W = T diag(A) K; then

    O   = diag(A) Q S0 + (M * (Q K^T)) Delta,         M_ts = A_t / A_s  (s <= t), 0 above
    S_C = A_C S0 + (diag(A_C / A) K)^T Delta

Everything but the unit-lower-triangular solve is a matrix product over the chunk (the tensor-core
shape of a chunked prefill); the ratios A_t / A_s (s <= t) are formed from cumulative log decays,
so they never overflow. This module is the numerical reference for such a prefill: the device
kernels walk the recurrence token by token today (deltanet.cu), and tests check the chunked form
against the recurrence here.

Parity: the reference's DeltaNet decode math, crates/hawking-core/shaders/qwen80_device_activations.metal:344-393
(gated delta update) and the token-serial oracle it is checked against.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


def gated_delta_recurrent(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                          log_alpha: torch.Tensor, state: Optional[torch.Tensor] = None
                          ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Token-serial gated delta rule for one head.

    q, k [T, dk]; v [T, dv]; beta, log_alpha [T]; state [dk, dv] (zeros if None).
    Returns (outputs [T, dv], final state [dk, dv])."""
    T, dk = k.shape
    dv = v.shape[1]
    S = torch.zeros(dk, dv, dtype=v.dtype, device=v.device) if state is None else state.clone()
    out = torch.empty(T, dv, dtype=v.dtype, device=v.device)
    for t in range(T):
        S = S * torch.exp(log_alpha[t])
        delta = beta[t] * (v[t] - S.t() @ k[t])
        S = S + torch.outer(k[t], delta)
        out[t] = S.t() @ q[t]
    return out, S


def gated_delta_chunk(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                      log_alpha: torch.Tensor, S0: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """One chunk of C tokens in the matrix form above. Returns (outputs [C, dv], state S_C)."""
    C = k.shape[0]
    g = torch.cumsum(log_alpha, 0)                      # log A_t
    diff = g[:, None] - g[None, :]                      # log (A_t / A_s)
    lower = torch.ones(C, C, dtype=torch.bool, device=k.device).tril()
    ratio = torch.where(lower, torch.exp(torch.where(lower, diff, torch.zeros_like(diff))),
                        torch.zeros_like(diff))         # A_t / A_s for s <= t, else 0
    kk = k @ k.t()
    L = (beta[:, None] * ratio * kk).tril(-1)
    eye = torch.eye(C, dtype=k.dtype, device=k.device)
    A = torch.exp(g)
    rhs = beta[:, None] * (v - A[:, None] * (k @ S0))
    delta = torch.linalg.solve_triangular(eye + L, rhs, upper=False, unitriangular=True)
    out = A[:, None] * (q @ S0) + (ratio * (q @ k.t())) @ delta
    tail = torch.exp(g[-1] - g)                         # A_C / A_s
    S = A[-1] * S0 + (tail[:, None] * k).t() @ delta
    return out, S


def gated_delta_chunked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, beta: torch.Tensor,
                        log_alpha: torch.Tensor, state: Optional[torch.Tensor] = None, chunk: int = 64
                        ) -> Tuple[torch.Tensor, torch.Tensor]:
    """The whole sequence in chunks of ``chunk`` tokens (the last may be shorter), the state carried
    from chunk to chunk. Same arguments and results as ``gated_delta_recurrent``."""
    T, dk = k.shape
    dv = v.shape[1]
    S = torch.zeros(dk, dv, dtype=v.dtype, device=v.device) if state is None else state.clone()
    outs = []
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        o, S = gated_delta_chunk(q[c0:c1], k[c0:c1], v[c0:c1], beta[c0:c1], log_alpha[c0:c1], S)
        outs.append(o)
    return torch.cat(outs) if outs else torch.empty(0, dv, dtype=v.dtype, device=v.device), S
