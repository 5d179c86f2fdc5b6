"""The fused decode routing kernel (router GEMV + top-k + sort by expert + active list in one
launch) against the separate router / top-k / align kernels: same experts, weights, order."""
import pytest
import torch

from hawking_b200 import ops
from hawking_b200._ext import kernels
from hawking_b200.ops import Q8Act

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("E,k,scoring,groups,tg,shared,T", [(256, 8, 1, 8, 4, True, 1), (256, 8, 1, 8, 4, True, 5),
                                                            (512, 10, 0, 1, 1, False, 3), (64, 2, 0, 1, 1, False, 8)])
def test_fused_route_matches_separate(E, k, scoring, groups, tg, shared, T):
    g = torch.Generator(device=DEV).manual_seed(E + k + T)
    H = 2048
    router = torch.randn(E, H, device=DEV, generator=g) * 0.02
    bias = torch.randn(E, device=DEV, generator=g) * 0.01 if scoring == 1 else None
    x = Q8Act(T, H, DEV)
    ops.rmsnorm_q8(torch.randn(T, H, device=DEV, generator=g), None, 1e-6, x)
    # separate kernels
    logits = torch.zeros(T, E, device=DEV)
    ids = torch.zeros(T, k, dtype=torch.int32, device=DEV)
    w = torch.zeros(T, k, device=DEV)
    ops.router_logits(router, x, logits)
    ops.moe_topk(logits, bias, k, scoring, groups, tg, True, 2.5, ids, w)
    counts = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    offsets = torch.zeros_like(counts)
    srt = torch.zeros(T * k + T, dtype=torch.int32, device=DEV)
    gx = Q8Act(T * k + T, H, DEV)
    ops.moe_align(ids, E, x, counts, offsets, srt, gx, shared=shared)
    active = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    n_active = torch.zeros(1, dtype=torch.int32, device=DEV)
    kernels().moe_active(counts, active, n_active, False)
    # fused
    logits2 = torch.zeros_like(logits)
    ids2, w2 = torch.zeros_like(ids), torch.zeros_like(w)
    counts2, offsets2, srt2 = torch.zeros_like(counts), torch.zeros_like(offsets), torch.zeros_like(srt)
    active2, n_active2 = torch.zeros_like(active), torch.zeros_like(n_active)
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):  # the arrival counter resets itself
        ops.moe_route(router, x, k, scoring, bias, groups, tg, True, 2.5, logits2, ids2, w2, counts2, offsets2, srt2,
                      active2, n_active2, shared, counter)
        torch.cuda.synchronize()
        assert int(counter.item()) == 0
        torch.testing.assert_close(logits2, logits, rtol=1e-5, atol=1e-6)
        assert torch.equal(ids2, ids)
        torch.testing.assert_close(w2, w)
        n = E + (1 if shared else 0)
        assert torch.equal(counts2[:n], counts[:n]) and torch.equal(offsets2[:n], offsets[:n])
        P = T * k + (T if shared else 0)
        assert torch.equal(srt2[:P], srt[:P])
        assert int(n_active2.item()) == int(n_active.item())
        na = int(n_active.item())
        assert sorted(active2[:na].tolist()) == sorted(active[:na].tolist())


def _route_oracle(logits, bias, k, scoring, groups, tg, renorm, scale):
    """Plain PyTorch routing (fp64): scores (softmax, or sigmoid with the learned bias added for
    selection only), group-limited selection (keep the `tg` groups with the largest sum of their
    two best selection scores), top-k with the lowest index winning ties, optional renormalise,
    routed scale. Returns ids [T, k] and weights [T, k] (DeepSeek-V3 noaux_tc / Mixtral top-k)."""
    lg = logits.double()
    T, E = lg.shape
    score = torch.softmax(lg, -1) if scoring == 0 else torch.sigmoid(lg)
    sel = score + (bias.double() if (scoring == 1 and bias is not None) else 0.0)
    if groups > 1:
        gs = sel.view(T, groups, E // groups).topk(2, dim=-1).values.sum(-1)
        keep = torch.zeros(T, groups, dtype=torch.bool, device=lg.device)
        for t in range(T):  # lowest group index wins a tie, as the kernel's strict comparison
            order = sorted(range(groups), key=lambda gi: (-gs[t, gi].item(), gi))[:tg]
            keep[t, order] = True
        sel = sel.masked_fill(~keep.repeat_interleave(E // groups, dim=1), float("-inf"))
    ids = torch.zeros(T, k, dtype=torch.long, device=lg.device)
    for t in range(T):
        order = sorted(range(E), key=lambda e: (-sel[t, e].item(), e))[:k]
        ids[t] = torch.tensor(order, device=lg.device)
    w = score.gather(1, ids)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return ids, w * scale


@pytest.mark.parametrize("E,k,scoring,groups,tg,T", [(256, 8, 1, 8, 4, 3), (512, 10, 0, 1, 1, 2), (64, 2, 0, 1, 1, 4)])
def test_fused_route_matches_torch_oracle(E, k, scoring, groups, tg, T):
    """Logits against a torch matmul of the dequantised activations; experts and weights against
    the plain PyTorch top-k oracle (wherever the k-th and (k+1)-th selection scores are not tied
    within the logits' rounding)."""
    g = torch.Generator(device=DEV).manual_seed(3 * E + k + T)
    H = 2048
    router = torch.randn(E, H, device=DEV, generator=g) * 0.02
    bias = torch.randn(E, device=DEV, generator=g) * 0.01 if scoring == 1 else None
    x = Q8Act(T, H, DEV)
    ops.rmsnorm_q8(torch.randn(T, H, device=DEV, generator=g), None, 1e-6, x)
    logits = torch.zeros(T, E, device=DEV)
    ids = torch.zeros(T, k, dtype=torch.int32, device=DEV)
    w = torch.zeros(T, k, device=DEV)
    counts = torch.zeros(E + 1, dtype=torch.int32, device=DEV)
    offsets, srt = torch.zeros_like(counts), torch.zeros(T * k + T, dtype=torch.int32, device=DEV)
    active, n_active = torch.zeros_like(counts), torch.zeros(1, dtype=torch.int32, device=DEV)
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.moe_route(router, x, k, scoring, bias, groups, tg, True, 2.5, logits, ids, w, counts, offsets, srt, active,
                  n_active, False, counter)
    torch.cuda.synchronize()
    xd = (x.q.view(T, H // 32, 32).float() * x.d.view(T, H // 32, 1)).view(T, H)
    ref_logits = xd.double() @ router.double().T
    torch.testing.assert_close(logits.double(), ref_logits, rtol=1e-4, atol=1e-5)
    rid, rw = _route_oracle(logits, bias, k, scoring, groups, tg, True, 2.5)
    assert torch.equal(ids.long(), rid)
    torch.testing.assert_close(w.double(), rw, rtol=1e-4, atol=1e-6)
