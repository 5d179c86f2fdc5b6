"""Tensor-core paged decode attention (attention_tc.cu) against a plain-PyTorch fp32 reference.

The kernel rounds the scaled query and the softmax weights to bf16 for the MMAs (K and V are bf16
already), so the tolerance is a few bf16 ulps of the output scale."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200 import ops  # noqa: E402

DEV = "cuda"


def _case(R, nh, nkv, hd, bs, ctxs, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    mb = max(-(-c // bs) for c in ctxs) + 1
    nblk = R * mb + 3
    kc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    perm = torch.randperm(nblk, device=DEV, generator=g).int()
    tables = perm[: R * mb].view(R, mb).contiguous()
    row_seq = torch.arange(R, dtype=torch.int32, device=DEV)
    row_ctx = torch.tensor(ctxs, dtype=torch.int32, device=DEV)
    q = torch.randn(R, nh, hd, device=DEV, generator=g)
    return q, kc, vc, tables, row_seq, row_ctx


def _reference(q, kc, vc, tables, row_ctx, scale):
    R, nh, hd = q.shape
    nkv, bs = kc.shape[1], kc.shape[2]
    G = nh // nkv
    out = torch.zeros(R, nh, hd, device=DEV)
    for r in range(R):
        c = int(row_ctx[r])
        blocks = tables[r, : -(-c // bs)].long()
        k = kc[blocks].permute(1, 0, 2, 3).reshape(nkv, -1, hd)[:, :c].float()
        v = vc[blocks].permute(1, 0, 2, 3).reshape(nkv, -1, hd)[:, :c].float()
        for h in range(nh):
            s = (q[r, h] @ k[h // G].T) * scale
            out[r, h] = torch.softmax(s, 0) @ v[h // G]
    return out.reshape(R, nh * hd)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("nh,nkv", [(32, 8), (8, 8), (16, 2), (32, 2)])
@pytest.mark.parametrize("bs,splits", [(64, 8), (16, 1), (32, 4), (64, 2)])
def test_attention_tc_matches_reference(hd, nh, nkv, bs, splits):
    ctxs = [1, 77, 2048][: 3]
    q, kc, vc, tables, row_seq, row_ctx = _case(3, nh, nkv, hd, bs, ctxs, hd + nh + bs + splits)
    scale = 1.0 / math.sqrt(hd)
    out = torch.full((3, nh * hd), float("nan"), device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.attention_decode(q, kc, vc, tables, row_seq, row_ctx, scale, splits, torch.zeros(1, device=DEV),
                         torch.zeros(1, device=DEV), out=out, cluster=True, tc=True, status=status)
    torch.cuda.synchronize()
    assert status.item() == 0
    ref = _reference(q, kc, vc, tables, row_ctx, scale)
    err = (out - ref).abs().max().item()
    assert err <= 2e-2 * ref.abs().max().item(), err


def test_attention_tc_bf16_and_q8_outputs_match_cuda_core_kernel():
    nh, nkv, hd, bs = 32, 8, 128, 64
    q, kc, vc, tables, row_seq, row_ctx = _case(2, nh, nkv, hd, bs, [300, 1500], 5)
    scale = 1.0 / math.sqrt(hd)
    outs = {}
    for tc in (True, False):
        ob = torch.zeros(2, nh * hd, dtype=torch.bfloat16, device=DEV)
        oq = ops.Q8Act(2, nh * hd, DEV)
        ops.attention_decode(q, kc, vc, tables, row_seq, row_ctx, scale, 8, torch.zeros(1, device=DEV),
                             torch.zeros(1, device=DEV), out_q8=oq, out_bf16=ob, cluster=True, tc=tc)
        outs[tc] = (ob.float(), oq.dequantize())
    torch.cuda.synchronize()
    for i in range(2):
        a, b = outs[True][i], outs[False][i]
        assert (a - b).abs().max().item() <= 3e-2 * b.abs().max().item()
