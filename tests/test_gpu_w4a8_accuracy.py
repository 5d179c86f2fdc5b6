"""What the opt-in W4A8 decode path (int8 activation blocks) costs in accuracy, on Llama-3-8B-shaped
layers: teacher-forced logits of single-token decode forwards against a plain fp32 PyTorch forward
of the same dequantised weights (no activation rounding, fp32 K/V), next to the default W4A16 path."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

from hawking_b200.engine.engine import Engine  # noqa: E402
from hawking_b200.formats.synth import random_prompt  # noqa: E402
from hawking_b200.models.config import preset  # noqa: E402
from hawking_b200.models.llama import random_llama_weights  # noqa: E402
from hawking_b200.models.torch_ref import rmsnorm_ref, rope_ref  # noqa: E402

DEV = "cuda"


def _fp32_forward(cfg, w, tokens):
    """Causal fp32 forward of the whole sequence; logits [len(tokens), vocab]."""
    H, hd, nh, nkv = cfg.hidden, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads
    n = len(tokens)
    ids = torch.tensor(tokens, device=DEV)
    x = w.embed.dequantize()[ids].float()
    pos = torch.arange(n, device=DEV)
    mask = torch.full((n, n), float("-inf"), device=DEV).triu(1)
    for lw in w.layers:
        qkv = rmsnorm_ref(x, lw.attn_norm, cfg.eps) @ lw.wqkv[0].dequantize().float().T
        q = qkv[:, : nh * hd].view(n, nh, hd)
        k = qkv[:, nh * hd: (nh + nkv) * hd].view(n, nkv, hd)
        v = qkv[:, (nh + nkv) * hd:].view(n, nkv, hd)
        q = rope_ref(q, pos, cfg.rope_theta, cfg.rope_dim, cfg.rope_style)
        k = rope_ref(k, pos, cfg.rope_theta, cfg.rope_dim, cfg.rope_style)
        G = nh // nkv
        k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(hd) + mask
        att = torch.einsum("hqk,khd->qhd", torch.softmax(s, -1), v).reshape(n, nh * hd)
        x = x + att @ lw.wo.dequantize().float().T
        h = rmsnorm_ref(x, lw.ffn_norm, cfg.eps)
        gu = h @ lw.w_gu.dequantize().float().T
        F = gu.shape[1] // 2
        x = x + (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ lw.w_down.dequantize().float().T
    return rmsnorm_ref(x, w.out_norm, cfg.eps) @ w.lm_head.dequantize().float().T


def _decode_logits(model, tokens, seq_id):
    kv = model.kv
    assert kv.bm.reserve(seq_id, len(tokens))
    kv.sync_tables([seq_id])
    r = kv.row(seq_id)
    out = []
    for i, t in enumerate(tokens):
        model.inp.upload([t], [i], [0], [r], [i + 1])
        model.forward(1, "none", n_logits=0)
        out.append(model.logits[0].clone())
    torch.cuda.synchronize()
    kv.drop(seq_id)
    return torch.stack(out)


def test_w4a8_logit_error_is_bounded_on_8b_shaped_layers():
    cfg = preset("llama3-8b").with_(layers=2, max_ctx=256)
    w = random_llama_weights(cfg, DEV, seed=21, std=0.02)
    prompt = random_prompt(48, cfg.vocab, seed=22)
    with torch.no_grad():
        ref = _fp32_forward(cfg, w, prompt)
    eng = Engine.build(cfg, w, device=DEV, max_batch=2, max_ctx=256, block_size=64, max_rows=8, num_blocks=16)
    m = eng.model
    got = {}
    for mode in ("w4a16", "w4a8"):
        m.small_batch = mode
        got[mode] = _decode_logits(m, prompt, seq_id=3 if mode == "w4a16" else 4)
    m.small_batch = "w4a16"
    scale = ref.abs().max().item()
    err = {k: (v - ref).abs().max().item() / scale for k, v in got.items()}
    top2 = ref.topk(2, dim=1).values
    margin = (top2[:, 0] - top2[:, 1]) / scale
    agree = {}
    for k, v in got.items():
        decided = margin > 2 * err[k]
        agree[k] = ((v.argmax(1) == ref.argmax(1))[decided].float().mean().item(), int(decided.sum()))
    print({"max_rel_logit_err": err, "top1_agreement_where_decided": agree})
    # Measured on B200: w4a16 7.8e-3 (bf16 K/V and the bf16 query / softmax weights of the
    # attention dominate), w4a8 2.9e-2. The default path tracks the fp32 forward at least twice as
    # closely as the int8-activation path, whose cost stays bounded relative to the logit scale
    # with top-1 intact wherever the reference is not a near tie.
    assert 2 * err["w4a16"] < err["w4a8"], err
    assert err["w4a16"] < 1.5e-2, err
    assert err["w4a8"] < 6e-2, err
    for k, (a, nd) in agree.items():
        assert nd >= 4 and a == 1.0, (k, a, nd)
