"""deepseek2 GGUF loading on the host: config keys, the GGUF -> table-weight mappings (bit-exact
for Q4_K / Q8_0 / Q4_0), the rope-row permutation and the YaRN frequencies."""
import math
import os

import numpy as np
import pytest
import torch

from hawking_b200.formats.ggml import GgmlType
from hawking_b200.formats.gguf import GgufBuilder, GgufModel
from hawking_b200.formats.synth import write_deepseek2_gguf
from hawking_b200.models.config import preset
from hawking_b200.models.deepseek_gguf import (deepseek_config_from_gguf, kva_row_order, q_row_order,
                                               yarn_attention_scale, yarn_freq_factors)
from hawking_b200.models.torch_ref import config_from_gguf
from hawking_b200.ops.mixed import Q4K, UNIFORM, MixedWeight


def small_cfg(**kw):
    base = dict(vocab=1024, hidden=512, layers=3, n_heads=4, n_kv_heads=4, ffn=512, n_experts=8, top_k=2,
                expert_ffn=256, shared_ffn=256, n_groups=4, topk_groups=2, first_dense_layers=1, q_lora_rank=256,
                max_ctx=512, weight_type="Q4_K")
    base.update(kw)
    return preset("deepseek-v3").with_(**base)


def test_config_from_gguf(tmp_path):
    cfg = small_cfg()
    p = write_deepseek2_gguf(str(tmp_path / "ds.gguf"), cfg, yarn=4.0)
    c = config_from_gguf(GgufModel(p))
    for f in ("hidden", "layers", "n_heads", "n_experts", "top_k", "expert_ffn", "shared_ffn", "n_groups",
              "topk_groups", "first_dense_layers", "q_lora_rank", "kv_lora_rank", "qk_nope_dim", "qk_rope_dim",
              "v_head_dim", "router", "norm_topk", "vocab", "ffn"):
        assert getattr(c, f) == getattr(cfg, f), f
    assert c.routed_scale == pytest.approx(cfg.routed_scale)
    assert c.rope_yarn_factor == 4.0 and c.rope_yarn_orig_ctx == 128
    assert c.rope_yarn_log_mul == pytest.approx(0.1)


def test_config_v2_lite_style(tmp_path):
    cfg = small_cfg(q_lora_rank=0, router="softmax", n_groups=1, topk_groups=1, norm_topk=False, routed_scale=1.0,
                    n_shared_experts=2, shared_ffn=512)
    p = write_deepseek2_gguf(str(tmp_path / "ds.gguf"), cfg)
    c = deepseek_config_from_gguf(GgufModel(p))
    assert c.q_lora_rank == 0 and c.router == "softmax" and not c.norm_topk
    assert c.n_shared_experts == 2 and c.shared_ffn == 512 and c.rope_yarn_factor == 0.0


def test_not_deepseek(tmp_path):
    b = GgufBuilder("llama")
    b.add("token_embd.weight", np.zeros((32, 32), np.float32))
    p = b.write(str(tmp_path / "l.gguf"))
    with pytest.raises(ValueError):
        deepseek_config_from_gguf(GgufModel(p))


@pytest.mark.parametrize("fmt,exact", [(GgmlType.Q4_K, True), (GgmlType.Q8_0, True), (GgmlType.Q4_0, True),
                                       (GgmlType.Q6_K, False), (GgmlType.F16, False)])
def test_mixed_from_gguf_tensor(tmp_path, fmt, exact):
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((48, 512)) * 0.05).astype(np.float32)
    b = GgufBuilder("llama")
    b.add("w", a, fmt)
    m = GgufModel(b.write(str(tmp_path / "w.gguf")))
    ref = torch.from_numpy(m.dequantize("w").reshape(48, 512))
    w = MixedWeight.from_gguf(torch.from_numpy(np.ascontiguousarray(m.raw("w"))), fmt, 48, 512, "cpu")
    got = w.dequantize()
    if exact:
        assert torch.equal(got, ref)
        assert w.kind == (Q4K if fmt == GgmlType.Q4_K else UNIFORM)
    else:
        step = ref.view(48, 16, 32).abs().amax(-1, keepdim=True) / 127
        assert ((got - ref).view(48, 16, 32).abs() <= step * 0.5 + 1e-6).all()
    rows = w.rows(8, 16).dequantize()
    assert torch.equal(rows, got[8:24])


def test_mixed_q4k_cols_slice(tmp_path):
    rng = np.random.default_rng(4)
    a = (rng.standard_normal((16, 1024)) * 0.05).astype(np.float32)
    b = GgufBuilder("llama")
    b.add("w", a, GgmlType.Q4_K)
    m = GgufModel(b.write(str(tmp_path / "w.gguf")))
    w = MixedWeight.from_gguf(torch.from_numpy(np.ascontiguousarray(m.raw("w"))), GgmlType.Q4_K, 16, 1024, "cpu")
    full = w.dequantize()
    assert torch.equal(w.cols(256, 768).dequantize(), full[:, 256:768])
    with pytest.raises(ValueError):
        w.cols(128, 512)


def _rope_adjacent(x, ang):
    a, b = x[0::2], x[1::2]
    out = torch.empty_like(x)
    out[0::2] = a * torch.cos(ang) - b * torch.sin(ang)
    out[1::2] = b * torch.cos(ang) + a * torch.sin(ang)
    return out


def _rope_halves(x, ang):
    h = x.shape[0] // 2
    a, b = x[:h], x[h:]
    return torch.cat([a * torch.cos(ang) - b * torch.sin(ang), b * torch.cos(ang) + a * torch.sin(ang)])


def test_rope_row_permutation_preserves_scores():
    torch.manual_seed(0)
    nh, nope, rd = 3, 8, 64
    Wq = torch.randn(nh * (nope + rd), 16, dtype=torch.float64)
    Wk = torch.randn(512 + rd, 16, dtype=torch.float64)
    x, y = torch.randn(16, dtype=torch.float64), torch.randn(16, dtype=torch.float64)
    ang_q = torch.arange(rd // 2, dtype=torch.float64) * 0.37
    ang_k = torch.arange(rd // 2, dtype=torch.float64) * 0.11
    q, k = (Wq @ x).view(nh, nope + rd), Wk @ y
    qp, kp = (Wq[q_row_order(nh, nope, rd)] @ x).view(nh, nope + rd), Wk[kva_row_order(rd)] @ y
    assert torch.equal(qp[:, :nope], q[:, :nope]) and torch.equal(kp[:512], k[:512])
    for h in range(nh):
        s_file = _rope_adjacent(q[h, nope:], ang_q) @ _rope_adjacent(k[512:], ang_k)
        s_dev = _rope_halves(qp[h, nope:], ang_q) @ _rope_halves(kp[512:], ang_k)
        assert s_dev.item() == pytest.approx(s_file.item(), rel=1e-12, abs=1e-12)


def test_yarn_frequencies_and_scale():
    cfg = small_cfg(rope_yarn_factor=40.0, rope_yarn_orig_ctx=4096, rope_yarn_log_mul=0.1, rope_theta=10000.0)
    ff = yarn_freq_factors(cfg)
    assert ff.shape == (32,)
    assert ff[0].item() == pytest.approx(1.0)       # highest frequency: extrapolated (kept)
    assert ff[-1].item() == pytest.approx(40.0)     # lowest frequency: interpolated by the factor
    assert (ff[1:] >= ff[:-1] - 1e-12).all()
    ms = 1 + 0.1 * math.log(40.0)
    assert yarn_attention_scale(cfg) == pytest.approx(ms * ms / math.sqrt(192))
    assert yarn_freq_factors(small_cfg()) is None
    assert yarn_attention_scale(small_cfg()) == pytest.approx(1 / math.sqrt(192))


def test_synthetic_file_names(tmp_path):
    cfg = small_cfg(q_lora_rank=0)
    m = GgufModel(write_deepseek2_gguf(str(tmp_path / "ds.gguf"), cfg))
    assert m.has("blk.0.attn_q.weight") and not m.has("blk.0.attn_q_a.weight")
    assert m.tensors["blk.1.ffn_down_exps.weight"].type == GgmlType.Q6_K
    assert m.tensors["blk.1.ffn_gate_exps.weight"].shape == (8, 256, 512)
    assert m.has("blk.1.exp_probs_b.bias") and not m.has("blk.0.exp_probs_b.bias")
    assert os.path.getsize(m.path) > 0
