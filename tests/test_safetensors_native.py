"""safetensors container and the native block-scaled pairs of DeepSeek-V4-style checkpoints on the
host: the container round trip, the pairing rules (fp4 I8 + E8M0 per 32 columns, fp8 E4M3 + E8M0
per 128 x 128 block) with their refusals, and the values the loaded mixed weights decode to."""
import numpy as np
import pytest
import torch

from hawking_b200.formats.safetensors import (SafeTensors, SafetensorsError, load_native_pair,
                                              native_scale_pairs, write_safetensors)
from hawking_b200.ops.mixed import FP4, FP8, _pack_lsb, e2m1_decode


def _fp4(N, K, g):
    codes = torch.randint(0, 16, (N, K), generator=g, dtype=torch.uint8)
    e = torch.randint(110, 135, (N, K // 32), generator=g, dtype=torch.uint8)
    return codes, e


def _file(tmp_path, tensors, name="m.safetensors"):
    return SafeTensors(write_safetensors(str(tmp_path / name), tensors, {"format": "pt"}))


def test_container_round_trip(tmp_path):
    a = np.arange(12, dtype=np.float32).reshape(3, 4)
    st = _file(tmp_path, {"a": ("F32", (3, 4), a.tobytes()), "b": ("U8", (5,), bytes(range(5)))})
    assert st.names() == ["a", "b"] and st.metadata == {"format": "pt"}
    assert np.array_equal(st.raw("a").view(np.float32).reshape(3, 4), a)
    assert bytes(st.raw("b")) == bytes(range(5))


def test_native_pairs_load_to_their_values(tmp_path):
    g = torch.Generator().manual_seed(0)
    codes, e4 = _fp4(64, 256, g)
    w8 = (torch.randn(256, 384, generator=g) * 3).to(torch.float8_e4m3fn)
    e8 = torch.randint(115, 130, (2, 3), generator=g, dtype=torch.uint8)
    st = _file(tmp_path, {
        "layers.0.ffn.experts.0.w1.weight": ("I8", (64, 128), _pack_lsb(codes, 4).numpy().tobytes()),
        "layers.0.ffn.experts.0.w1.scale": ("F8_E8M0", (64, 8), e4.numpy().tobytes()),
        "layers.0.attn.wq.weight": ("F8_E4M3", (256, 384), w8.view(torch.uint8).numpy().tobytes()),
        "layers.0.attn.wq.scale": ("F8_E8M0", (2, 3), e8.numpy().tobytes()),
        "layers.0.attn_norm.weight": ("F32", (4,), np.ones(4, np.float32).tobytes()),
    })
    pairs = native_scale_pairs(st)
    assert set(pairs) == {"layers.0.ffn.experts.0.w1.weight", "layers.0.attn.wq.weight"}
    p4 = pairs["layers.0.ffn.experts.0.w1.weight"]
    assert (p4.logical_k, p4.scale_cols) == (256, 8)
    m4 = load_native_pair(st, p4, "cpu")
    assert m4.kind == FP4 and (m4.N, m4.K) == (64, 256)
    ref4 = e2m1_decode(codes) * torch.exp2(e4.float() - 127).repeat_interleave(32, 1)
    assert torch.equal(m4.dequantize(), ref4)
    m8 = load_native_pair(st, pairs["layers.0.attn.wq.weight"], "cpu")
    assert m8.kind == FP8 and (m8.N, m8.K) == (256, 384)
    blk = torch.exp2(e8.float() - 127).repeat_interleave(128, 0).repeat_interleave(128, 1)
    assert torch.equal(m8.dequantize(), w8.float() * blk)


@pytest.mark.parametrize("case", ["missing_scale", "bad_shape", "orphan_scale", "name", "fp8_dims", "rank"])
def test_native_pair_refusals(tmp_path, case):
    w = ("I8", (4, 16), bytes(64))
    s = ("F8_E8M0", (4, 1), bytes([127] * 4))
    t = {"x.weight": w, "x.scale": s}
    if case == "missing_scale":
        del t["x.scale"]
    elif case == "bad_shape":
        t["x.scale"] = ("F8_E8M0", (4, 2), bytes([127] * 8))
    elif case == "orphan_scale":
        t["y.scale"] = ("F8_E8M0", (1, 1), bytes([127]))
    elif case == "name":
        t = {"x.w": w, "x.scale": s}
    elif case == "fp8_dims":
        t = {"x.weight": ("F8_E4M3", (100, 128), bytes(100 * 128)), "x.scale": ("F8_E8M0", (1, 1), bytes([127]))}
    elif case == "rank":
        t["x.scale"] = ("F8_E8M0", (4,), bytes([127] * 4))
    with pytest.raises(SafetensorsError):
        native_scale_pairs(_file(tmp_path, t))


def test_corrupt_offsets_are_refused(tmp_path):
    import json
    import struct
    p = tmp_path / "bad.safetensors"
    hdr = json.dumps({"a": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}).encode()
    p.write_bytes(struct.pack("<Q", len(hdr)) + hdr + bytes(16))
    with pytest.raises(SafetensorsError):
        SafeTensors(str(p))


def test_act_quant_scale_rule_and_values():
    from hawking_b200.formats.safetensors import act_quant_e8m0
    x = torch.zeros(3, 256)
    x[0, 0] = 448.0           # scaled 1.0: a power of two, e = 0
    x[0, 128] = 449.0         # just above: e = 1
    x[1, 5] = -3.0            # 3 / 448 -> 2^-7 (0.0078125 >= 0.0066964)
    x[1, 130] = 1e-6          # below the floor: 1e-4 / 448 -> 2^-22
    x[2] = torch.linspace(-10, 10, 256)
    q, e = act_quant_e8m0(x)
    assert e.tolist()[0] == [127, 128] and e.tolist()[1] == [120, 105]
    s = torch.exp2(e.float() - 127).repeat_interleave(128, 1)
    back = q.view(torch.float8_e4m3fn).float() * s
    assert back[0, 0].item() == 448.0 and back[1, 5].item() == -3.0
    # e4m3 keeps 3 mantissa bits: every value within half a step of its input
    rel = ((back - x).abs() / x.abs().clamp_min(1e-30))[x.abs() > 1e-3]
    assert (rel <= 2 ** -4 + 1e-7).all()


def test_fp8_block_matvec_matches_dense_product():
    from hawking_b200.formats.safetensors import act_quant_e8m0, fp8_block_matvec
    g = torch.Generator().manual_seed(3)
    w = (torch.randn(256, 384, generator=g) * 2).to(torch.float8_e4m3fn)
    we = torch.randint(120, 130, (2, 3), generator=g, dtype=torch.uint8)
    x = torch.randn(384, generator=g)
    aq, ae = act_quant_e8m0(x)
    y = fp8_block_matvec(w.view(torch.uint8), we, aq, ae)
    wd = w.float() * torch.exp2(we.float() - 127).repeat_interleave(128, 0).repeat_interleave(128, 1)
    ad = aq.view(torch.float8_e4m3fn).float() * torch.exp2(ae.float() - 127).repeat_interleave(128)
    assert torch.allclose(y.double(), wd.double() @ ad.double(), rtol=1e-5, atol=1e-5)


def test_deepseek_v3_weight_scale_inv_pairs(tmp_path):
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(200, 256, generator=g) * 4).to(torch.float8_e4m3fn)   # 200 rows: a partial row block
    inv = torch.rand(2, 2, generator=g) * 0.01 + 1e-3
    st = _file(tmp_path, {
        "model.layers.0.mlp.down_proj.weight": ("F8_E4M3", (200, 256), w.view(torch.uint8).numpy().tobytes()),
        "model.layers.0.mlp.down_proj.weight_scale_inv": ("F32", (2, 2), inv.numpy().tobytes())})
    pairs = native_scale_pairs(st)
    p = pairs["model.layers.0.mlp.down_proj.weight"]
    assert p.kind == "native.fp8_e4m3fn_f32" and (p.scale_rows, p.scale_cols) == (2, 2)
    m = load_native_pair(st, p, "cpu")
    assert m.kind == FP8 and (m.N, m.K) == (200, 256) and m.scales.shape == (200, 2)
    blk = inv.repeat_interleave(128, 0)[:200].repeat_interleave(128, 1)
    assert torch.equal(m.dequantize(), w.float() * blk)
    bad = _file(tmp_path, {"a.weight": ("F8_E4M3", (200, 256), bytes(200 * 256)),
                           "a.weight_scale_inv": ("F32", (1, 2), bytes(8))}, name="bad.safetensors")
    with pytest.raises(SafetensorsError):
        native_scale_pairs(bad)
