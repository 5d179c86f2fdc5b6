"""`.gravity` shards, directories, mixed codecs and the HQ80M15 catalog (CPU)."""
import json
import os

import numpy as np
import pytest

from hawking_b200.formats import mixed
from hawking_b200.formats.gravity import GravityModel, is_gravity, write_index, write_shard


def _payload(n, seed):
    return np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)


def test_shard_round_trip_and_verify(tmp_path, native):
    a, b = _payload(100, 1), _payload(37, 2)
    p = tmp_path / "model-00001.gravity"
    hdr = write_shard(str(p), [{"name": "w.a", "codec": "native.f32", "shape": [25], "data": a},
                               {"name": "w.b", "codec": "ggml.q8_0", "shape": [37], "data": b, "elements": 0}],
                      meta={"model": {"name": "t"}, "architecture": {"name": "llama"}})
    assert hdr["schema"] == "hawking.gravity.shard_header.v1"
    raw = p.read_bytes()
    assert raw[:8] == b"GRAVITY\0" and int.from_bytes(raw[8:12], "little") == 1
    hl = int.from_bytes(raw[12:20], "little")
    text = raw[20:20 + hl].decode()
    assert text == native.canonical_json(json.loads(text))  # canonical: sorted keys, compact
    assert is_gravity(str(p))
    m = GravityModel(str(p), verify_on_open=True)
    np.testing.assert_array_equal(m.raw("w.a"), a)
    np.testing.assert_array_equal(m.raw("w.b"), b)
    rep = m.verify()[p.name]
    assert rep["ok"] and rep["tensor_count"] == 2
    assert m.tensors["w.a"].offset == 0 and m.tensors["w.b"].offset == 100


def test_corruption_detected(tmp_path):
    p = tmp_path / "m.gravity"
    write_shard(str(p), [{"name": "x", "codec": "native.f16", "shape": [8], "data": _payload(16, 3)}])
    data = bytearray(p.read_bytes())
    data[-1] ^= 0xFF
    p.write_bytes(bytes(data))
    m = GravityModel(str(p))
    rep = m.verify()["m.gravity"]
    assert not rep["ok"] and rep["bad_tensors"] == ["x"] and not rep["body_sha256_ok"]
    with pytest.raises(RuntimeError, match="sha256"):
        GravityModel(str(p), verify_on_open=True)


def test_bad_magic_and_truncation(tmp_path):
    p = tmp_path / "bad.gravity"
    p.write_bytes(b"NOTGRAV!" + b"\0" * 20)
    with pytest.raises(RuntimeError, match="magic"):
        GravityModel(str(p))
    write_shard(str(p), [{"name": "x", "codec": "native.f32", "shape": [4], "data": _payload(16, 4)}])
    p.write_bytes(p.read_bytes()[:-8])
    with pytest.raises(RuntimeError):
        GravityModel(str(p))


def test_directory_index(tmp_path):
    d = tmp_path / "art"
    d.mkdir()
    write_shard(str(d / "model-00001.gravity"), [{"name": "a", "codec": "native.f32", "shape": [2], "data": _payload(8, 5)}])
    write_shard(str(d / "model-00002.gravity"), [{"name": "b", "codec": "native.f32", "shape": [2], "data": _payload(8, 6)}])
    write_index(str(d), {"a": "model-00001.gravity", "b": "model-00002.gravity"}, {"name": "llama"},
                {"a": "native.f32", "b": "native.f32"})
    m = GravityModel(str(d))
    assert set(m.tensors) == {"a", "b"} and m.architecture == "llama"
    (d / "model-00002.gravity").write_bytes((d / "model-00002.gravity").read_bytes()[:-1] + b"\0")
    with pytest.raises(RuntimeError, match="shard"):
        GravityModel(str(d))


def test_ggml_codec_dequant(tmp_path, native):
    x = np.random.default_rng(0).standard_normal((4, 256)).astype(np.float32)
    q = native.quantize_rows(12, x)
    p = tmp_path / "q.gravity"
    write_shard(str(p), [{"name": "w", "codec": "ggml.q4_k", "shape": [4, 256], "data": q}])
    m = GravityModel(str(p))
    np.testing.assert_array_equal(m.dequantize("w"), native.dequantize_rows(12, q, 4, 256))


@pytest.mark.parametrize("bits", [2, 3, 4, 8])
def test_uniform_codec(bits):
    w = np.random.default_rng(bits).standard_normal((8, 128)).astype(np.float32)
    p = mixed.encode_uniform(w, bits, 64)
    magic, hdr, _, _ = mixed.header(p)
    assert magic == b"HGRAVU01" and hdr["bits"] == bits and hdr["group_size"] == 64
    d = mixed.decode(p)
    bound = (1 << (bits - 1)) - 1
    g = w.reshape(-1, 64)
    step = np.abs(g).max(1, keepdims=True) / bound
    assert (np.abs(d.reshape(-1, 64) - g) <= 0.5 * step + 1e-3 * step + np.abs(g) * 2e-3).all()


def test_binary_codec_reconstruction():
    w = np.random.default_rng(1).standard_normal((4, 128)).astype(np.float32)
    p = mixed.encode_binary(w, 64)
    d = mixed.decode(p)
    g = w.reshape(-1, 64)
    scale = np.abs(g).mean(1, keepdims=True)
    np.testing.assert_allclose(np.abs(d.reshape(-1, 64)), np.broadcast_to(scale, g.shape), rtol=1e-3)
    assert (np.sign(d) == np.where(w >= 0, 1, -1)).all()
    big = np.random.default_rng(9).standard_normal((512, 2048)).astype(np.float32)
    assert mixed.payload_bits(mixed.encode_binary(big, 64), big.size) < 1.26  # 1 sign + 16/64 scale bits


def test_rice_residual_codec(native):
    w = np.random.default_rng(2).standard_normal((16, 256)).astype(np.float32)
    p = mixed.encode_binary_residual(w, 128, 0.02, 5)
    idx = native.rice_indices(p)
    assert len(idx) == int(np.ceil(w.size * 0.02)) and idx == sorted(idx)
    base = mixed.decode(mixed.encode_binary(w, 128))
    d = mixed.decode(p)
    changed = np.flatnonzero(np.abs(d - base).reshape(-1) > 0)
    assert set(changed.tolist()) == set(idx)
    # residual selection is the global top-|w - binary(w)|
    r = np.abs(w - base).reshape(-1)
    assert r[idx].min() >= np.sort(r)[-len(idx)] - 1e-6


def test_low_rank_codec():
    rng = np.random.default_rng(3)
    L, R = rng.standard_normal((32, 8)).astype(np.float32), rng.standard_normal((8, 64)).astype(np.float32)
    p = mixed.encode_low_rank(L, R, bits=3, group=64)
    magic, hdr, _, _ = mixed.header(p)
    assert magic == b"HGRAVS01" and hdr["representation"] == "activation_weighted_svd_low_rank_q"
    d = mixed.decode(p)
    assert d.shape == (32, 64)
    Lq = mixed.decode(mixed.encode_uniform(L, 3, 64))
    Rq = mixed.decode(mixed.encode_uniform(R, 3, 64))
    np.testing.assert_allclose(d, Lq @ Rq, rtol=1e-5, atol=1e-5)  # y = L @ (R @ x) semantics


def test_catalog_round_trip(tmp_path, native):
    c = native.Catalog()
    s = native.CatalogSegment()
    s.id, s.name, s.bytes, s.sha256 = 0, "L00.hq80seg", 123, "ab" * 32
    t = native.CatalogTensor()
    t.name, t.codec, t.organ, t.ndim, t.dims = "blk.0.ffn_gate_exps.0", 0, 0, 2, [512, 2048]
    t.elements, t.segment, t.offset, t.nbytes, t.sha256, t.codec_bpw = 512 * 2048, 0, 0, 123, "cd" * 32, 1.25
    c.segments = [s]
    c.tensors = [t]
    p = str(tmp_path / "catalog.hq80m15")
    native.write_catalog(p, c)
    raw = open(p, "rb").read()
    assert raw[:8] == b"HQ80M15\0"
    r = native.read_catalog(p)
    assert r.tensors[0].name == t.name and r.tensors[0].dims == [512, 2048, 0, 0]
    assert r.segments[0].sha256 == "ab" * 32 and abs(r.tensors[0].codec_bpw - 1.25) < 1e-6
