"""Fixed-header codecs (GLM52CPK, LLM52RPK, GLM52AAP, HQ30G1B1 / HQ30UQ4 / HQ30GR2) and the
`.hawking` sidecar: C++ parsers/decoders against an independent NumPy restatement, round trips,
and rejection of malformed payloads (reference: crates/hawking-core/src/artifact_pq.rs tests,
artifact_aap.rs, qwen_complete_binary/mod.rs, sidecar.rs tier-map tests)."""
import numpy as np
import pytest

from hawking_b200.formats import codecs, sidecar


def test_msb_bit_packing_matches_numpy():
    rng = np.random.default_rng(0)
    for bits in (1, 3, 7, 8, 11, 16):
        v = rng.integers(0, 1 << bits, size=257, dtype=np.uint64).astype(np.uint32)
        cb = rng.standard_normal((1, 1 << bits if bits <= 8 else 256, 2)).astype(np.float16)
        idx = (v % cb.shape[1]).reshape(257, 1, 1)
        payload = codecs.encode_pq(cb, idx, bits)
        hdr, (c, i) = codecs.payload_sections(payload)
        assert (i.reshape(-1).astype(np.uint32) == idx.reshape(-1)).all()
        stream = payload[64 + cb.size * 2:]
        assert (codecs.unpack_msb_np(stream, idx.size, bits) == idx.reshape(-1)).all()


def test_pq_decode_and_matvec():
    rng = np.random.default_rng(1)
    s, card, sub, rows, nchunk = 4, 16, 2, 12, 6
    cb = rng.standard_normal((s, card, sub)).astype(np.float16)
    idx = rng.integers(0, card, size=(rows, nchunk, s))
    payload = codecs.encode_pq(cb, idx, bits=4, seed=7)
    h = codecs.header(payload)
    assert (h["d"], h["s"], h["sub"], h["rows"], h["cols"], h["nchunk"], h["seed"]) == (8, 4, 2, rows, 48, 6, 7)
    w = codecs.decode(payload)
    ref = codecs.pq_decode_np(cb.astype(np.float32), idx)
    np.testing.assert_array_equal(w, ref)
    x = rng.standard_normal(48).astype(np.float32)
    np.testing.assert_allclose(codecs.matvec_f64(payload, x), ref.astype(np.float64) @ x, rtol=1e-12, atol=1e-9)


def test_residual_pq_decode():
    rng = np.random.default_rng(2)
    stages, card, d, rows, nchunk = 3, 8, 4, 5, 7
    cb = rng.standard_normal((stages, card, d)).astype(np.float16)
    idx = rng.integers(0, card, size=(rows, nchunk, stages))
    payload = codecs.encode_residual_pq(cb, idx, bits=3)
    w = codecs.decode(payload)
    np.testing.assert_allclose(w, codecs.rpq_decode_np(cb.astype(np.float32), idx), rtol=1e-6, atol=1e-6)
    x = rng.standard_normal(nchunk * d).astype(np.float32)
    np.testing.assert_allclose(codecs.matvec_f64(payload, x), w.astype(np.float64) @ x, rtol=1e-5, atol=1e-5)


def test_pq_rejects_malformed():
    rng = np.random.default_rng(3)
    cb = rng.standard_normal((2, 4, 2)).astype(np.float16)
    idx = rng.integers(0, 4, size=(3, 2, 2))
    p = codecs.encode_pq(cb, idx, bits=2)
    bad = p.copy()
    bad[8 + 27] = 3  # codebook count != S
    with pytest.raises(RuntimeError):
        codecs.header(bad)
    with pytest.raises(RuntimeError):
        codecs.decode(p[:-1])  # truncated indices
    bad = p.copy()
    bad[8 + 26] = 1  # rotated: parsed but not decodable
    codecs.header(bad)
    with pytest.raises(RuntimeError):
        codecs.decode(bad)
    r = codecs.encode_residual_pq(cb, idx, bits=2)
    bad = r.copy()
    bad[8 + 26] = 1
    with pytest.raises(RuntimeError):
        codecs.header(bad)


@pytest.mark.parametrize("side", ["input", "output"])
def test_activation_aware(side):
    rng = np.random.default_rng(4)
    rows, cols, rank = 9, 14, 3
    if side == "input":
        coeff, basis = rng.standard_normal((rows, rank)), rng.standard_normal((cols, rank))
        ref = coeff.astype(np.float16).astype(np.float32) @ basis.astype(np.float16).astype(np.float32).T
    else:
        coeff, basis = rng.standard_normal((rank, cols)), rng.standard_normal((rows, rank))
        ref = basis.astype(np.float16).astype(np.float32) @ coeff.astype(np.float16).astype(np.float32)
    p = codecs.encode_aap(coeff, basis, side=side, basis_layer=5)
    h = codecs.header(p)
    assert (h["rows"], h["cols"], h["rank"], h["side"], h["basis_layer"]) == (rows, cols, rank, side, 5)
    np.testing.assert_allclose(codecs.decode(p), ref, rtol=1e-5, atol=1e-5)
    x = rng.standard_normal(cols).astype(np.float32)
    np.testing.assert_allclose(codecs.matvec_f64(p, x), ref.astype(np.float64) @ x, rtol=1e-5, atol=1e-5)
    with pytest.raises(RuntimeError):
        codecs.decode(np.concatenate([p, np.zeros(2, np.uint8)]))  # size must match exactly


def test_hq30_family():
    rng = np.random.default_rng(5)
    w = rng.standard_normal((6, 256)).astype(np.float32)
    b = codecs.encode_hq30(w, "complete_binary", 128)
    h = codecs.header(b)
    assert h["shape"] == [6, 256] and h["groups"] == 12
    dec = codecs.decode(b)
    g = w.reshape(-1, 128)
    ref = (np.where(g >= 0, 1.0, -1.0) * np.abs(g).mean(1, keepdims=True).astype(np.float16).astype(np.float32))
    np.testing.assert_allclose(dec.reshape(-1, 128), ref, rtol=1e-6, atol=1e-7)
    q = codecs.encode_hq30(w, "uniform_q4", 64)
    dq = codecs.decode(q)
    assert np.abs(dq - w).max() <= np.abs(w).max() / 7 * 0.51 + 1e-6
    r = codecs.encode_hq30(w, "binary_residual", 128, keep=40)
    hr = codecs.header(r)
    assert len(hr["indices"]) == 40 and hr["indices"] == sorted(hr["indices"])
    dr = codecs.decode(r)
    assert np.abs(dr - w).mean() < np.abs(dec - w).mean()
    bad = b.copy()
    bad[18] = 1  # reserved field
    with pytest.raises(RuntimeError):
        codecs.header(bad)


def test_sidecar_round_trip_and_compat(tmp_path):
    rng = np.random.default_rng(6)
    raw = rng.integers(0, 256, size=144 * 3, dtype=np.uint8)
    raw[0:2] = np.frombuffer(np.float16(0.5).tobytes(), np.uint8)
    raw[2:4] = np.frombuffer(np.float16(0.25).tobytes(), np.uint8)
    t = sidecar.predecode_q4k(raw)
    assert t.shape == (48,)
    sc = raw[4:16]
    s0, m0 = sc[0] & 63, sc[4] & 63
    s7, m7 = (sc[11] & 0xF) | ((sc[3] >> 6) << 4), (sc[11] >> 4) | ((sc[7] >> 6) << 4)
    assert t[0] == 0.5 * s0 and t[1] == 0.25 * m0 and t[14] == 0.5 * s7 and t[15] == 0.25 * m7
    p = str(tmp_path / "m.hawking")
    hdr = sidecar.make_header("abc", profile="race", tier_map=[{"tensor": "blk.0.ffn_down.weight", "dtype": "q8_0"}])
    sidecar.write(p, hdr, [(4096, t), (99, t[:16])])
    h2, entries = sidecar.read(p)
    assert list(h2) == ["version", "source_gguf_hash", "tokenizer_hash", "shader_hash", "bake_profile", "contents",
                        "quality", "bake_device", "bake_time_secs", "tier_map"]
    assert h2["contents"]["mixed_quant_tier_map"] and entries[0][0] == 4096
    np.testing.assert_array_equal(entries[0][1], t)
    assert sidecar.compatibility(h2, "abc") == "compatible"
    assert sidecar.compatibility(h2, "abd") == "gguf_hash_mismatch"
    assert sidecar.compatibility(h2, "abc", "shader") == "shader_hash_mismatch"
    assert sidecar.compatibility(dict(h2, version=2), "abc") == "version_too_new"
    with pytest.raises(ValueError):
        sidecar.validate_tier_map([{"tensor": "a", "dtype": "q8_0"}, {"tensor": "a", "dtype": "q4_K"}])
    with pytest.raises(ValueError):
        sidecar.validate_tier_map([{"tensor": "a", "dtype": "f16"}])


def test_sidecar_bake_from_gguf(tmp_path):
    from hawking_b200.formats.ggml import GgmlType
    from hawking_b200.formats.gguf import GgufBuilder, GgufModel
    rng = np.random.default_rng(7)
    path = str(tmp_path / "t.gguf")
    GgufBuilder("llama").add("w", rng.standard_normal((4, 256)).astype(np.float32), GgmlType.Q4_K).write(path)
    out = sidecar.bake(path)
    assert out.endswith("t.hawking")
    tables = sidecar.load_predecoded(path)
    m = GgufModel(path)
    t = m.tensors["w"]
    np.testing.assert_array_equal(tables[t.offset], sidecar.predecode_q4k(m.raw("w")))
