"""GGML block formats: C++ oracle vs an independent torch restatement, round-trip error bounds."""
import numpy as np
import pytest
import torch

from hawking_b200.formats import quant_torch
from hawking_b200.formats.ggml import LAYOUTS, GgmlType

QUANT_TYPES = [GgmlType.Q4_0, GgmlType.Q4_1, GgmlType.Q5_0, GgmlType.Q5_1, GgmlType.Q8_0,
               GgmlType.Q4_K, GgmlType.Q5_K, GgmlType.Q6_K, GgmlType.F16, GgmlType.BF16]
# Worst-case relative (to row max-abs) round-trip error per format.
TOL = {GgmlType.Q4_0: 0.10, GgmlType.Q4_1: 0.08, GgmlType.Q5_0: 0.05, GgmlType.Q5_1: 0.04,
       GgmlType.Q8_0: 0.01, GgmlType.Q4_K: 0.12, GgmlType.Q5_K: 0.06, GgmlType.Q6_K: 0.03,
       GgmlType.F16: 1e-3, GgmlType.BF16: 8e-3}


@pytest.mark.parametrize("t", QUANT_TYPES)
def test_round_trip(native, t):
    rng = np.random.default_rng(int(t))
    x = rng.standard_normal((8, 512)).astype(np.float32)
    q = native.quantize_rows(t, x)
    assert q.shape == (8, 512 // LAYOUTS[t].block_elems * LAYOUTS[t].block_bytes)
    y = native.dequantize_rows(t, q, 8, 512)
    err = np.abs(y - x).max(axis=1) / np.abs(x).max(axis=1)
    assert err.max() < TOL[t], (LAYOUTS[t].name, err.max())


@pytest.mark.parametrize("t", [t for t in QUANT_TYPES if t in quant_torch.SUPPORTED])
def test_cpp_matches_torch_restatement(native, t):
    rng = np.random.default_rng(100 + int(t))
    x = (rng.standard_normal((4, 1024)) * 0.05).astype(np.float32)
    q = native.quantize_rows(t, x)
    a = native.dequantize_rows(t, q, 4, 1024)
    b = quant_torch.dequantize(torch.from_numpy(q.copy()), t, (4, 1024)).numpy()
    np.testing.assert_array_equal(a, b)


@pytest.mark.parametrize("t", [GgmlType.Q2_K, GgmlType.Q3_K])
def test_lower_k_quants_decode_random_bytes(native, t):
    # Readers for Q2_K/Q3_K: decode random blocks, check finiteness and torch-free invariants.
    lay = LAYOUTS[t]
    rng = np.random.default_rng(7)
    raw = rng.integers(0, 256, size=(4 * lay.block_bytes,), dtype=np.uint8)
    d_off = {GgmlType.Q2_K: 80, GgmlType.Q3_K: 108}[t]
    for i in range(4):  # sane fp16 super-scales
        raw[i * lay.block_bytes + d_off: i * lay.block_bytes + d_off + 2] = np.frombuffer(
            np.float16(0.01).tobytes(), np.uint8)
        if t == GgmlType.Q2_K:
            raw[i * lay.block_bytes + 82: i * lay.block_bytes + 84] = np.frombuffer(np.float16(0.02).tobytes(), np.uint8)
    y = native.dequantize(t, raw, 4 * 256)
    assert np.isfinite(y).all()
    assert y.shape == (1024,)


def test_q3_k_known_pattern(native):
    # All-zero qs with every hmask bit set decodes to 0; with hmask clear to -4 * d * (scale-32).
    lay = LAYOUTS[GgmlType.Q3_K]
    blk = np.zeros(lay.block_bytes, np.uint8)
    blk[108:110] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    # scales: all six-bit scales = 33 -> (33-32)=1; low nibble 1 everywhere, high bits 2 (=32)
    blk[96:104] = 0x11
    blk[104:108] = 0xAA
    y = native.dequantize(GgmlType.Q3_K, blk, 256)
    np.testing.assert_allclose(y, -4.0)
    blk[0:32] = 0xFF
    y = native.dequantize(GgmlType.Q3_K, blk, 256)
    np.testing.assert_allclose(y, 0.0)


def test_q8_0_zeros(native):
    x = np.zeros((1, 64), np.float32)
    q = native.quantize_rows(GgmlType.Q8_0, x)
    np.testing.assert_array_equal(native.dequantize_rows(GgmlType.Q8_0, q, 1, 64), x)


def test_fp16_conversions(native):
    for v in [0.0, 1.0, -2.5, 65504.0, 6.1e-5, 5.96e-8, 1e-9, 3.14159]:
        h = native.f32_to_fp16(v)
        assert h == int(np.float16(v).view(np.uint16)), v
        assert native.fp16_to_f32(h) == float(np.float16(v))
