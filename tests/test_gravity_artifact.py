"""Lossless `.gravity` envelopes for device-quantised mixed weights (HGRAVB01 / HGRAVU01 wrapped
around existing planes, no re-quantisation): the payload maps back onto the same planes and the
C++ decoder reconstructs the same values; a Qwen3-Next-shaped artifact round-trips on the CPU."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from hawking_b200._ext import native  # noqa: E402
from hawking_b200.ops.mixed import BINARY, UNIFORM, MixedWeight  # noqa: E402


@pytest.mark.parametrize("kind,bits", [(BINARY, 1), (UNIFORM, 2), (UNIFORM, 4), (UNIFORM, 8)])
def test_wrap_round_trip(kind, bits):
    g = torch.Generator().manual_seed(kind * 10 + bits)
    w = torch.randn(48, 256, generator=g) * 0.05
    mw = MixedWeight.quantize(w, kind, bits, 64)
    scales = mw.scales.contiguous().view(torch.uint8).numpy().reshape(-1)
    codes = mw.codes.contiguous().numpy().reshape(-1)
    if kind == BINARY:
        payload = native().wrap_hgravb01(48, 256, 64, scales, codes)
    else:
        payload = native().wrap_hgravu01(48, 256, 64, bits, scales, codes)
    back = MixedWeight.from_payload(payload, "cpu")
    assert (back.kind, back.bits, back.group, back.N, back.K) == (mw.kind, mw.bits, mw.group, mw.N, mw.K)
    assert torch.equal(back.codes, mw.codes) and torch.equal(back.scales, mw.scales)
    dense = native().mixed_decode(np.ascontiguousarray(payload))
    assert np.array_equal(dense, mw.dequantize().numpy())


def test_wrap_rejects_wrong_plane_sizes():
    with pytest.raises(Exception):
        native().wrap_hgravu01(4, 64, 64, 4, np.zeros(8, np.uint8), np.zeros(3, np.uint8))


def test_r02_s01_device_planes_match_cpu_decode():
    """The planes the device GEMVs use (binary base + CSR outliers; the two low-rank factors)
    reconstruct the C++ decode of the payload."""
    from hawking_b200.formats import mixed as mx
    from hawking_b200.ops.mixed import LowRankWeight, RiceResidualWeight
    rng = np.random.default_rng(1)
    w = (rng.standard_normal((96, 512)) * 0.05).astype(np.float32)
    w[rng.random((96, 512)) < 0.01] *= 12
    p = mx.encode_binary_residual(w, group=128, ratio=0.02, rice_k=5)
    rw = RiceResidualWeight.from_payload(p, "cpu")
    assert rw.cols.numel() > 0 and int(rw.row_ptr[-1]) == rw.cols.numel()
    assert np.array_equal(rw.dequantize().numpy(), mx.decode(p))
    L = (rng.standard_normal((128, 64)) * 0.1).astype(np.float32)
    R = (rng.standard_normal((64, 512)) * 0.1).astype(np.float32)
    p = mx.encode_low_rank(L, R, bits=4, group=64)
    lw = LowRankWeight.from_payload(p, "cpu")
    assert np.allclose(lw.dequantize().numpy(), mx.decode(p), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("size", [0, 1, 55, 56, 63, 64, 65, 127, 128, 1000, 4113, 1 << 20])
def test_sha256_paths_agree(size):
    """The SHA-extension compression path, the portable one and hashlib give the same digest."""
    import hashlib
    a = np.random.default_rng(size).integers(0, 256, size=size, dtype=np.uint8)
    want = hashlib.sha256(a.tobytes()).hexdigest()
    assert native().sha256_hex(a) == want
    assert native().sha256_hex_portable(a) == want
