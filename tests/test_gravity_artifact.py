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
