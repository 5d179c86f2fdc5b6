"""fp4 e2m1 weights with power-of-two block scales (the source layout of DeepSeek-V4-style expert
tensors: packed e2m1 pairs and e8m0 exponents per 32 columns) on the host: the code table, the
MX quantisation rule, and the lossless loader.

Parity: crates/hawking-core/shaders/dsv4f_activation_x_batch.metal:82 (e2m1 value of a nibble, the
high nibble for odd columns) and :181 (fp4 x e8m0 block GEMM)."""
import torch

from hawking_b200.ops.mixed import E2M1_MAGNITUDES, FP4, MixedWeight, _pack_lsb, e2m1_decode


def test_e2m1_code_table():
    codes = torch.arange(16)
    vals = e2m1_decode(codes)
    assert vals[:8].tolist() == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert vals[8:].tolist() == [-v for v in E2M1_MAGNITUDES]


def test_loader_keeps_codes_and_makes_exact_scales():
    g = torch.Generator().manual_seed(0)
    N, K = 6, 96
    codes = torch.randint(0, 16, (N, K), generator=g, dtype=torch.uint8)
    e = torch.randint(100, 140, (N, K // 32), generator=g, dtype=torch.uint8)
    packed = _pack_lsb(codes, 4)
    # the source layout: column c in byte c // 2, the high nibble for odd c
    assert int(packed[0, 0]) == int(codes[0, 0]) | (int(codes[0, 1]) << 4)
    w = MixedWeight.from_e2m1_e8m0(packed, e, N, K, "cpu")
    assert w.kind == FP4 and w.bits == 4 and w.group == 32 and torch.equal(w.codes, packed)
    ref = e2m1_decode(codes) * torch.exp2(e.float() - 127).repeat_interleave(32, 1)
    assert torch.equal(w.dequantize(), ref)


def test_mx_quantisation_rule():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(8, 256, generator=g) * 0.05
    m = MixedWeight.quantize_fp4(w)
    d = m.dequantize()
    s = m.scales.repeat_interleave(32, 1)
    # power-of-two scales, 2^(floor(log2 amax) - 2)
    amax = w.view(8, 8, 32).abs().amax(-1)
    assert torch.equal(m.scales, torch.exp2(torch.floor(torch.log2(amax)) - 2))
    # every value is an e2m1 value times its block scale; below 6 scale units an element is within
    # half a grid gap (at most one unit, the 4 -> 6 gap), above it saturates at 6 (amax / scale < 8)
    q = d / s
    assert bool(torch.isin(q.abs(), torch.tensor(E2M1_MAGNITUDES)).all())
    inside = w.abs() <= 6 * s
    assert ((d - w).abs()[inside] <= s[inside] + 1e-7).all()
    assert ((d - w).abs() < 2 * s).all()
    # inputs already on the grid come back exactly
    assert torch.equal(MixedWeight.quantize_fp4(d).dequantize(), d)


def test_halfway_values_take_the_even_code():
    # amax 4 -> scale 2^(2 - 2) = 1; each value sits halfway between two e2m1 neighbours
    vals = [0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 4.0]
    w = torch.tensor(vals + [0.0] * 24).view(1, 32)
    m = MixedWeight.quantize_fp4(w)
    assert m.scales.tolist() == [[1.0]]
    got = m.dequantize()[0, :8].tolist()
    assert got == [0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 4.0]
    neg = MixedWeight.quantize_fp4(-w).dequantize()[0, :8].tolist()
    assert neg == [-0.0 if x == 0 else -x for x in got]
