"""The allocation-free attention entry point, called through its exported C symbol.

Some callers of this library cannot allocate device memory (an engine embedded in a host whose
allocator owns the GPU's memory, or a decode loop where cudaMalloc's possible device
synchronisation is not allowed). ``hk_attention_decode_noalloc`` serves them: the same split-KV
paged decode attention as ``attention_decode``, with its scratch in fixed device arrays inside the
library. These tests call it through ctypes (no Python binding involved), with the argument types
read from its C header, twice in a row and with differently sized calls back to back, compare each
result with the regular entry point, and check the refusals (oversized, small blocks, misaligned).
"""
import ctypes
import math
import os
import re

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "hawking_b200", "csrc", "kernels",
                      "noalloc.h")
_CTYPES = {"const float*": ctypes.c_void_p, "const void*": ctypes.c_void_p, "const int*": ctypes.c_void_p,
           "float*": ctypes.c_void_p, "void*": ctypes.c_void_p, "int": ctypes.c_int, "float": ctypes.c_float}


def _header_argtypes():
    """ctypes argument types of hk_attention_decode_noalloc, parsed from its declaration in noalloc.h."""
    src = open(HEADER).read()
    m = re.search(r"int\s+hk_attention_decode_noalloc\s*\(([^)]*)\)\s*;", src)
    assert m, "declaration not found in noalloc.h"
    types = []
    for p in m.group(1).split(","):
        p = " ".join(p.split())
        t = re.sub(r"\s*\w+$", "", p).replace(" *", "*")
        assert t in _CTYPES, f"unmapped C type {t!r}"
        types.append(_CTYPES[t])
    return types


def _lib():
    import hawking_b200._kernels as k  # loads libtorch first; the symbol lives in this library
    lib = ctypes.CDLL(k.__file__)
    f = lib.hk_attention_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = _header_argtypes()
    assert len(f.argtypes) == 16
    err = lib.hk_attention_decode_noalloc_error
    err.restype = ctypes.c_char_p
    return f, err


def _inputs(nh=32, nkv=8, hd=128, bs=16, nblk=40, R=3, seed=11):
    g = torch.Generator(device=DEV).manual_seed(seed)
    kc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    perm = torch.randperm(nblk, device=DEV, generator=g).int()
    half = nblk // 2
    tables = torch.stack([perm[:half], perm[half:2 * half]]).contiguous()
    cap = half * bs
    row_seq = torch.tensor([0, 1, 0, 1], dtype=torch.int32, device=DEV)[:R]
    row_ctx = torch.tensor([5, min(100, cap), cap - 1, cap], dtype=torch.int32, device=DEV)[:R]
    q = torch.randn(R, nh, hd, device=DEV, generator=g)
    return q, kc, vc, tables, row_seq, row_ctx


def _call(f, q, kc, vc, tables, row_seq, row_ctx, splits, out, stream=None):
    R, nh, hd = q.shape
    if stream is None:
        stream = torch.cuda.current_stream().cuda_stream
    return f(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), tables.shape[1], row_seq.data_ptr(),
             row_ctx.data_ptr(), 1.0 / math.sqrt(hd), R, nh, kc.shape[1], hd, kc.shape[2], splits, out.data_ptr(),
             stream)


def _reference(q, kc, vc, tables, row_seq, row_ctx, splits):
    from hawking_b200 import ops
    R, nh, hd = q.shape
    ref = torch.zeros(R, nh * hd, device=DEV)
    ops.attention_decode(q, kc, vc, tables, row_seq, row_ctx, 1.0 / math.sqrt(hd), splits,
                         torch.zeros(R * nh * splits * hd, device=DEV), torch.zeros(R * nh * splits, device=DEV),
                         out=ref, counters=torch.zeros(R * kc.shape[1], dtype=torch.int32, device=DEV),
                         cluster=False)
    return ref


def test_noalloc_matches_regular_entry_point_twice():
    f, err = _lib()
    q, kc, vc, tables, row_seq, row_ctx = _inputs()
    splits = 7
    ref = _reference(q, kc, vc, tables, row_seq, row_ctx, splits)
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        rc = _call(f, q, kc, vc, tables, row_seq, row_ctx, splits, out)
        torch.cuda.synchronize()
        assert rc == 0, err().decode()
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("hd,splits", [(64, 1), (64, 64), (128, 1), (128, 64), (256, 1), (256, 7), (256, 32)])
def test_noalloc_head_dims_and_splits(hd, splits):
    f, err = _lib()
    q, kc, vc, tables, row_seq, row_ctx = _inputs(hd=hd, seed=hd + splits)
    ref = _reference(q, kc, vc, tables, row_seq, row_ctx, splits)
    out = torch.full_like(ref, float("nan"))
    rc = _call(f, q, kc, vc, tables, row_seq, row_ctx, splits, out)
    torch.cuda.synchronize()
    assert rc == 0, err().decode()
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)


def test_noalloc_back_to_back_different_shapes():
    """A smaller call right after a larger one: the counters the first call used are cleared for
    the second, and the second's result does not depend on what the first left in the scratch."""
    f, err = _lib()
    big = _inputs(nh=32, nkv=8, hd=128, R=4, seed=1)
    small = _inputs(nh=8, nkv=2, hd=64, bs=32, R=2, seed=2)
    ref_big = _reference(*big, 16)
    ref_small = _reference(*small, 5)
    out_big = torch.full_like(ref_big, float("nan"))
    out_small = torch.full_like(ref_small, float("nan"))
    assert _call(f, *big, 16, out_big) == 0, err().decode()
    assert _call(f, *small, 5, out_small) == 0, err().decode()
    torch.cuda.synchronize()
    torch.testing.assert_close(out_big, ref_big, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(out_small, ref_small, rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_oversized_requests():
    f, err = _lib()
    q, kc, vc, tables, row_seq, row_ctx = _inputs(hd=256)
    out = torch.zeros(q.shape[0], q.shape[1] * q.shape[2], device=DEV)
    rc = _call(f, q, kc, vc, tables, row_seq, row_ctx, 64, out)  # 3 * 32 * 64 * 256 floats > 1 Mi
    assert rc == 2
    assert b"fixed scratch" in err()


def test_noalloc_rejects_small_blocks_and_misalignment():
    f, err = _lib()
    q, kc, vc, tables, row_seq, row_ctx = _inputs(bs=4, nblk=80)
    out = torch.zeros(q.shape[0], q.shape[1] * q.shape[2], device=DEV)
    assert _call(f, q, kc, vc, tables, row_seq, row_ctx, 4, out) == 1
    assert b"block_size" in err()
    q, kc, vc, tables, row_seq, row_ctx = _inputs()
    flat = torch.zeros(kc.numel() + 8, dtype=torch.bfloat16, device=DEV)
    kc_off = flat[1:1 + kc.numel()].view(kc.shape)  # 2-byte aligned
    kc_off.copy_(kc)
    assert _call(f, q, kc_off, vc, tables, row_seq, row_ctx, 4, out) == 1
    assert b"aligned" in err()
    torch.cuda.synchronize()
