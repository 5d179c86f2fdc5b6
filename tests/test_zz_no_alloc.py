"""The allocation-free attention entry point, called through its exported C symbol.

Some callers of this library cannot allocate device memory (an engine embedded in a host whose
allocator owns the GPU's memory, or a decode loop where cudaMalloc's possible device
synchronisation is not allowed). ``hk_attention_decode_noalloc`` serves them: same split-KV paged
decode attention as ``attention_decode``, scratch in fixed device arrays inside the library. This
test calls it through ctypes (no Python binding involved) twice in a row and compares each result
with the regular entry point, then checks that an oversized request is refused.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _lib():
    import hawking_b200._kernels as k  # loads libtorch first; the symbol lives in this library
    lib = ctypes.CDLL(k.__file__)
    f = lib.hk_attention_decode_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    err = lib.hk_attention_decode_noalloc_error
    err.restype = ctypes.c_char_p
    return f, err


def _inputs(nh=32, nkv=8, hd=128, bs=16, nblk=40, R=3):
    g = torch.Generator(device=DEV).manual_seed(11)
    kc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    vc = torch.randn(nblk, nkv, bs, hd, device=DEV, generator=g).bfloat16()
    perm = torch.randperm(nblk, device=DEV, generator=g).int()
    tables = torch.stack([perm[:20], perm[20:]]).contiguous()
    row_seq = torch.tensor([0, 1, 0], dtype=torch.int32, device=DEV)[:R]
    row_ctx = torch.tensor([5, 100, 319], dtype=torch.int32, device=DEV)[:R]
    q = torch.randn(R, nh, hd, device=DEV, generator=g)
    return q, kc, vc, tables, row_seq, row_ctx


def _call(f, q, kc, vc, tables, row_seq, row_ctx, splits, out):
    R, nh, hd = q.shape
    stream = torch.cuda.current_stream().cuda_stream
    return f(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), tables.data_ptr(), tables.shape[1], row_seq.data_ptr(),
             row_ctx.data_ptr(), 1.0 / math.sqrt(hd), R, nh, kc.shape[1], hd, kc.shape[2], splits, out.data_ptr(),
             stream)


def test_noalloc_matches_regular_entry_point_twice():
    from hawking_b200 import ops
    f, err = _lib()
    q, kc, vc, tables, row_seq, row_ctx = _inputs()
    R, nh, hd = q.shape
    splits = 7
    ref = torch.zeros(R, nh * hd, device=DEV)
    ops.attention_decode(q, kc, vc, tables, row_seq, row_ctx, 1.0 / math.sqrt(hd), splits,
                         torch.zeros(R * nh * splits * hd, device=DEV), torch.zeros(R * nh * splits, device=DEV),
                         out=ref, counters=torch.zeros(R * kc.shape[1], dtype=torch.int32, device=DEV))
    for _ in range(2):
        out = torch.full((R, nh * hd), float("nan"), device=DEV)
        rc = _call(f, q, kc, vc, tables, row_seq, row_ctx, splits, out)
        torch.cuda.synchronize()
        assert rc == 0, err().decode()
        torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_oversized_requests():
    f, err = _lib()
    q, kc, vc, tables, row_seq, row_ctx = _inputs(hd=256)
    out = torch.zeros(q.shape[0], q.shape[1] * q.shape[2], device=DEV)
    rc = _call(f, q, kc, vc, tables, row_seq, row_ctx, 64, out)  # 3 * 32 * 64 * 256 floats > 1 Mi
    assert rc == 2
    assert b"fixed scratch" in err()
