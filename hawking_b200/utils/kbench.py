"""Kernel micro-benchmarks on one GPU: the decode-batch hot kernels at Llama-3-8B shapes, timed
with CUDA events over several weight / cache copies whose total exceeds the 126 MB L2 (each
launch reads from HBM, as in a real step).

    python -m hawking_b200.utils.kbench gemm --rows 64 [--shape gate_up] [--iters 40]
    python -m hawking_b200.utils.kbench attn --rows 64 [--splits 1,2] [--ctx 2048]

``gemm``: the tcgen05 Q4_K GEMM (``ops.tc_gemm``, split-K as the model picks it) per projection;
prints microseconds, weight bytes per second, TFLOP/s and the error against an fp32 product.
``attn``: the tensor-core paged decode attention (``ops.attention_decode``); prints microseconds
and KV bytes per second. One JSON line each.

Parity: the reference times single kernels with example harnesses of its own (e.g.
crates/hawking-core/examples/ascension_qwen38_matmul_k_amortization.rs, the packed matvec receipts in
its README); this module plays that part here.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

LLAMA8B = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336)}


def _time(fn, iters: int, warmup: int = 6) -> float:
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(iters):
        fn(i)
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1000.0


def bench_gemm(rows: int, shapes, iters: int, copies: int = 4) -> dict:
    from hawking_b200 import ops
    from hawking_b200.formats.ggml import GgmlType
    from hawking_b200.ops import QWeight
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(0)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    out = {}
    for name in shapes:
        N, K = LLAMA8B[name]
        ws = [QWeight.quantize(torch.randn(N, K, device=dev, generator=g) * 0.02, GgmlType.Q4_K)
              for _ in range(copies)]
        x = torch.randn(rows, K, device=dev, generator=g).bfloat16()
        y = torch.zeros(rows, N, device=dev)
        us = _time(lambda i: ops.tc_gemm(ws[i % copies], x, y, st, atomic=True), iters)
        y.zero_()
        ops.tc_gemm(ws[0], x, y, st, atomic=True)
        ref = x.float() @ ws[0].dequantize().T
        torch.cuda.synchronize()
        wbytes = N * K * 144 / 256
        out[name] = {"us": round(us, 1), "weight_TBps": round(wbytes / us / 1e6, 3),
                     "tflops": round(2 * rows * N * K / us / 1e6, 1),
                     "rel_err": round(((y - ref).abs().max() / ref.abs().max()).item(), 5)}
        del ws
    return {"kernel": "tc_gemm_q4k", "rows": rows, "results": out, "status": int(st.item())}


def bench_attn(rows: int, splits, ctx: int, iters: int, copies: int = 4) -> dict:
    from hawking_b200 import ops
    dev = "cuda"
    nh, nkv, hd, bs = 32, 8, 128, 64
    g = torch.Generator(device=dev).manual_seed(0)
    mb = -(-ctx // bs) + 1
    nblk = rows * mb + 3
    caches = [(torch.randn(nblk, nkv, bs, hd, device=dev, generator=g).bfloat16(),
               torch.randn(nblk, nkv, bs, hd, device=dev, generator=g).bfloat16()) for _ in range(copies)]
    tables = torch.randperm(nblk, device=dev, generator=g).int()[: rows * mb].view(rows, mb).contiguous()
    row_seq = torch.arange(rows, dtype=torch.int32, device=dev)
    row_ctx = torch.full((rows,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(rows, nh, hd, device=dev, generator=g)
    ob = torch.zeros(rows, nh * hd, dtype=torch.bfloat16, device=dev)
    z = torch.zeros(1, device=dev)
    out = {}
    kv_bytes = rows * nkv * ctx * hd * 2 * 2
    for s in splits:
        def run(i, s=s):
            kc, vc = caches[i % copies]
            ops.attention_decode(q, kc, vc, tables, row_seq, row_ctx, 1 / math.sqrt(hd), s, z, z, out_bf16=ob,
                                 cluster=True, tc=True)
        us = _time(run, iters)
        out[str(s)] = {"us": round(us, 1), "kv_TBps": round(kv_bytes / us / 1e6, 3)}
    return {"kernel": "attn_decode_tc", "rows": rows, "ctx": ctx, "results": out}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("kernel", choices=["gemm", "attn"])
    ap.add_argument("--rows", type=int, default=64)
    ap.add_argument("--shape", default="qkv,o,gate_up,down", help="gemm: projections (comma list)")
    ap.add_argument("--splits", default="1,2", help="attn: KV splits (comma list)")
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=40)
    a = ap.parse_args(argv)
    if a.kernel == "gemm":
        r = bench_gemm(a.rows, a.shape.split(","), a.iters)
    else:
        r = bench_attn(a.rows, [int(s) for s in a.splits.split(",")], a.ctx, a.iters)
    print(json.dumps(r))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
