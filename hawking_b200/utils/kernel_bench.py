"""Per-kernel microbenchmark for the decode hot ops (Llama-3-8B shapes, Q4_K weights).

Each case is replayed inside one CUDA graph (``--iters`` launches back to back, as in a decode
step) and timed with CUDA events on the capturing stream after warm-up; achieved bandwidth is the
case's algorithmic bytes divided by the per-launch time. Every weight case cycles through enough
copies of its matrices (> 256 MB in total) that no launch finds its weights in the 126 MB L2, as in
a real decode step where 32 layers of weights pass through.

``--plain`` runs every selected case a few times eagerly with no graph and no timing: that is the
form to put under a profiler (few launches, small device footprint).

    python -m hawking_b200.utils.kernel_bench                       # all cases, timed
    python -m hawking_b200.utils.kernel_bench --case down --plain   # one case, 3 eager launches
    python -m hawking_b200.utils.kernel_bench --rows 64 --case tc_gate_up --case tc_down   # tensor cores
    python -m hawking_b200.utils.kernel_bench --rows 2048 --case attention_prefill
"""
from __future__ import annotations

import argparse
import json

import torch

H, F, V = 4096, 14336, 128256
NH, NKV, HD, BS = 32, 8, 128, 64


def _time_graph(fn, iters: int) -> float:
    for i in range(3):
        fn(i)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        fn(0)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1000.0 / iters


def build_cases(dev: str = "cuda", ctx: int = 2048, rows: int = 1, only=None, bn: int = 0):
    from hawking_b200 import ops
    from hawking_b200.formats.ggml import GgmlType
    from hawking_b200.ops import Q8Act, QWeight

    g = torch.Generator(device=dev).manual_seed(0)

    def w(n, k):
        return QWeight.random(GgmlType.Q4_K, n, k, 0.02, g, dev)

    def copies(*shape_list):
        one = sum(n * k for n, k in shape_list) * 144 // 256
        reps = max(1, -(-(256 << 20) // one))
        return [[w(n, k) for n, k in shape_list] for _ in range(reps)]

    cases = {}
    if only is not None and all(c.startswith("tc_") or c == "attention_prefill" for c in only):
        return _tc_cases(dev, ctx, rows, g, only, bn)
    if only is not None and all(c.startswith("mla_") for c in only):
        return _mla_cases(dev, ctx, rows, g)
    wo, wd, wqkv, wgu = copies((H, H)), copies((H, F)), copies((6144, H)), copies((F, H), (F, H))
    x = torch.randn(rows, H, device=dev)
    nw = torch.ones(H, device=dev)
    xa = Q8Act(rows, H, dev)
    ops.rmsnorm_q8(x, nw, 1e-5, xa)
    ha = Q8Act(rows, F, dev)
    ops.rmsnorm_q8(torch.randn(rows, F, device=dev), None, 1e-5, ha, norm=False)
    hq = Q8Act(rows, F, dev)
    y = torch.zeros(rows, 6144, device=dev)
    cases["rmsnorm_q8"] = (lambda i: ops.rmsnorm_q8(x, nw, 1e-5, xa), rows * H * 4 * 2)
    cases["qkv"] = (lambda i: ops.gemv(wqkv[i % len(wqkv)][0], xa, y), wqkv[0][0].nbytes)
    cases["o_proj"] = (lambda i: ops.gemv(wo[i % len(wo)][0], xa, y[:, :H], residual=True), wo[0][0].nbytes)
    cases["gate_up_swiglu"] = (lambda i: ops.gemv_swiglu(*wgu[i % len(wgu)], xa, hq),
                               wgu[0][0].nbytes + wgu[0][1].nbytes)
    cases["down"] = (lambda i: ops.gemv(wd[i % len(wd)][0], ha, y[:, :H], residual=True), wd[0][0].nbytes)

    if only is not None and not any(c.startswith("attention") or c == "lm_head" for c in only):
        return cases
    nblk = (ctx + BS - 1) // BS
    kc = torch.randn(nblk * rows, NKV, BS, HD, device=dev).bfloat16()
    vc = torch.randn_like(kc)
    tables = torch.arange(nblk * rows, dtype=torch.int32, device=dev).view(rows, nblk).contiguous()
    rs = torch.arange(rows, dtype=torch.int32, device=dev)
    rc = torch.full((rows,), ctx, dtype=torch.int32, device=dev)
    q = torch.randn(rows, NH, HD, device=dev)
    splits = 1
    while splits < 8 and rows * NKV * splits < 148:
        splits *= 2
    old_splits = max(1, min(64, (296 + rows * NKV - 1) // (rows * NKV)))
    po = torch.zeros(rows * old_splits * NH * HD, device=dev)
    pl = torch.zeros(rows * old_splits * NH, device=dev)
    cnt = torch.zeros(rows * NKV, dtype=torch.int32, device=dev)
    att = Q8Act(rows, NH * HD, dev)
    cases["attention"] = (
        lambda i: ops.attention_decode(q, kc, vc, tables, rs, rc, HD ** -0.5, splits, po, pl, out_q8=att,
                                     counters=cnt),
        rows * ctx * NKV * HD * 2 * 2)
    cases["attention_scratch"] = (
        lambda i: ops.attention_decode(q, kc, vc, tables, rs, rc, HD ** -0.5, old_splits, po, pl, out_q8=att,
                                       counters=cnt, cluster=False),
        rows * ctx * NKV * HD * 2 * 2)

    if only is not None and "lm_head" not in only:
        return cases
    wl = w(V, H)
    logits = torch.zeros(rows, V, device=dev)
    cases["lm_head"] = (lambda i: ops.gemv(wl, xa, logits), wl.nbytes)
    return cases


def _mla_cases(dev, ctx, rows, g):
    """Absorbed MLA decode over a ``ctx``-token bf16 latent cache (576 per token): all 64 heads of
    the DeepSeek-V3-style config (one GPU) and the 8 heads of one rank at TP8."""
    from hawking_b200._ext import kernels
    K = kernels()
    bs = 64
    nblk = (ctx + bs - 1) // bs
    cache = torch.randn(nblk * rows, bs, 576, device=dev).bfloat16()
    tables = torch.arange(nblk * rows, dtype=torch.int32, device=dev).view(rows, nblk).contiguous()
    rs = torch.arange(rows, dtype=torch.int32, device=dev)
    rc = torch.full((rows,), ctx, dtype=torch.int32, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    cases = {}
    for nh in (64, 8):
        ql, qp = torch.randn(rows, nh, 512, device=dev), torch.randn(rows, nh, 64, device=dev)
        o = torch.zeros(rows, nh, 512, device=dev)
        groups = nh // K.mla_heads_per_cta(nh, rows)
        splits = 1
        while splits < 8 and rows * groups * splits < 148:
            splits *= 2
        cases[f"mla_flash_h{nh}"] = (
            lambda i, ql=ql, qp=qp, o=o: K.mla_decode(ql, qp, cache, tables, rs, rc, 0.07, 0, o, st, True),
            rows * ctx * 576 * 2, 2.0 * rows * ctx * nh * (576 + 512))
        cases[f"mla_decode_h{nh}"] = (
            lambda i, ql=ql, qp=qp, o=o, splits=splits: K.mla_decode(ql, qp, cache, tables, rs, rc, 0.07, splits, o, st,
                                                                     True),
            rows * ctx * 576 * 2, 2.0 * rows * ctx * nh * (576 + 512))
    return cases


def _tc_cases(dev, ctx, rows, g, only, bn=0):
    """Tensor-core cases at ``rows`` tokens: the Q4_K dequant GEMMs of one layer and the causal
    prefill attention of one ``rows``-token chunk at the end of a ``ctx``-token prompt."""
    from hawking_b200 import ops
    from hawking_b200.formats.ggml import GgmlType
    from hawking_b200.ops import QWeight

    cases = {}
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    x = torch.randn(rows, F, device=dev).bfloat16()
    for name, (n, k) in (("tc_gate_up", (2 * F, H)), ("tc_down", (H, F)), ("tc_qkv", (6144, H)),
                         ("tc_o", (H, H))):
        if name not in only:
            continue
        one = n * k * 144 // 256
        ws = [QWeight.random(GgmlType.Q4_K, n, k, 0.02, g, dev) for _ in range(max(1, -(-(256 << 20) // one)))]
        y = torch.zeros(rows, n, device=dev)
        cases[name] = (lambda i, ws=ws, y=y, k=k: ops.tc_gemm(ws[i % len(ws)], x[:, :k], y, status, atomic=True,
                                                                         bn=bn),
                       one, 2.0 * rows * n * k)
    if "tc_gate_up_swiglu" in only:
        from hawking_b200.ops import cat_rows
        one = 2 * F * H * 144 // 256
        ws = [cat_rows([QWeight.random(GgmlType.Q4_K, F, H, 0.02, g, dev), QWeight.random(GgmlType.Q4_K, F, H, 0.02, g, dev)])
              for _ in range(max(1, -(-(256 << 20) // one)))]
        hb = torch.zeros(rows, F, dtype=torch.bfloat16, device=dev)
        cases["tc_gate_up_swiglu"] = (lambda i: ops.tc_gemm_swiglu(ws[i % len(ws)], x[:, :H], hb, status, bn=bn),
                                      one, 2.0 * rows * 2 * F * H)
    if "attention_prefill" in only:
        nblk = (ctx + BS - 1) // BS
        kc = torch.randn(nblk, NKV, BS, HD, device=dev).bfloat16()
        vc = torch.randn_like(kc)
        tables = torch.arange(nblk, dtype=torch.int32, device=dev).view(1, nblk).contiguous()
        rs = torch.zeros(rows, dtype=torch.int32, device=dev)
        rc = torch.arange(ctx - rows + 1, ctx + 1, dtype=torch.int32, device=dev)
        q = torch.randn(rows, NH, HD, device=dev)
        ob = torch.zeros(rows, NH * HD, dtype=torch.bfloat16, device=dev)
        keys = float(rc.sum().item())  # causal keys summed over the rows
        cases["attention_prefill"] = (
            lambda i: ops.attention_prefill(q, kc, vc, tables, rs, rc, HD ** -0.5, out_bf16=ob),
            ctx * NKV * HD * 2 * 2, 4.0 * keys * NH * HD)
    return cases


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--case", action="append", help="case name (repeatable); default all")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--rows", type=int, default=1, help="decode batch (GEMV rows)")
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--plain", action="store_true", help="3 eager launches per case, no timing")
    ap.add_argument("--bn", type=int, default=0, help="tensor-core token tile (0: the engine's choice)")
    args = ap.parse_args(argv)
    cases = build_cases(ctx=args.ctx, rows=args.rows, only=args.case, bn=args.bn)
    names = args.case or list(cases)
    for n in names:
        fn, nbytes = cases[n][:2]
        flops = cases[n][2] if len(cases[n]) > 2 else None
        if args.plain:
            for i in range(3):
                fn(i)
            torch.cuda.synchronize()
            print(json.dumps({"case": n, "plain": True}))
            continue
        us = _time_graph(fn, args.iters)
        rec = {"case": n, "rows": args.rows, "bn": args.bn, "us": round(us, 3), "gb_s": round(nbytes / us / 1e3, 1),
               "bytes": int(nbytes)}
        if flops:
            rec["tflops"] = round(flops / us / 1e6, 1)
        print(json.dumps(rec), flush=True)


if __name__ == "__main__":
    main()
