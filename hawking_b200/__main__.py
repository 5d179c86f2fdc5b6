"""``python -m hawking_b200 <command>``: the command-line front end.

Commands:
  serve      OpenAI-compatible HTTP server (see ``python -m hawking_b200 serve --help``)
  generate   one prompt through the engine, text out (``--gguf`` model or ``--preset`` random weights)
  tokenize   text -> token ids with a GGUF file's tokenizer (``--decode`` for ids -> text)
  info       a GGUF / `.gravity` / `.safetensors` file's architecture, config and tensor summary
  verify     `.gravity` integrity: per-tensor and body sha256, gaps / overlaps (exit 1 on failure)
  bench      the headline decode / TTFT benchmark (bench.py) or one kernel microbenchmark
  doctor     environment report: Python, PyTorch, CUDA devices, the native and kernel modules, NCCL
  version    package and toolchain versions

Parity: crates/hawking/src/main.rs:401-814 (clap ``Cmd``: serve, generate, tokenize, bench, doctor,
stats, version, verify; dispatch :815-1336).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from typing import List, Optional


def _cmd_generate(a) -> int:
    from ._ext import native
    from .engine.sampling import SamplingParams
    from .config import runtime_profile
    extra = {k: v for k, v in runtime_profile(a.profile).engine.items() if k != "max_batch"}
    if a.gguf:
        from .engine.engine import Engine
        eng = Engine.from_gguf(a.gguf, max_batch=1, max_ctx=a.max_ctx, **extra)
        tok = native().Tokenizer.from_gguf(native().GgufFile.open(a.gguf))
    elif a.model:
        from .serve.__main__ import path_engine
        eng, tok = path_engine(a.model, 1, a.max_ctx, a.tokenizer_gguf, **extra)
    else:
        from .serve.__main__ import preset_engine
        eng, tok = preset_engine(a.preset, a.layers, 1, a.max_ctx, **extra)
    eng.apply_profile(a.profile)
    ids = tok.encode(a.prompt, True)
    p = SamplingParams(temperature=a.temperature, top_p=a.top_p, top_k=a.top_k, seed=a.seed, max_tokens=a.max_tokens,
                       stop_ids=list(tok.eog_ids()))
    import time
    t0 = time.perf_counter()
    out = eng.generate([ids], p)[0]
    dt = time.perf_counter() - t0
    text = tok.decode([t for t in out if not tok.is_eog(t)])
    if a.stats:
        print(json.dumps(eng.stats_json()), file=sys.stderr)
    if a.json:
        print(json.dumps({"text": text, "tokens": out, "prompt_tokens": len(ids), "seconds": round(dt, 4)}))
    else:
        print(text)
        print(f"[{len(out)} tokens in {dt:.3f} s]", file=sys.stderr)
    return 0


def _cmd_tokenize(a) -> int:
    from ._ext import native
    tok = native().Tokenizer.from_gguf(native().GgufFile.open(a.gguf))
    if a.decode:
        print(tok.decode([int(x) for x in a.text.replace(",", " ").split()], skip_special=False))
    else:
        print(json.dumps(tok.encode(a.text, not a.no_special)))
    return 0


def _cmd_info(a) -> int:
    path = a.path
    with open(path, "rb") as f:
        magic = f.read(8)
    if magic.startswith(b"GGUF"):
        from .formats.gguf import GgufModel
        from .models.torch_ref import config_from_gguf
        m = GgufModel(path)
        types = {}
        n_el = 0
        for t in m.tensors.values():
            types[t.type_name] = types.get(t.type_name, 0) + 1
            n_el += t.n_elements
        out = {"format": f"GGUF v{m.version}", "architecture": m.architecture, "tensors": len(m.tensors),
               "parameters": n_el, "tensor_types": types}
        try:
            out["config"] = {k: v for k, v in vars(config_from_gguf(m)).items()}
        except Exception as e:  # noqa: BLE001 - an architecture the engine does not load
            out["config_error"] = str(e)
    elif magic == b"GRAVITY\0" or os.path.isdir(path):
        from .formats.gravity import GravityModel
        g = GravityModel(path)
        out = {"format": ".gravity", "shards": len(g.shards),
               "tensors": sum(len(s.tensors) for s in g.shards.values()),
               "architecture": next(iter(g.shards.values())).architecture if g.shards else {}}
    elif path.endswith(".safetensors"):
        from .formats.safetensors import SafeTensors, SafetensorsError, native_scale_pairs
        st = SafeTensors(path)
        dtypes = {}
        for t in st.tensors.values():
            dtypes[t.dtype] = dtypes.get(t.dtype, 0) + 1
        out = {"format": "safetensors", "tensors": len(st.tensors), "tensor_dtypes": dtypes,
               "metadata": st.metadata}
        try:
            pairs = native_scale_pairs(st)
            kinds = {}
            for p in pairs.values():
                kinds[p.kind] = kinds.get(p.kind, 0) + 1
            out["native_pairs"] = kinds
        except SafetensorsError as e:
            out["native_pairs_error"] = str(e)
    else:
        print(f"{path}: not a GGUF, .gravity or .safetensors file", file=sys.stderr)
        return 2
    print(json.dumps(out, indent=1, default=str))
    return 0


def _cmd_verify(a) -> int:
    from .formats.gravity import GravityModel
    rep = GravityModel(a.path).verify()
    print(json.dumps(rep, indent=1, default=str))
    ok = all(bool(r.get("ok", False)) for r in rep.values())
    return 0 if ok else 1


def _cmd_bench(a, rest: List[str]) -> int:
    if a.kernel:
        from .utils import kernel_bench
        kernel_bench.main(rest)
        return 0
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, here)
    import bench  # the repository's headline benchmark (one JSON line)
    sys.argv = ["bench.py"] + rest
    return int(bench.main() or 0)


def _cmd_doctor(a) -> int:
    rep = {"python": sys.version.split()[0]}
    try:
        import torch
        rep["torch"] = torch.__version__
        rep["cuda_available"] = torch.cuda.is_available()
        if torch.cuda.is_available():
            rep["devices"] = [{"name": torch.cuda.get_device_name(i),
                               "capability": "sm_%d%d" % torch.cuda.get_device_capability(i),
                               "memory_gb": round(torch.cuda.get_device_properties(i).total_memory / 1e9, 1)}
                              for i in range(torch.cuda.device_count())]
            rep["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
    except Exception as e:  # noqa: BLE001
        rep["torch_error"] = str(e)
    try:
        from ._ext import native
        n = native()
        rep["native_module"] = n.__file__
        rep["nvtx"] = bool(n.trace_available())
    except Exception as e:  # noqa: BLE001
        rep["native_error"] = str(e)
    try:
        from ._ext import kernels
        rep["kernel_module"] = kernels().__file__
    except Exception as e:  # noqa: BLE001
        rep["kernel_module_error"] = str(e)
    from .config import ENV_FLAGS
    rep["env"] = {k: os.environ[k] for k in ENV_FLAGS if k in os.environ}
    print(json.dumps(rep, indent=1))
    return 0


def _cmd_version(a) -> int:
    from . import __version__
    out = {"hawking_b200": __version__}
    try:
        import torch
        out["torch"] = torch.__version__
        out["cuda"] = torch.version.cuda
    except Exception:  # noqa: BLE001
        pass
    print(json.dumps(out))
    return 0


def main(argv: Optional[List[str]] = None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "serve":
        from .serve.__main__ import main as serve_main
        serve_main(argv[1:])
        return 0
    ap = argparse.ArgumentParser(prog="python -m hawking_b200", description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    sub.add_parser("serve", help="OpenAI-compatible HTTP server")
    g = sub.add_parser("generate", help="generate text for one prompt")
    g.add_argument("--gguf")
    g.add_argument("--model", help="a GGUF file or a .gravity artifact (container sniffed)")
    g.add_argument("--tokenizer-gguf", default=None, help="with --model: the tokenizer of a .gravity artifact")
    g.add_argument("--preset")
    g.add_argument("--layers", type=int, default=0)
    g.add_argument("--prompt", required=True)
    g.add_argument("--max-tokens", type=int, default=64)
    g.add_argument("--max-ctx", type=int, default=None)
    g.add_argument("--temperature", type=float, default=0.0)
    g.add_argument("--top-p", type=float, default=1.0)
    g.add_argument("--top-k", type=int, default=0)
    g.add_argument("--seed", type=int, default=42)
    g.add_argument("--json", action="store_true")
    g.add_argument("--profile", default="default", help="runtime profile: default, fast, race, efficient, exact")
    g.add_argument("--stats", action="store_true", help="print the engine's stats JSON to stderr")
    t = sub.add_parser("tokenize", help="text <-> token ids")
    t.add_argument("--gguf", required=True)
    t.add_argument("text")
    t.add_argument("--decode", action="store_true", help="the text is a list of ids to decode")
    t.add_argument("--no-special", action="store_true", help="do not add the BOS token")
    i = sub.add_parser("info", help="summary of a GGUF, .gravity or .safetensors file")
    i.add_argument("path")
    v = sub.add_parser("verify", help="verify a .gravity shard or directory")
    v.add_argument("path")
    b = sub.add_parser("bench", help="headline benchmark (bench.py flags) or --kernel microbenchmarks")
    b.add_argument("--kernel", action="store_true", help="run hawking_b200.utils.kernel_bench with the remaining flags")
    sub.add_parser("doctor", help="environment report")
    sub.add_parser("version", help="versions")
    a, rest = ap.parse_known_args(argv)
    if a.cmd == "bench":
        return _cmd_bench(a, rest)
    if rest:
        ap.error("unrecognized arguments: " + " ".join(rest))
    if a.cmd == "generate":
        if sum(map(bool, (a.gguf, a.preset, a.model))) != 1:
            ap.error("give exactly one of --gguf, --model and --preset")
        return _cmd_generate(a)
    return {"tokenize": _cmd_tokenize, "info": _cmd_info, "verify": _cmd_verify, "doctor": _cmd_doctor,
            "version": _cmd_version}[a.cmd](a)


if __name__ == "__main__":
    sys.exit(main())
