"""``python -m hawking_b200.serve --gguf MODEL.gguf [--port 8000]``: serve a GGUF model over the
OpenAI-compatible HTTP API on one GPU.

``--preset deepseek-v3 | qwen3-next | NAME [--layers N]`` serves random-init weights of a named
architecture instead (the fp8 MLA + MoE model or the `.gravity` hybrid DeltaNet model, which have
no GGUF of their own here) with the synthetic byte-level tokenizer, or ``--tokenizer-gguf``'s."""
from __future__ import annotations

import argparse

from .._ext import native
from ..config import RUNTIME_PROFILES, runtime_profile
from ..engine.engine import Engine
from .server import ServeLoop


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gguf", default=None)
    ap.add_argument("--preset", default=None, help="serve random-init weights of this architecture preset")
    ap.add_argument("--layers", type=int, default=0, help="with --preset: override the layer count")
    ap.add_argument("--tokenizer-gguf", default=None, help="with --preset: the tokenizer (default: synthetic)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model-id", default=None)
    ap.add_argument("--max-batch", type=int, default=None)
    ap.add_argument("--max-ctx", type=int, default=None)
    ap.add_argument("--chat-template", default="auto", choices=["auto", "llama3", "chatml", "deepseek", "generic"])
    ap.add_argument("--policy", type=int, default=None, help="0 default, 1 greedy-first, 2 prefix-grouped")
    ap.add_argument("--profile", default="default", choices=sorted(RUNTIME_PROFILES),
                    help="runtime profile (lever plan): " + "; ".join(p.contract for p in RUNTIME_PROFILES.values()))
    args = ap.parse_args(argv)
    plan = runtime_profile(args.profile)
    # explicit flags win over the profile's engine overrides
    max_batch = args.max_batch if args.max_batch is not None else int(plan.engine.get("max_batch", 8))
    policy = args.policy if args.policy is not None else int(plan.engine.get("policy", 0))
    extra = {k: v for k, v in plan.engine.items() if k not in ("max_batch", "policy")}
    if (args.gguf is None) == (args.preset is None):
        ap.error("give exactly one of --gguf and --preset")
    if args.gguf:
        eng = Engine.from_gguf(args.gguf, max_batch=max_batch, max_ctx=args.max_ctx, policy=policy, **extra)
        tok = native().Tokenizer.from_gguf(native().GgufFile.open(args.gguf))
        name = args.gguf.rsplit("/", 1)[-1]
    else:
        eng, tok = preset_engine(args.preset, args.layers, max_batch, args.max_ctx, args.tokenizer_gguf,
                                 policy=policy, **extra)
        name = args.preset
    eng.apply_profile(args.profile)
    loop = ServeLoop(eng, tok, host=args.host, port=args.port, chat_template=args.chat_template,
                     model_id=args.model_id or name, **plan.serve)
    loop.start()
    print(f"serving {args.gguf} on http://{args.host}:{loop.port}", flush=True)
    try:
        loop.run()
    except KeyboardInterrupt:
        pass
    finally:
        loop.stop()


def preset_engine(preset: str, layers: int = 0, max_batch: int = 8, max_ctx=None, tokenizer_gguf=None,
                  device="cuda", policy: int = 0, **build_kw):
    """(Engine, tokenizer) for random-init weights of a named architecture preset. ``build_kw``
    (EngineConfig fields) reach the dense/MoE GGUF-architecture build; the MLA and hybrid engines
    size their own prefill chunks."""
    import os
    import tempfile

    from ..formats.synth import write_tokenizer_gguf
    from ..models.config import preset as get_preset
    cfg = get_preset(preset)
    if layers:
        cfg = cfg.with_(layers=layers)
    if max_ctx:
        cfg = cfg.with_(max_ctx=max_ctx)
    if cfg.arch == "deepseek2":
        from ..models.deepseek import random_deepseek_weights
        eng = Engine.build_deepseek(cfg, random_deepseek_weights(cfg, device), device=device, max_batch=max_batch,
                                    policy=policy)
    elif cfg.arch == "qwen3next":
        from ..models.qwen_next import random_qwen_next_weights
        eng = Engine.build_qwen_next(cfg, random_qwen_next_weights(cfg, device), device=device, max_batch=max_batch,
                                     policy=policy)
    else:
        from ..models.llama import random_llama_weights
        eng = Engine.build(cfg, random_llama_weights(cfg, device), device=device, max_batch=max_batch, policy=policy,
                           **build_kw)
    path = tokenizer_gguf
    if path is None:
        path = os.path.join(tempfile.mkdtemp(prefix="hk-tok-"), "tokenizer.gguf")
        write_tokenizer_gguf(path, cfg.vocab)
    tok = native().Tokenizer.from_gguf(native().GgufFile.open(path))
    return eng, tok


if __name__ == "__main__":
    main()
