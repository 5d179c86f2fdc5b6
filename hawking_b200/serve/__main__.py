"""``python -m hawking_b200.serve --gguf MODEL.gguf [--port 8000]``: serve a GGUF model over the
OpenAI-compatible HTTP API. Under ``torch.distributed.run --nproc-per-node N`` the model is
tensor parallel over the N GPUs (expert parallel for the MoE layers): rank 0 serves HTTP and the
other ranks step the same schedule in lockstep (``serve/lockstep.py``).

``--preset deepseek-v3 | qwen3-next | NAME [--layers N]`` serves random-init weights of a named
architecture instead (the fp8 MLA + MoE model or the `.gravity` hybrid DeltaNet model, which have
no GGUF of their own here) with the synthetic byte-level tokenizer, or ``--tokenizer-gguf``'s."""
from __future__ import annotations

import argparse
import os

from .._ext import native
from ..config import RUNTIME_PROFILES, runtime_profile
from ..engine.engine import Engine
from .server import ServeLoop


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gguf", default=None)
    ap.add_argument("--model", default=None, help="a GGUF file or a .gravity artifact (container sniffed)")
    ap.add_argument("--preset", default=None, help="serve random-init weights of this architecture preset")
    ap.add_argument("--layers", type=int, default=0, help="with --preset: override the layer count")
    ap.add_argument("--tokenizer-gguf", default=None,
                    help="with --preset / --model: the tokenizer, a GGUF or a tokenizer.json (default: synthetic)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model-id", default=None)
    ap.add_argument("--max-batch", type=int, default=None)
    ap.add_argument("--max-ctx", type=int, default=None)
    ap.add_argument("--chat-template", default="auto", choices=["auto", "llama3", "chatml", "deepseek", "generic"])
    ap.add_argument("--policy", type=int, default=None, help="0 default, 1 greedy-first, 2 prefix-grouped")
    ap.add_argument("--spec", type=int, default=0,
                    help="speculative decoding: n-gram drafts of up to K tokens when one greedy request decodes")
    ap.add_argument("--prefix-disk", default=None,
                    help="directory of prompt-prefix KV snapshots reused at admission (per rank under TP)")
    ap.add_argument("--vocab-prune", default=None,
                    help="JSON whitelist of token ids ({vocab_size_original, keep_token_ids}): the LM head keeps those rows")
    ap.add_argument("--vocab-first", type=int, default=0,
                    help="prune the LM head to the first N token ids (plus the end-of-generation ids)")
    ap.add_argument("--quant-tier-map", default=None,
                    help="with --gguf: JSON of per-layer FFN formats, re-quantised at load")
    ap.add_argument("--profile", default="default", choices=sorted(RUNTIME_PROFILES),
                    help="runtime profile (lever plan): " + "; ".join(p.contract for p in RUNTIME_PROFILES.values()))
    args = ap.parse_args(argv)
    plan = runtime_profile(args.profile)
    # explicit flags win over the profile's engine overrides
    max_batch = args.max_batch if args.max_batch is not None else int(plan.engine.get("max_batch", 8))
    policy = args.policy if args.policy is not None else int(plan.engine.get("policy", 0))
    extra = {k: v for k, v in plan.engine.items() if k not in ("max_batch", "policy")}
    if sum(x is not None for x in (args.gguf, args.preset, args.model)) != 1:
        ap.error("give exactly one of --gguf, --model and --preset")
    world, rank, gloo = init_ranks()
    device = f"cuda:{int(os.environ.get('LOCAL_RANK', '0'))}" if world > 1 else "cuda"
    if args.gguf:
        eng = Engine.from_gguf(args.gguf, device=device, max_batch=max_batch, max_ctx=args.max_ctx, policy=policy,
                               tp_rank=rank, tp_world=world, quant_tier_map=args.quant_tier_map, **extra)
        tok = native().Tokenizer.from_gguf(native().GgufFile.open(args.gguf))
        name = args.gguf.rsplit("/", 1)[-1]
    elif args.model:
        if world > 1:
            ap.error("--model serves on one GPU (use --gguf or --preset under tensor parallelism)")
        eng, tok = path_engine(args.model, max_batch, args.max_ctx, args.tokenizer_gguf, device=device,
                               policy=policy, **extra)
        name = os.path.basename(os.path.normpath(args.model))
    else:
        eng, tok = preset_engine(args.preset, args.layers, max_batch, args.max_ctx, args.tokenizer_gguf,
                                 device=device, policy=policy, tp_rank=rank, tp_world=world, **extra)
        name = args.preset
    eng.apply_profile(args.profile)
    if args.vocab_prune or args.vocab_first:
        if world > 1:
            ap.error("vocabulary pruning serves on one GPU")
        from ..engine.vocab_prune import PrunedVocab
        pv = PrunedVocab.load(args.vocab_prune) if args.vocab_prune else \
            PrunedVocab.first(args.vocab_first, eng.cfg.vocab, list(tok.eog_ids()))
        eng.enable_vocab_prune(pv)
        print(f"LM head pruned to {len(pv)} of {eng.cfg.vocab} tokens", flush=True)
    if args.spec:
        eng.enable_speculative(args.spec)
    if args.prefix_disk:
        eng.enable_prefix_disk(os.path.join(args.prefix_disk, f"rank{rank}") if world > 1 else args.prefix_disk)
    if rank > 0:  # follower: the leader's schedule, step for step
        from .lockstep import follow
        eng.tokenizer = tok
        try:
            follow(eng, gloo)
        finally:
            shutdown_ranks(eng)
        return
    if world > 1:
        from .lockstep import LeaderEngine
        eng = LeaderEngine(eng, gloo)
    loop = ServeLoop(eng, tok, host=args.host, port=args.port, chat_template=args.chat_template,
                     model_id=args.model_id or name, **plan.serve)
    loop.start()
    print(f"serving {name} on http://{args.host}:{loop.port}" + (f" over {world} GPUs" if world > 1 else ""),
          flush=True)
    try:
        loop.run()
    except KeyboardInterrupt:
        pass
    finally:
        loop.stop()
        if world > 1:
            eng.stop()
            shutdown_ranks(eng)


def init_ranks():
    """(world, rank, gloo group) from the torch.distributed.run environment; NCCL for the model's
    collectives, a gloo group for the lockstep broadcast."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return 1, 0, None
    import datetime

    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=torch.device("cuda", local))
    return world, dist.get_rank(), dist.new_group(backend="gloo")


def shutdown_ranks(eng) -> None:
    import torch.distributed as dist
    if not dist.is_initialized():
        return
    m = getattr(eng, "model", None)
    if m is not None and hasattr(m, "release_graphs"):
        m.release_graphs()
    tp = getattr(m, "tp", None)
    dist.barrier()
    if tp is not None:
        tp.close()
    dist.destroy_process_group()


def path_engine(path: str, max_batch: int = 8, max_ctx=None, tokenizer_gguf=None, device="cuda", policy: int = 0,
                **build_kw):
    """(Engine, tokenizer) for a model file or artifact (``Engine.from_path``): a GGUF brings its
    own tokenizer; a `.gravity` artifact takes ``tokenizer_gguf``'s or the synthetic byte-level
    one over its vocabulary."""
    import tempfile

    from ..formats.synth import write_tokenizer_gguf
    eng = Engine.from_path(path, device=device, max_batch=max_batch, max_ctx=max_ctx, policy=policy, **build_kw)
    tp = tokenizer_gguf
    if tp is None:
        is_gguf = False
        if not os.path.isdir(path):
            with open(path, "rb") as f:
                is_gguf = f.read(4) == b"GGUF"
        if is_gguf:
            tp = path
        else:
            tp = os.path.join(tempfile.mkdtemp(prefix="hk-tok-"), "tokenizer.gguf")
            write_tokenizer_gguf(tp, eng.cfg.vocab)
    return eng, load_tokenizer(tp)


def load_tokenizer(path: str):
    """A GGUF file's embedded vocabulary, or a Hugging Face tokenizer.json (with the
    tokenizer_config.json beside it when present)."""
    if path.endswith(".json"):
        cfg = os.path.join(os.path.dirname(os.path.abspath(path)), "tokenizer_config.json")
        return native().Tokenizer.from_json(path, cfg if os.path.exists(cfg) else "")
    return native().Tokenizer.from_gguf(native().GgufFile.open(path))


def preset_engine(preset: str, layers: int = 0, max_batch: int = 8, max_ctx=None, tokenizer_gguf=None,
                  device="cuda", policy: int = 0, tp_rank: int = 0, tp_world: int = 1, **build_kw):
    """(Engine, tokenizer) for random-init weights of a named architecture preset. ``build_kw``
    (EngineConfig fields) reach the dense/MoE GGUF-architecture build; the MLA and hybrid engines
    size their own prefill chunks. ``tp_world > 1``: this rank's tensor / expert parallel shard."""
    import os
    import tempfile

    from ..formats.synth import write_tokenizer_gguf
    from ..models.config import preset as get_preset
    cfg = get_preset(preset)
    if layers:
        cfg = cfg.with_(layers=layers)
    if max_ctx:
        cfg = cfg.with_(max_ctx=max_ctx)
    import torch
    dev = torch.device(device)
    if cfg.arch == "deepseek2":
        if tp_world > 1:
            from ..parallel.ep import local_deepseek_config, random_deepseek_weights_ep
            from ..parallel.tp import TPComm
            tp = TPComm(tp_rank, tp_world, 2 * cfg.layers, 8, cfg.hidden, dev)
            eng = Engine.build_deepseek(local_deepseek_config(cfg, tp_world),
                                        random_deepseek_weights_ep(cfg, tp_rank, tp_world, dev), device=device,
                                        max_batch=max_batch, policy=policy, tp=tp)
        else:
            from ..models.deepseek import random_deepseek_weights
            eng = Engine.build_deepseek(cfg, random_deepseek_weights(cfg, device), device=device, max_batch=max_batch,
                                        policy=policy)
    elif cfg.arch == "qwen3next":
        from ..models.qwen_next import random_qwen_next_weights
        if tp_world > 1:
            from ..parallel.ep import local_qwen_next_config
            from ..parallel.tp import TPComm
            tp = TPComm(tp_rank, tp_world, 2 * cfg.layers, 8, cfg.hidden, dev)
            eng = Engine.build_qwen_next(local_qwen_next_config(cfg, tp_world),
                                         random_qwen_next_weights(cfg, dev, shard=(tp_rank, tp_world)), device=device,
                                         max_batch=max_batch, policy=policy, tp=tp)
        else:
            eng = Engine.build_qwen_next(cfg, random_qwen_next_weights(cfg, device), device=device,
                                         max_batch=max_batch, policy=policy)
    elif tp_world > 1:
        from ..parallel.tp import TPComm, local_config, random_llama_weights_tp
        tp = TPComm(tp_rank, tp_world, 2 * cfg.layers, 8, cfg.hidden, dev)
        eng = Engine.build(local_config(cfg, tp_world), random_llama_weights_tp(cfg, tp_rank, tp_world, dev),
                           device=device, max_batch=max_batch, policy=policy, tp=tp, **build_kw)
    else:
        from ..models.llama import random_llama_weights
        eng = Engine.build(cfg, random_llama_weights(cfg, device), device=device, max_batch=max_batch, policy=policy,
                           **build_kw)
    path = tokenizer_gguf
    if path is None:
        path = os.path.join(tempfile.mkdtemp(prefix="hk-tok-"), "tokenizer.gguf")
        write_tokenizer_gguf(path, cfg.vocab)
    return eng, load_tokenizer(path)


if __name__ == "__main__":
    main()
