"""``python -m hawking_b200.serve --gguf MODEL.gguf [--port 8000]``: serve a GGUF model over the
OpenAI-compatible HTTP API on one GPU."""
from __future__ import annotations

import argparse

from .._ext import native
from ..engine.engine import Engine
from .server import ServeLoop


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gguf", required=True)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--model-id", default=None)
    ap.add_argument("--max-batch", type=int, default=8)
    ap.add_argument("--max-ctx", type=int, default=None)
    ap.add_argument("--chat-template", default="auto", choices=["auto", "llama3", "chatml", "deepseek", "generic"])
    ap.add_argument("--policy", type=int, default=0, help="0 default, 1 greedy-first, 2 prefix-grouped")
    args = ap.parse_args(argv)
    eng = Engine.from_gguf(args.gguf, max_batch=args.max_batch, max_ctx=args.max_ctx, policy=args.policy)
    tok = native().Tokenizer.from_gguf(native().GgufFile.open(args.gguf))
    loop = ServeLoop(eng, tok, host=args.host, port=args.port, chat_template=args.chat_template,
                     model_id=args.model_id or args.gguf.rsplit("/", 1)[-1])
    loop.start()
    print(f"serving {args.gguf} on http://{args.host}:{loop.port}", flush=True)
    try:
        loop.run()
    except KeyboardInterrupt:
        pass
    finally:
        loop.stop()


if __name__ == "__main__":
    main()
