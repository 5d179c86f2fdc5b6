"""Serving loop: the native HTTP server on its own threads, the engine stepped here.

``ServeLoop.run()`` alternates between admitting requests that the server parsed and tokenized
(``HttpServer.poll``), one engine step (continuous batching: every running sequence decodes
while prompts prefill in budgeted chunks), and pushing the sampled tokens back
(``HttpServer.push``), which the connection threads stream as SSE or collect into one JSON
response. Client disconnects and stop strings come back through ``take_cancelled`` and abort the
request in the engine. Embedding requests are answered between steps.

Parity: crates/hawking-serve/src/lib.rs:525-1121 (run: admission, Phase A prefill, Phase B decode,
Phase C stream/release), crates/hawking-serve/src/http.rs:1410 (embeddings), :329-365 (metrics).
"""
from __future__ import annotations

import threading
import time
from typing import Dict, List, Optional

from .._ext import native
from ..engine.sampling import SamplingParams


class ServeLoop:
    def __init__(self, engine, tokenizer, host: str = "127.0.0.1", port: int = 8000, model_id: str = "hawking-b200",
                 chat_template: str = "auto", max_context: Optional[int] = None, max_queue: Optional[int] = None,
                 default_max_tokens: int = 256, request_timeout_s: float = 600.0):
        o = native().ServeOptions()
        o.host, o.port, o.model_id, o.chat_template = host, port, model_id, chat_template
        o.max_context = int(max_context or getattr(getattr(engine, "cfg", None), "max_ctx", 8192))
        o.max_queue = int(max_queue or 8 * getattr(engine, "max_batch", 64))
        o.default_max_tokens = default_max_tokens
        o.request_timeout_s = request_timeout_s
        o.max_batch = int(getattr(engine, "max_batch", 8))
        cfg = getattr(engine, "cfg", None)
        o.architecture = str(getattr(cfg, "arch", "llama"))
        model = getattr(engine, "model", None)
        if model is not None and hasattr(model, "ssm_state"):  # recurrent state per sequence
            per = model.ssm_state[:, 0].numel() * model.ssm_state.element_size() + \
                model.conv_state[:, 0].numel() * model.conv_state.element_size()
            o.recurrent_state_bytes = int(per)
        self.engine = engine
        self.tokenizer = tokenizer
        if hasattr(engine, "tokenizer"):
            engine.tokenizer = tokenizer  # JSON-mode requests mask tokens by their bytes
        self.server = native().HttpServer(o, tokenizer)
        self._to_server: Dict[int, int] = {}    # engine request id -> server request id
        self._to_engine: Dict[int, int] = {}
        self._stop = threading.Event()
        self.steps = 0

    @property
    def port(self) -> int:
        return self.server.port

    def start(self) -> "ServeLoop":
        self.server.start()
        return self

    def stop(self):
        self._stop.set()
        self.server.stop()

    # ---- one iteration ----
    def _admit(self, reqs) -> None:
        for r in reqs:
            if r.kind == "embedding":
                try:
                    vecs = [self.engine.embed(list(ids)) for ids in r.inputs]
                    self.server.push_embeddings(r.id, vecs)
                except Exception as e:  # noqa: BLE001 - reported to the client
                    self.server.fail(r.id, 500, f"embedding failed: {e}")
                continue
            p = SamplingParams(temperature=r.temperature, top_k=r.top_k, top_p=r.top_p,
                               repetition_penalty=r.repetition_penalty, seed=r.seed, max_tokens=r.max_tokens,
                               stop_ids=list(r.stop_ids), json_mode=bool(r.json_mode))
            try:
                erid = self.engine.add_request(list(r.prompt), p)
            except Exception as e:  # noqa: BLE001
                self.server.fail(r.id, 500, f"admission failed: {e}")
                continue
            self._to_server[erid] = r.id
            self._to_engine[r.id] = erid

    def _cancel(self) -> None:
        for sid in self.server.take_cancelled():
            erid = self._to_engine.pop(sid, None)
            if erid is not None:
                self._to_server.pop(erid, None)
                self.engine.abort(erid)

    def iterate(self, idle_wait_ms: int = 20) -> int:
        """Admit, step once, stream. Returns the number of tokens pushed."""
        self._admit(self.server.poll(0 if self.engine.has_work() else idle_wait_ms))
        self._cancel()
        if not self.engine.has_work():
            return 0
        events = self.engine.step()
        self.steps += 1
        pushed = 0
        for erid, tok, fin in events:
            sid = self._to_server.get(erid)
            if sid is None:
                continue
            self.server.push(sid, [int(tok)] if tok >= 0 else [], int(fin))
            pushed += 1
            if fin:
                self._to_server.pop(erid, None)
                self._to_engine.pop(sid, None)
        st = getattr(self.engine, "stats", None)
        if st is not None and self.steps % 16 == 0:
            self.server.set_metric("hawking_engine_steps_total", st.steps, "Engine steps", True)
            self.server.set_metric("hawking_graph_decode_steps_total", st.graph_steps,
                                   "Decode steps replayed from a captured CUDA graph", True)
            self.server.set_metric("hawking_gpu_readback_bytes_total", st.d2h_bytes,
                                   "Cumulative device-to-host readback bytes", True)
        return pushed

    def run(self, max_seconds: Optional[float] = None) -> None:
        t_end = None if max_seconds is None else time.time() + max_seconds
        while not self._stop.is_set() and (t_end is None or time.time() < t_end):
            self.iterate()

    def run_in_thread(self) -> threading.Thread:
        th = threading.Thread(target=self.run, daemon=True)
        th.start()
        return th
