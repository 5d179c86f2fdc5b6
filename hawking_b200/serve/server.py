"""Serving loop: the native HTTP server on its own threads, the engine stepped here.

``ServeLoop.run()`` alternates between admitting requests that the server parsed and tokenized
(``HttpServer.poll``), one engine step (continuous batching: every running sequence decodes
while prompts prefill in budgeted chunks), and pushing the sampled tokens back
(``HttpServer.push``), which the connection threads stream as SSE or collect into one JSON
response. Client disconnects and stop strings come back through ``take_cancelled`` and abort the
request in the engine. Embedding requests are answered between steps.

Failure handling: an engine step that raises (including a tensor-parallel collective that timed
out on a peer and reported it through its status word) fails every in-flight request with 503,
aborts them in the engine, and marks the server unhealthy (``/healthz`` 503 with the reason, new
generation requests refused). Latency metrics: TTFT (admission to first token) and inter-token
latency quantiles over the most recent requests, exported as gauges on ``/metrics``.

Parity: crates/hawking-serve/src/lib.rs:525-1121 (run: admission, Phase A prefill, Phase B decode,
Phase C stream/release), crates/hawking-serve/src/http.rs:1410 (embeddings), :329-365 (metrics).
"""
from __future__ import annotations

import threading
import time
from collections import deque
from typing import Deque, Dict, List, Optional

from .._ext import native
from ..engine.sampling import SamplingParams


class ServeLoop:
    def __init__(self, engine, tokenizer, host: str = "127.0.0.1", port: int = 8000, model_id: str = "hawking-b200",
                 chat_template: str = "auto", max_context: Optional[int] = None, max_queue: Optional[int] = None,
                 default_max_tokens: int = 256, request_timeout_s: float = 600.0, gather_ms: float = 0.0):
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
        self.healthy = True
        self._t_admit: Dict[int, float] = {}    # server request id -> admission time
        self._t_last: Dict[int, float] = {}     # server request id -> last token time
        self._ttft: Deque[float] = deque(maxlen=2048)
        self._itl: Deque[float] = deque(maxlen=8192)
        # gather window: with work in flight and free batch slots, a step first waits up to this
        # long for new arrivals (wider steps, fewer weight passes per token; profile "efficient")
        self.gather_ms = float(gather_ms)

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
            except ValueError as e:  # a request this engine cannot serve (e.g. JSON mode, pruned vocabulary)
                self.server.fail(r.id, 400, str(e))
                continue
            except Exception as e:  # noqa: BLE001
                self.server.fail(r.id, 500, f"admission failed: {e}")
                continue
            self._to_server[erid] = r.id
            self._to_engine[r.id] = erid
            self._t_admit[r.id] = time.perf_counter()

    def _cancel(self) -> None:
        for sid in self.server.take_cancelled():
            erid = self._to_engine.pop(sid, None)
            if erid is not None:
                self._to_server.pop(erid, None)
                self.engine.abort(erid)

    def iterate(self, idle_wait_ms: int = 20) -> int:
        """Admit, step once, stream. Returns the number of tokens pushed."""
        wait = idle_wait_ms
        if self.engine.has_work():
            free_slots = len(self._to_engine) < getattr(self.engine, "max_batch", 0)
            wait = int(round(self.gather_ms)) if free_slots else 0
        self._admit(self.server.poll(wait))
        self._cancel()
        if not self.engine.has_work():
            return 0
        try:
            # the engine reads every device status word after each step and raises before
            # committing tokens when one is set (e.g. a peer's collective timed out)
            events = self.engine.step()
        except Exception as e:  # noqa: BLE001 - the step failed: drain and report
            self._engine_failed(e)
            return 0
        self.steps += 1
        pushed = 0
        now = time.perf_counter()
        for erid, tok, fin in events:
            sid = self._to_server.get(erid)
            if sid is None:
                continue
            self.server.push(sid, [int(tok)] if tok >= 0 else [], int(fin))
            pushed += 1
            last = self._t_last.get(sid)
            if last is None:
                t0 = self._t_admit.get(sid)
                if t0 is not None:
                    self._ttft.append((now - t0) * 1000.0)
            else:
                self._itl.append((now - last) * 1000.0)
            self._t_last[sid] = now
            if fin:
                self._to_server.pop(erid, None)
                self._to_engine.pop(sid, None)
                self._t_admit.pop(sid, None)
                self._t_last.pop(sid, None)
        if self.steps % 16 == 0:
            self._latency_metrics()
        st = getattr(self.engine, "stats", None)
        if st is not None and self.steps % 16 == 0:
            self.server.set_metric("hawking_engine_steps_total", st.steps, "Engine steps", True)
            self.server.set_metric("hawking_graph_decode_steps_total", st.graph_steps,
                                   "Decode steps replayed from a captured CUDA graph", True)
            self.server.set_metric("hawking_gpu_readback_bytes_total", st.d2h_bytes,
                                   "Cumulative device-to-host readback bytes", True)
        return pushed

    def _engine_failed(self, err: Exception) -> None:
        msg = f"engine step failed: {type(err).__name__}: {err}"
        self.healthy = False
        self.server.set_health(False, msg)
        for sid, erid in list(self._to_engine.items()):
            self.server.fail(sid, 503, msg)
            try:
                self.engine.abort(erid)
            except Exception:  # noqa: BLE001 - best effort while draining
                pass
        self._to_engine.clear()
        self._to_server.clear()
        self._t_admit.clear()
        self._t_last.clear()

    def _latency_metrics(self) -> None:
        import numpy as np
        for name, xs, what in (("hawking_ttft_ms", self._ttft, "Time to first token"),
                               ("hawking_itl_ms", self._itl, "Inter-token latency")):
            if not xs:
                continue
            a = np.asarray(xs)
            for q in (50, 95, 99):
                self.server.set_metric(f"{name}_p{q}", float(np.percentile(a, q)),
                                       f"{what} p{q} over the last {len(a)} samples, ms", False)

    def run(self, max_seconds: Optional[float] = None) -> None:
        t_end = None if max_seconds is None else time.time() + max_seconds
        while not self._stop.is_set() and (t_end is None or time.time() < t_end):
            self.iterate()

    def run_in_thread(self) -> threading.Thread:
        th = threading.Thread(target=self.run, daemon=True)
        th.start()
        return th
