"""The inference engine: model + paged KV + C++ scheduler, driven one step at a time.

``Engine.step()`` asks the scheduler for a plan (decode rows for every running sequence plus
budgeted prefill chunks), lays the plan out as forward rows, runs the model (decode-only steps
replay a captured CUDA graph), samples on the device and reads back only the sampled ids
(4 bytes per sequence), then commits the tokens to the scheduler.

Parity: crates/hawking-core/src/engine.rs:352 (trait Engine: generate, prefill_slot,
forward_multiseq_greedy_tokens :616, copy_kv_prefix_to_slot :600, embed :687),
crates/hawking-serve/src/batch/driver.rs:52 (decode_ready_once: greedy token-only lane vs full-logits
lane), crates/hawking-serve/src/lib.rs:785-1115 (prefill phase, decode phase, stream phase).
"""
from __future__ import annotations

import itertools
import json
import os
import sys
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from .._ext import native
from ..config import check_memory_budget, env_flag
from ..models.config import ModelConfig
from ..utils.trace import trace
from .kv_cache import PagedKVCache
from .sampling import RequestRng, SamplingParams


class DeviceStatusError(RuntimeError):
    """A kernel of the step reported a failed bounded wait through a device status word
    (1 bounds guard, 2 peer timeout, 3 mbarrier timeout, 4 bad argument)."""

    NAMES = {1: "bounds guard", 2: "peer timeout", 3: "mbarrier timeout", 4: "bad argument"}

    def __init__(self, codes):
        self.codes = list(codes)
        what = ", ".join(f"{c} ({self.NAMES.get(c, 'unknown')})" for c in self.codes if c)
        super().__init__(f"device status word set: {what}; the step's tokens were discarded")


@dataclass
class RequestState:
    id: int
    params: SamplingParams
    rng: RequestRng
    output: List[int] = field(default_factory=list)
    finish: int = 0
    t_arrival: float = 0.0
    t_first: Optional[float] = None
    t_done: Optional[float] = None
    json: Optional[object] = None  # JsonConstraint of a JSON-mode request


@dataclass
class EngineStats:
    steps: int = 0
    decode_rows: int = 0
    prefill_rows: int = 0
    tokens_generated: int = 0
    h2d_bytes: int = 0
    d2h_bytes: int = 0
    graph_steps: int = 0
    step_s: float = 0.0   # wall time inside Engine.step()


class Engine:
    def __init__(self, cfg: ModelConfig, model, kv: PagedKVCache, max_batch: int = 8, max_prefill_tokens: int = 512,
                 policy: int = 0, use_graphs: bool = True, ledger: Optional[bool] = None):
        self.cfg, self.model, self.kv = cfg, model, kv
        self.max_batch = max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.sched = native().Scheduler(kv.bm, max_batch, max_prefill_tokens, policy)
        self.requests: Dict[int, RequestState] = {}
        self._ids = itertools.count(1)
        self._keep: Optional[List[int]] = None  # pruned LM head: original id of every kept row
        self.use_graphs = use_graphs
        self.stats = EngineStats()
        self._host_ids = torch.zeros(model.max_rows, dtype=torch.int32).pin_memory()
        # device status words read back after every step (model kernels' bounded waits, and the
        # tensor-parallel collectives' peer waits): a nonzero word fails the step before any of
        # its tokens are committed
        self._status_dev = [t for t in (getattr(model, "status", None),
                                        getattr(getattr(model, "tp", None), "status", None)) if t is not None]
        self._host_status = torch.zeros(max(1, len(self._status_dev)), dtype=torch.int32).pin_memory()
        self.tokenizer = None  # token bytes for JSON-mode requests (set by the server)
        # per-step cost ledger (HK_LEDGER=1 or ledger=True): host phases of every step, in us
        self.ledger_on = (os.environ.get("HK_LEDGER", "0") == "1") if ledger is None else ledger
        self.ledger: List[dict] = []
        self.profile = "default"
        self.startup: Dict[str, float] = {}  # load phases in ms (Engine.from_gguf)
        self.spec = None  # speculative decoding in the step (enable_speculative)
        self.prefix_disk = None  # disk prefix-KV reuse at admission (enable_prefix_disk)

    # ---- construction helpers ----
    @staticmethod
    def build(cfg: ModelConfig, weights, device="cuda", max_batch: int = 8, max_ctx: Optional[int] = None,
              block_size: int = 64, num_blocks: Optional[int] = None, max_rows: int = 64,
              max_prefill_tokens: int = 512, kv_fraction: float = 0.5, policy: int = 0, tp=None):
        """``tp`` (parallel.tp.TPComm): ``cfg`` and ``weights`` are this rank's tensor-parallel shard."""
        from ..models.llama import LlamaModel
        max_ctx = max_ctx or cfg.max_ctx
        if cfg.is_moe and tp is None:
            # MoE prefill decodes every expert once per forward (grouped tensor-core GEMMs):
            # prompts run in forwards of up to 2048 rows so that cost is shared by more tokens
            max_prefill_tokens = max(max_prefill_tokens, 2048)
        bpb = PagedKVCache.bytes_per_block(cfg.layers, cfg.n_kv_heads, cfg.head_dim, block_size)
        free, _ = torch.cuda.mem_get_info(device)
        if num_blocks is None:
            num_blocks = int(free * kv_fraction // bpb)
            num_blocks = min(num_blocks, max_batch * (-(-max_ctx // block_size)) + 16)
        # refuse a pool that cannot hold one full-context sequence, or that does not fit
        check_memory_budget(max(num_blocks, -(-max_ctx // block_size)) * bpb, free,
                            f"paged KV pool ({num_blocks} blocks of {block_size} tokens)", reserve_bytes=0)
        # one block-table row beyond max_batch: scratch sequences (embeddings) never starve
        kv = PagedKVCache(cfg.layers, cfg.n_kv_heads, cfg.head_dim, num_blocks, block_size, max_batch + 1,
                          -(-max_ctx // block_size), device)
        # one forward holds a whole prefill budget (the tensor-core GEMMs and prefill attention
        # want long row runs)
        model = LlamaModel(cfg, weights, kv, max_rows=max(max_rows, max_batch, max_prefill_tokens), device=device,
                           tp=tp)
        return Engine(cfg, model, kv, max_batch=max_batch, max_prefill_tokens=max_prefill_tokens, policy=policy)

    @staticmethod
    def build_deepseek(cfg: ModelConfig, weights, device="cuda", max_batch: int = 8, max_ctx: Optional[int] = None,
                       block_size: int = 64, num_blocks: Optional[int] = None, kv_fraction: float = 0.5,
                       policy: int = 0, tp=None, prefill_rows: int = 2048):
        """Engine around the MLA + MoE model (paged latent cache; decode forwards of <= 8 rows;
        prompts prefill in forwards of up to ``prefill_rows`` rows)."""
        from ..models.deepseek import LAT, ROPE, DeepSeekModel, LatentCache
        max_ctx = max_ctx or cfg.max_ctx
        max_blocks = -(-max_ctx // block_size)
        if num_blocks is None:
            free, _ = torch.cuda.mem_get_info(device)
            bpb = cfg.layers * block_size * (LAT + ROPE) * 2
            num_blocks = min(int(free * kv_fraction // bpb), (max_batch + 1) * max_blocks + 16)
        kv = LatentCache(cfg.layers, num_blocks, block_size, max_batch + 1, max_blocks, device)
        model = DeepSeekModel(cfg, weights, kv, max_rows=prefill_rows, device=device, tp=tp)
        return Engine(cfg, model, kv, max_batch=max_batch, max_prefill_tokens=model.row_limit, policy=policy)

    @staticmethod
    def build_qwen_next(cfg: ModelConfig, weights, device="cuda", max_batch: int = 8, max_ctx: Optional[int] = None,
                        block_size: int = 64, num_blocks: Optional[int] = None, kv_fraction: float = 0.5,
                        policy: int = 0, tp=None, prefill_rows: int = 2048):
        """Engine around the hybrid DeltaNet / gated-attention model: paged KV for the full-
        attention layers, one recurrent-state slot per block-table row (reset when a sequence
        starts), no prefix reuse (a cached prefix would not restore the recurrent state), and
        one row per sequence per forward (the recurrence is sequential). ``tp``: ``cfg`` and
        ``weights`` are this rank's tensor / expert-parallel shard."""
        from ..models.qwen_next import QwenNextModel
        max_ctx = max_ctx or cfg.max_ctx
        max_blocks = -(-max_ctx // block_size)
        n_full = sum(cfg.layer_is_full_attention(l) for l in range(cfg.layers))
        if num_blocks is None:
            free, _ = torch.cuda.mem_get_info(device)
            bpb = PagedKVCache.bytes_per_block(max(1, n_full), cfg.n_kv_heads, cfg.head_dim, block_size)
            num_blocks = min(int(free * kv_fraction // bpb), (max_batch + 1) * max_blocks + 16)
        kv = PagedKVCache(max(1, n_full), cfg.n_kv_heads, cfg.head_dim, num_blocks, block_size, max_batch + 1,
                          max_blocks, device, prefix_cache=False)
        # prompts prefill in forwards of up to prefill_rows rows (decode forwards take up to 8)
        model = QwenNextModel(cfg, weights, kv, max_rows=prefill_rows, max_seqs=max_batch + 1, device=device, tp=tp)
        return Engine(cfg, model, kv, max_batch=max_batch, max_prefill_tokens=max(model.row_limit, 8 * max_batch),
                      policy=policy)

    @staticmethod
    def from_config(cfg: ModelConfig, weights, config, device="cuda", tp=None) -> "Engine":
        """Engine.build with a typed ``hawking_b200.config.EngineConfig``."""
        return Engine.build(cfg, weights, device=device, tp=tp, **config.build_kwargs())

    @staticmethod
    def from_path(path: str, device="cuda", max_batch: int = 8, max_ctx: Optional[int] = None, verify: bool = True,
                  **kw):
        """Open a model file or artifact by its container: a `.gravity` artifact directory of the
        Qwen3-Next hybrid (payload sha256s verified once at admission when ``verify``), or a GGUF
        file (``from_gguf``).

        Parity: crates/hawking-core/src/model/mod.rs:120-171 (load_engine: container sniff, then
        the architecture switch)."""
        from ..formats.gravity import is_gravity
        if is_gravity(path):
            from ..models import qwen_next_artifact as qa
            if not qa.is_artifact(path):
                raise ValueError(f"{path}: a .gravity artifact of an architecture this build does not load from files")
            cfg, w = qa.load(path, device, verify=verify)
            if max_ctx:
                cfg = cfg.with_(max_ctx=max_ctx)
            return Engine.build_qwen_next(cfg, w, device=device, max_batch=max_batch,
                                          **{k: v for k, v in kw.items() if k in ("block_size", "num_blocks",
                                                                                  "kv_fraction", "policy")})
        with open(path, "rb") as f:
            magic = f.read(4)
        if magic == b"GGUF":
            return Engine.from_gguf(path, device=device, max_batch=max_batch, max_ctx=max_ctx, **kw)
        raise ValueError(f"{path}: neither a GGUF file nor a .gravity artifact")

    @staticmethod
    def from_gguf(path: str, device="cuda", max_batch: int = 8, max_ctx: Optional[int] = None,
                  tp_rank: int = 0, tp_world: int = 1, quant_tier_map: Optional[str] = None, **kw):
        """Load a GGUF model (weights re-laid for the kernels) and build an engine around it.
        ``tp_world > 1``: this rank's tensor-parallel shard (the process group must be up).
        ``quant_tier_map``: JSON of per-layer FFN formats; those weights are re-quantised on the
        device before the kernels' re-lay (engine/vocab_prune.py QuantTierMap)."""
        from ..formats.gguf import GgufModel
        from ..models.llama import load_llama_weights
        from ..models.torch_ref import config_from_gguf
        timing = env_flag("HK_STARTUP_TIMING") == "1"
        ph: Dict[str, float] = {}
        t = time.perf_counter()
        m = GgufModel(path)
        ph["open"] = (time.perf_counter() - t) * 1e3
        t = time.perf_counter()
        cfg = config_from_gguf(m)
        if max_ctx:
            cfg = cfg.with_(max_ctx=max_ctx)
        ph["config"] = (time.perf_counter() - t) * 1e3
        free, _ = torch.cuda.mem_get_info(device)
        check_memory_budget(sum(ti.nbytes for ti in m.tensors.values()), free, f"weights of {path}")
        if cfg.arch == "deepseek2":
            return Engine._deepseek_from_gguf(m, cfg, path, device, max_batch, tp_rank, tp_world, ph, timing,
                                              **{k: v for k, v in kw.items()
                                                 if k in ("block_size", "num_blocks", "kv_fraction", "policy",
                                                          "prefill_rows")})
        t = time.perf_counter()
        w = load_llama_weights(m, cfg, device)
        if quant_tier_map:
            from .vocab_prune import QuantTierMap
            QuantTierMap.load(quant_tier_map).apply(w, cfg)
        torch.cuda.synchronize(device)
        ph["weights"] = (time.perf_counter() - t) * 1e3
        t = time.perf_counter()
        if tp_world > 1:
            from ..parallel.tp import TPComm, local_config, shard_llama_weights
            w = shard_llama_weights(w, cfg, tp_rank, tp_world)
            tp = TPComm(tp_rank, tp_world, 2 * cfg.layers, 8, cfg.hidden, torch.device(device))
            eng = Engine.build(local_config(cfg, tp_world), w, device=device, max_batch=max_batch, max_ctx=max_ctx,
                               tp=tp, **kw)
        else:
            eng = Engine.build(cfg, w, device=device, max_batch=max_batch, max_ctx=max_ctx, **kw)
        ph["engine"] = (time.perf_counter() - t) * 1e3
        eng.startup = {k: round(v, 2) for k, v in ph.items()}
        if timing:
            print(json.dumps({"startup_ms": eng.startup, "path": path}), file=sys.stderr, flush=True)
        return eng

    @staticmethod
    def _deepseek_from_gguf(m, cfg, path, device, max_batch, tp_rank, tp_world, ph, timing, **kw):
        """The MLA + MoE engine over a ``deepseek2`` GGUF (models/deepseek_gguf.py); under
        ``tp_world > 1`` this rank's head / expert shard."""
        from ..models.deepseek_gguf import load_deepseek_weights
        t = time.perf_counter()
        w = load_deepseek_weights(m, cfg, device)
        ph["weights"] = (time.perf_counter() - t) * 1e3
        t = time.perf_counter()
        if tp_world > 1:
            from ..parallel.ep import local_deepseek_config, shard_deepseek_weights
            from ..parallel.tp import TPComm
            w = shard_deepseek_weights(w, cfg, tp_rank, tp_world)
            tp = TPComm(tp_rank, tp_world, 2 * cfg.layers, 8, cfg.hidden, torch.device(device))
            eng = Engine.build_deepseek(local_deepseek_config(cfg, tp_world), w, device=device, max_batch=max_batch,
                                        tp=tp, **kw)
        else:
            eng = Engine.build_deepseek(cfg, w, device=device, max_batch=max_batch, **kw)
        ph["engine"] = (time.perf_counter() - t) * 1e3
        eng.startup = {k: round(v, 2) for k, v in ph.items()}
        if timing:
            print(json.dumps({"startup_ms": eng.startup, "path": path}), file=sys.stderr, flush=True)
        return eng

    # ---- disk prefix-KV reuse ----
    def enable_prefix_disk(self, directory: str, min_blocks: int = 4, max_entries: int = 64):
        """At admission, a prompt whose longest whole-block prefix is not in the in-memory prefix
        cache but is on disk (a KV snapshot keyed by the SHA-256 of the prefix's token ids) has the
        snapshot loaded into cache blocks and registered as a cached prefix, so the scheduler
        attaches it like any in-memory hit. When a prompt's prefill completes, its longest
        whole-block prefix of at least ``min_blocks`` blocks is written to disk (LRU over
        ``max_entries`` files). Attention-only KV caches (no recurrent state).

        Parity: crates/hawking-core/src/cache/prefill_disk.rs:1-45 (rolling-hash prefix keys,
        longest-prefix lookup, LRU), crates/hawking-serve/src/http.rs:206-263 (lookup at admission)."""
        from .checkpoint import PrefixDiskCache
        self.prefix_disk = PrefixDiskCache(directory, max_entries)
        self._pd_min = max(1, min_blocks) * self.kv.block_size
        self._pd_pending: Dict[int, int] = {}  # request id -> prefix length to store after prefill
        self.stats_disk = {"hits": 0, "hit_tokens": 0, "stored": 0}

    def _prefix_from_disk(self, prompt: List[int]) -> None:
        kv, bs = self.kv, self.kv.block_size
        have = kv.bm.cached_prefix(prompt)
        top = (len(prompt) - 1) // bs * bs
        for n in range(top, max(have, self._pd_min - 1), -bs):
            path = self.prefix_disk._path(prompt[:n])
            if not os.path.exists(path):
                continue
            from .checkpoint import load_sequence
            tmp = -next(self._ids)
            try:
                toks = load_sequence(kv, tmp, path)  # sha256 of the payload verified on read
                kv.bm.commit_prefix(tmp, toks, len(toks))
                os.utime(path)  # LRU touch
                self.stats_disk["hits"] += 1
                self.stats_disk["hit_tokens"] += n
            except (ValueError, RuntimeError):
                pass  # a corrupt or foreign snapshot is a miss
            finally:
                kv.drop(tmp)
            return

    def _prefix_to_disk(self, events) -> None:
        """After a step: store the prompt prefix of requests whose prefill just completed."""
        for rid, n in list(self._pd_pending.items()):
            if self.sched.state(rid) != 2:  # not decoding yet (or gone)
                if self.sched.state(rid) == 3:
                    self._pd_pending.pop(rid, None)
                continue
            self._pd_pending.pop(rid, None)
            toks = list(self.sched.tokens(rid))[:n]
            path = self.prefix_disk._path(toks)
            if not os.path.exists(path) and self.kv.bm.num_tokens(rid) >= n:
                self.prefix_disk.store(self.kv, rid, toks)
                self.stats_disk["stored"] += 1

    # ---- requests ----
    def enable_vocab_prune(self, pv):
        """Prune the model's LM head to the whitelist ``pv`` (engine/vocab_prune.py): logits and
        sampling run over the kept rows and every emitted id is an original token id. JSON-mode
        requests are refused afterwards (the constraint masks the whole vocabulary)."""
        from .vocab_prune import apply_vocab_prune
        apply_vocab_prune(self.model, pv)
        self._keep = list(pv.keep)
        self._keep_row = {t: i for i, t in enumerate(self._keep)}

    def add_request(self, prompt: List[int], params: Optional[SamplingParams] = None) -> int:
        params = params or SamplingParams()
        if params.json_mode and getattr(self, "_keep", None) is not None:
            raise ValueError("JSON mode is not available with a pruned vocabulary")
        if self.prefix_disk is not None and len(prompt) > self._pd_min:
            self._prefix_from_disk(list(map(int, prompt)))
        rid = next(self._ids)
        if self.prefix_disk is not None and len(prompt) > self._pd_min:
            self._pd_pending[rid] = (len(prompt) - 1) // self.kv.block_size * self.kv.block_size
        self.sched.add(rid, list(map(int, prompt)), params.max_tokens, params.greedy, list(params.stop_ids),
                       self.cfg.max_ctx)
        st = RequestState(rid, params, RequestRng(params.seed), t_arrival=time.perf_counter())
        if params.json_mode:
            if self.tokenizer is None:
                raise ValueError("JSON mode needs the engine's tokenizer (Engine.tokenizer)")
            st.json = native().JsonConstraint()
        self.requests[rid] = st
        return rid

    def abort(self, rid: int):
        self.sched.abort(rid)
        self.kv.drop(rid)
        st = self.requests.get(rid)
        if st:
            st.finish = 3

    def has_work(self) -> bool:
        return not self.sched.idle()

    # ---- speculative decoding inside the step ----
    def enable_speculative(self, k: int = 4, min_accept_rate: float = 0.2):
        """Steps that decode exactly one greedy request run a speculative cycle instead: an n-gram
        draft of up to ``k`` tokens from the request's own history, verified by one forward of
        ``k + 1`` rows, the accepted tokens plus the verifier's next token committed at once. The
        output is bitwise the plain greedy output (attention splits pinned to the single-row
        count, per-row GEMV math independent of the row count). A governor turns drafting off
        while acceptance stays low. ``k = 0`` disables it.

        Parity: crates/hawking-core/src/model/qwen_dense.rs:1986-2010 (speculation inside the
        decode loop), crates/hawking-serve/src/spec_gov.rs:13-90 (governor)."""
        m = self.model
        if k <= 0:
            self.spec = None
            return
        n = native()
        self.spec = {"k": max(1, min(k, n.MAX_VERIFY_BATCH - 1, m.max_rows - 1)),
                     "gov": n.SpecGovernor(16, min_accept_rate), "drafts": {}, "cycles": 0, "drafted": 0,
                     "accepted": 0, "emitted": 0}
        if hasattr(m, "num_splits"):
            m.force_splits = m.num_splits(1)
            if hasattr(m, "release_graphs"):
                m.release_graphs()

    def _spec_eligible(self, items) -> bool:
        if self.spec is None or len(items) != 1:
            return False
        it = items[0]
        st = self.requests.get(it.id)
        return bool(it.sample and it.greedy and it.p1 - it.p0 == 1 and st is not None and st.json is None
                    and not getattr(self.model, "serial_rows", False))

    def _spec_step(self, it) -> List[tuple]:
        sp, m, kv = self.spec, self.model, self.kv
        toks = list(self.sched.tokens(it.id))
        d = sp["drafts"].get(it.id)
        if d is None:
            d = sp["drafts"][it.id] = native().NgramDraft()
            d.warm_start(toks)
        p = it.p0  # the last token's position (its KV is computed by this forward)
        k = min(sp["k"], self.requests[it.id].params.max_tokens - (len(toks) - self.sched.prompt_len(it.id)) - 1)
        draft = list(d.propose(toks[-2:], k)) if k > 0 and sp["gov"].enabled else []
        rows = [toks[-1]] + draft
        if not kv.bm.reserve(it.id, p + len(rows)):
            draft, rows = [], [toks[-1]]  # no room for the draft: a plain decode row
        kv.sync_tables([it.id])
        r = kv.row(it.id)
        slots = kv.bm.slots(it.id, p, p + len(rows))
        pos = list(range(p, p + len(rows)))
        self.stats.h2d_bytes += m.inp.upload(rows, pos, slots, [r] * len(rows), [q + 1 for q in pos])
        if hasattr(m, "long_runs"):
            m.long_runs = False
        m.forward(len(rows), "greedy")
        n = len(rows)
        self._host_ids[:n].copy_(m.next_ids[:n], non_blocking=True)
        torch.cuda.current_stream(m.dev).synchronize()
        self.stats.d2h_bytes += 4 * n
        verifier = self._host_ids[:n].tolist()
        self._check_device_status()
        emit, a = native().accept_draft(draft, verifier)
        kv.bm.truncate(it.id, p + 1 + a)
        events = self.sched.commit_run(it.id, list(emit), p + 1 + a)
        for e in events:
            d.note_token(int(e.token))
        sp["cycles"] += 1
        sp["drafted"] += len(draft)
        sp["accepted"] += a
        sp["emitted"] += len(events)
        if draft:
            sp["gov"].step(a > 0)
        else:
            sp["gov"].tick_disabled()
        self.stats.steps += 1
        self.stats.decode_rows += n
        self.stats.tokens_generated += len(events)
        now = time.perf_counter()
        out = []
        for e in events:
            out.append((e.id, e.token, e.finish))
            st = self.requests.get(e.id)
            if st is not None:
                st.output.append(e.token)
                if st.t_first is None:
                    st.t_first = now
                if e.finish:
                    st.finish = e.finish
                    st.t_done = now
                    self.kv.drop(e.id)
                    sp["drafts"].pop(e.id, None)
        return out

    def spec_stats(self) -> Optional[dict]:
        sp = self.spec
        if sp is None:
            return None
        return {k: sp[k] for k in ("k", "cycles", "drafted", "accepted", "emitted")} | {
            "accept_rate": round(sp["accepted"] / sp["drafted"], 3) if sp["drafted"] else 0.0,
            "tokens_per_cycle": round(sp["emitted"] / sp["cycles"], 3) if sp["cycles"] else 0.0}

    # ---- one step ----
    def step(self) -> List[tuple]:
        """Run one scheduler step. Returns [(request_id, token, finish_reason)] for sampled rows."""
        t0 = time.perf_counter()
        with trace("engine.step"):
            out = self._step()
        if self.prefix_disk is not None and self._pd_pending:
            self._prefix_to_disk(out)
        self.stats.step_s += time.perf_counter() - t0
        return out

    def apply_profile(self, name: str):
        """Set a runtime profile's model levers on this engine and drop captured graphs (the
        profile's engine overrides are build-time: ``config.apply_profile`` then
        ``Engine.from_config``). Returns the profile's LeverPlan."""
        from ..config import runtime_profile
        plan = runtime_profile(name)
        for k, v in plan.model.items():
            if hasattr(self.model, k):
                setattr(self.model, k, v)
        if hasattr(self.model, "release_graphs"):
            self.model.release_graphs()
        self.profile = name
        return plan

    def stats_json(self) -> dict:
        """Counters since construction: steps, rows, tokens, host<->device bytes, graph replays,
        decode tokens/s over the engine's step wall time, and the active profile.

        Parity: crates/hawking-core/src/engine.rs:321-349 (GenStats::stats_json)."""
        st = self.stats
        out = {k: getattr(st, k) for k in st.__dataclass_fields__}
        out["decode_tok_s"] = round(st.decode_rows / st.step_s, 2) if st.step_s > 0 else None
        out["profile"] = self.profile
        out["active_requests"] = len(self.requests)
        if self.startup:
            out["startup_ms"] = dict(self.startup)
        return out

    def ledger_json(self) -> str:
        """The per-step ledger as JSON lines (host microseconds per phase; the sample phase holds
        the device synchronisation, so it carries the forward's device time)."""
        return "\n".join(json.dumps(e) for e in self.ledger)

    def _step(self) -> List[tuple]:
        t0 = time.perf_counter()
        with trace("schedule"):
            plan = self.sched.schedule()
        items = plan.items
        if not items:
            return []
        if self._spec_eligible(items):
            return self._spec_step(items[0])
        m = self.model
        ids, pos, slots, rseq, rctx, sample_rows = [], [], [], [], [], []
        live = [it.id for it in items]
        self.kv.sync_tables(live)
        serial = getattr(m, "serial_rows", False)
        R = getattr(m, "row_limit", m.max_rows)
        per_item = []
        for it in items:
            toks = self.sched.tokens(it.id)
            r = self.kv.row(it.id)
            if it.p0 == 0 and hasattr(m, "reset_state"):
                m.reset_state(r)  # a new sequence on this row: fresh recurrent state
            sl = self.kv.bm.slots(it.id, it.p0, it.p1)
            per_item.append((it, toks, r, sl))
        if not serial:
            for it, toks, r, sl in per_item:
                for p in range(it.p0, it.p1):
                    ids.append(toks[p])
                    pos.append(p)
                    rseq.append(r)
                    rctx.append(p + 1)
                slots.extend(sl)
                if it.sample:
                    sample_rows.append((it, len(ids) - 1))
            bounds = [(c0, min(len(ids), c0 + R)) for c0 in range(0, len(ids), R)]
        else:
            # waves of at most one row per sequence, in position order (each wave <= R rows)
            bounds = []
            longest = max(it.p1 - it.p0 for it in items)
            for k in range(longest):
                wave = [(it, toks, r, sl) for it, toks, r, sl in per_item if it.p0 + k < it.p1]
                for w0 in range(0, len(wave), R):
                    b0 = len(ids)
                    for it, toks, r, sl in wave[w0:w0 + R]:
                        p = it.p0 + k
                        ids.append(toks[p])
                        pos.append(p)
                        rseq.append(r)
                        rctx.append(p + 1)
                        slots.append(sl[k])
                        if it.sample and p == it.p1 - 1:
                            sample_rows.append((it, len(ids) - 1))
                    bounds.append((b0, len(ids)))
        n = len(ids)
        decode_only = all(it.p1 - it.p0 == 1 for it in items)
        if hasattr(m, "long_runs"):
            m.long_runs = max((it.p1 - it.p0 for it in items), default=0) >= 16
        greedy = all(it.greedy for it, _ in sample_rows)
        mode = "greedy" if greedy else "none"
        sampled: List[int] = []
        t_sched = time.perf_counter()
        t_fwd = t_smp = 0.0
        for c0, c1 in bounds:
            ta = time.perf_counter()
            self.stats.h2d_bytes += m.inp.upload(ids[c0:c1], pos[c0:c1], slots[c0:c1], rseq[c0:c1], rctx[c0:c1])
            rows_here = [(it, r - c0) for it, r in sample_rows if c0 <= r < c1]
            with trace("forward"):
                if self.use_graphs and decode_only and c1 - c0 == n:
                    m.graph_forward(c1 - c0, mode)
                    self.stats.graph_steps += 1
                    picks = [(it, r) for it, r in rows_here]
                else:
                    k = len(rows_here)
                    if k == 0:
                        m.forward(c1 - c0, "none", n_logits=-1)
                    else:
                        if k == c1 - c0:
                            m.forward(c1 - c0, mode)
                        else:
                            m.logit_rows[:k].copy_(torch.tensor([r for _, r in rows_here], dtype=torch.int32),
                                                   non_blocking=True)
                            m.forward(c1 - c0, mode, n_logits=k)
                    picks = [(it, j) for j, (it, _) in enumerate(rows_here)] if 0 < k < c1 - c0 else rows_here
            tb = time.perf_counter()
            t_fwd += tb - ta
            if rows_here:
                with trace("sample"):
                    sampled.extend(self._sample(picks, greedy))
            t_smp += time.perf_counter() - tb
        self._check_device_status()
        if serial and sample_rows:  # back to the plan's item order (rows ran in wave order)
            by_id = {it.id: tok for (it, _), tok in zip(sample_rows, sampled)}
            sampled = [by_id[it.id] for it in items if it.id in by_id]
        events = self.sched.commit(plan, sampled)
        now = time.perf_counter()
        out = []
        for e in events:
            st = self.requests.get(e.id)
            if st is None or e.token < 0:
                continue
            st.output.append(e.token)
            if st.t_first is None:
                st.t_first = now
            if e.finish:
                st.finish = e.finish
                st.t_done = now
                self.kv.drop(e.id)
            out.append((e.id, e.token, e.finish))
        self.stats.steps += 1
        self.stats.tokens_generated += len(sampled)
        if self.ledger_on:
            t_end = time.perf_counter()
            self.ledger.append({"step": self.stats.steps, "rows": n, "decode": decode_only,
                                "sampled": len(sampled), "schedule_us": round((t_sched - t0) * 1e6, 1),
                                "launch_us": round(t_fwd * 1e6, 1), "sample_sync_us": round(t_smp * 1e6, 1),
                                "total_us": round((t_end - t0) * 1e6, 1)})
        if decode_only:
            self.stats.decode_rows += n
        else:
            self.stats.prefill_rows += n
        return out

    def _check_device_status(self):
        """Read every device status word of this step (one small copy, then a stream sync, which
        the sampled ids needed anyway) and raise DeviceStatusError when a kernel reported a failed
        bounded wait. Nothing of the step is committed then; the words stay set until
        ``clear_device_status``."""
        if not self._status_dev:
            return
        m = self.model
        for i, t in enumerate(self._status_dev):
            self._host_status[i:i + 1].copy_(t.view(-1)[:1], non_blocking=True)
        torch.cuda.current_stream(m.dev).synchronize()
        self.stats.d2h_bytes += 4 * len(self._status_dev)
        codes = [int(v) for v in self._host_status[:len(self._status_dev)].tolist()]
        if any(codes):
            raise DeviceStatusError(codes)

    def clear_device_status(self):
        """Zero the status words (and the small-batch GEMV's split-K counters, which a failed
        launch can leave half counted) after the cause was handled."""
        for t in self._status_dev:
            t.zero_()
        from ..ops import mg
        mg.MgScratch.get(self.model.dev).reset()
        if getattr(self.model, "dstep", None) is not None:
            self.model.dstep.reset()

    def _sample(self, rows_here, greedy: bool) -> List[int]:
        m = self.model
        idx = [r for _, r in rows_here]
        if greedy:
            k = len(idx)
            if idx == list(range(idx[0], idx[0] + k)):
                self._host_ids[:k].copy_(m.next_ids[idx[0]:idx[0] + k], non_blocking=True)
            else:
                self._host_ids[:k].copy_(m.next_ids[torch.tensor(idx, device=m.dev)], non_blocking=True)
            torch.cuda.current_stream(m.dev).synchronize()
            self.stats.d2h_bytes += 4 * k
            return self._host_ids[:k].tolist()
        # full-logits lane: device sampler for temperature / top-k / top-p; repetition penalty on host.
        # Under tensor parallelism the vocabulary slices are gathered first (every rank, same rows).
        gathered = getattr(m, "gathered_logits", None)
        logits = gathered(max(r for _, r in rows_here) + 1) if gathered is not None else m.logits
        keep = getattr(self, "_keep", None)
        if keep is not None:  # pruned head: rows of the logits are kept ids, emitted as original ids
            return [keep[t] for t in self._sample_rows(rows_here, logits, self._keep_row)]
        return self._sample_rows(rows_here, logits, None)

    def _sample_rows(self, rows_here, logits, keep_row) -> List[int]:
        m = self.model
        out = []
        for it, r in rows_here:
            st = self.requests[it.id]
            p = st.params
            if st.json is not None:
                out.append(self._sample_json(st, logits[r]))
                continue
            if p.temperature <= 0.0 and p.repetition_penalty == 1.0:
                torch.cuda.current_stream(m.dev).synchronize()
                out.append(int(torch.argmax(logits[r]).item()))
                continue
            if p.repetition_penalty != 1.0:
                row = logits[r].float().cpu().numpy()
                s = native().Sampler(p.seed)
                for t in self.sched.tokens(it.id)[-64:]:
                    if keep_row is None:
                        s.record(t)
                    elif t in keep_row:
                        s.record(keep_row[t])
                sp = native().SamplingParams()
                sp.temperature, sp.top_k, sp.top_p, sp.repetition_penalty = p.temperature, p.top_k, p.top_p, p.repetition_penalty
                out.append(int(s.sample(row, sp)))
                self.stats.d2h_bytes += row.nbytes
                continue
            m.temperature[r] = p.temperature
            m.top_k[r] = p.top_k
            m.top_p[r] = p.top_p
            m.uniforms[r] = st.rng.uniform()
            from .. import ops
            ops.sample(logits[r:r + 1], m.temperature[r:r + 1], m.top_k[r:r + 1], m.top_p[r:r + 1], None, None,
                       m.uniforms[r:r + 1], m.next_ids[r:r + 1])
            out.append(int(m.next_ids[r].item()))
            self.stats.d2h_bytes += 4
        return out

    def _sample_json(self, st: RequestState, logits: torch.Tensor) -> int:
        """JSON mode: the best allowed token (greedy) or a draw from the allowed tokens; the
        constraint then advances by the token's bytes. With no allowed token left, end of
        generation."""
        p = st.params
        v = logits.float().cpu().numpy().copy()
        self.stats.d2h_bytes += v.nbytes
        tok = self.tokenizer
        if p.temperature <= 0.0:
            t = st.json.pick(tok, v)
        else:
            import numpy as np
            st.json.mask(tok, v)
            z = v / p.temperature
            z -= np.max(z)
            pr = np.exp(z)
            if p.top_k > 0:
                pr[np.argsort(-pr)[p.top_k:]] = 0.0
            if pr.sum() <= 0 or not np.isfinite(pr.sum()):
                t = -1
            else:
                pr /= pr.sum()
                order = np.argsort(-pr)
                keep = np.cumsum(pr[order]) - pr[order] < p.top_p
                pr2 = np.zeros_like(pr)
                pr2[order[keep]] = pr[order[keep]]
                pr2 /= pr2.sum()
                t = int(np.searchsorted(np.cumsum(pr2), st.rng.uniform(), side="right"))
                t = min(t, len(pr2) - 1)
        if t < 0:
            eog = tok.eog_ids()
            return int(eog[0]) if eog else 0
        if not tok.is_eog(t):
            st.json.advance(tok.token_bytes(t))
        return int(t)

    def embed(self, ids: List[int]) -> List[float]:
        """L2-normalised final-position logits of a teacher-forced forward of ``ids`` on a scratch
        sequence (the reference's embedding semantics: crates/hawking-core/src/engine.rs:687-699)."""
        sid = -next(self._ids)
        try:
            logits = self.model.forward_tokens(list(map(int, ids)), seq_id=sid)
            v = logits[-1].float()
            v = v / v.norm().clamp_min(1e-8)
            self.stats.d2h_bytes += v.numel() * 4
            return v.cpu().tolist()
        finally:
            self.kv.drop(sid)

    def generate_speculative(self, prompt: List[int], params: Optional[SamplingParams] = None, k: int = 4):
        """Greedy generation of one prompt with n-gram speculative decoding (bitwise the greedy
        output). Returns (tokens, SpecStats)."""
        from .speculative import SpeculativeDecoder
        params = params or SamplingParams()
        dec = SpeculativeDecoder(self, k=k)
        out = dec.generate(prompt, params.max_tokens, params.stop_ids)
        return out, dec.stats

    # ---- convenience ----
    def generate(self, prompts: List[List[int]], params: Optional[SamplingParams] = None) -> List[List[int]]:
        rids = [self.add_request(p, params) for p in prompts]
        while self.has_work():
            self.step()
        return [self.requests[r].output for r in rids]
