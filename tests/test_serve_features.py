"""Serving features on the CPU: JSON-mode constraint automaton, tool-call rendering and extraction,
the native /v1/hawking routes and tool calls through the HTTP server (scripted engine).

Parity: crates/hawking-core/src/json_constrain.rs, crates/hawking-serve/src/tool_calls.rs:43-123,
crates/hawking-serve/src/http.rs:272-276 (/v1/hawking routes), :389-420 (context), :971-1140.
"""
import http.client
import json
import threading

import numpy as np
import pytest

from hawking_b200.serve import ServeLoop
from test_tokenizer import bpe_spec


# ---- JSON constraint ----
@pytest.mark.parametrize("text", ['{}', '{"a": 1}', ' {"a": [1, -2.5e3, true, null, "x\\"y"], "b": {"c": false}} ',
                                  '{"u": "\\u00e9\\n", "n": 0.25}'])
def test_json_constraint_accepts_complete_objects(native, text):
    assert native.JsonConstraint.validate(text)
    c = native.JsonConstraint(lenient_whitespace=True)
    for ch in text.encode():  # byte by byte, every prefix is acceptable
        assert c.advance(bytes([ch])), (text, ch)
    assert c.done


@pytest.mark.parametrize("text", ['[1]', '{"a" 1}', '{"a": 01}', '{"a": tru}', '{a: 1}', '{"a": 1,}', '{"a": "x\ny"}',
                                  '{"a": 1}}', '"s"', '{"a": 1.}'])
def test_json_constraint_rejects(native, text):
    assert not native.JsonConstraint.validate(text)


def test_json_constraint_generation_makes_progress(native):
    c = native.JsonConstraint()
    assert not c.accepts(b" ") and not c.accepts(b"\n")  # the object starts at once
    assert c.advance(b'{"a": 1,')
    assert c.accepts(b" ") and not c.accepts(b"  ")   # one whitespace byte at a time
    assert c.advance(b" ") and not c.accepts(b"\n")
    assert c.accepts(b'"k "')                          # inside strings anything printable goes


def test_json_constraint_token_choice(native):
    tok = native.Tokenizer.from_spec(bpe_spec(native))
    c = native.JsonConstraint()
    assert c.advance(b'{"a":')
    logits = np.full(tok.vocab_size, -10.0, dtype=np.float32)
    bad = tok.encode("hello", False)[0]   # cannot start a JSON value
    good = tok.find("1") if tok.find("1") >= 0 else tok.encode("1", False)[0]
    logits[bad] = 5.0
    logits[good] = 1.0
    assert c.pick(tok, logits) == good
    masked = logits.copy()
    c.mask(tok, masked)
    assert masked[bad] == -np.inf and masked[good] == 1.0
    for e in tok.eog_ids():  # end of generation only once the object is closed
        assert masked[e] == -np.inf


# ---- tool calls ----
TOOLS = [{"type": "function", "function": {"name": "get_weather", "description": "weather",
                                           "parameters": {"type": "object", "properties": {"city": {"type": "string"}}}}}]


def test_tools_preamble_and_extraction(native):
    pre = native.render_tools_preamble(json.dumps(TOOLS))
    assert "<tools>" in pre and '"name":"get_weather"' in pre and "<tool_call>" in pre
    tagged = 'Sure.\n<tool_call>\n{"name": "get_weather", "arguments": {"city": "Paris"}}\n</tool_call>'
    calls = native.extract_tool_calls(tagged, ["get_weather"])
    assert calls == [("call_0", "get_weather", '{"city":"Paris"}')]
    # untagged: only a declared tool name counts
    assert native.extract_tool_calls('{"name": "get_weather", "arguments": "{\\"city\\": \\"Oslo\\"}"}',
                                     ["get_weather"]) == [("call_0", "get_weather", '{"city":"Oslo"}')]
    assert native.extract_tool_calls('My friend {"name": "Bob"} says hi', ["get_weather"]) == []
    two = '<tool_call>{"name": "a", "arguments": {}}</tool_call><tool_call>{"name": "b"}</tool_call>'
    assert [c[1] for c in native.extract_tool_calls(two, [])] == ["a", "b"]


# ---- HTTP ----
class Scripted:
    max_batch = 4

    def __init__(self, tok, script):
        self.script = tok.encode(script, False)
        self.reqs, self.params = {}, []
        self.next_id = 1

    def add_request(self, prompt, params):
        rid = self.next_id
        self.next_id += 1
        self.reqs[rid] = {"n": 0, "max": params.max_tokens, "prompt": list(prompt)}
        self.params.append(params)
        return rid

    def abort(self, rid):
        self.reqs.pop(rid, None)

    def has_work(self):
        return bool(self.reqs)

    def step(self):
        out = []
        for rid, r in list(self.reqs.items()):
            done = r["n"] >= len(self.script) - 1 or r["n"] + 1 >= r["max"]
            out.append((rid, self.script[r["n"]], 1 if done else 0))
            r["n"] += 1
            if done:
                del self.reqs[rid]
        return out


CALL = '<tool_call>\n{"name": "get_weather", "arguments": {"city": "Paris"}}\n</tool_call>'


@pytest.fixture(scope="module")
def served(native):
    tok = native.Tokenizer.from_spec(bpe_spec(native))
    eng = Scripted(tok, CALL)
    loop = ServeLoop(eng, tok, port=0, model_id="m", max_context=4096).start()
    th = loop.run_in_thread()
    yield loop, eng, tok
    loop.stop()
    th.join(timeout=5)


def call(loop, method, path, body=None):
    c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=30)
    c.request(method, path, body=json.dumps(body) if body is not None else None)
    r = c.getresponse()
    out = r.status, r.read().decode()
    c.close()
    return out


def test_chat_tool_calls_response(served):
    loop, eng, _ = served
    st, body = call(loop, "POST", "/v1/chat/completions",
                    {"messages": [{"role": "user", "content": "weather in Paris?"}], "tools": TOOLS,
                     "max_tokens": 200, "temperature": 0})
    assert st == 200, body
    o = json.loads(body)
    ch = o["choices"][0]
    assert ch["finish_reason"] == "tool_calls"
    tc = ch["message"]["tool_calls"][0]
    assert tc["type"] == "function" and tc["function"]["name"] == "get_weather"
    assert json.loads(tc["function"]["arguments"]) == {"city": "Paris"}
    assert ch["message"]["content"] is None


def test_chat_tools_stream_and_json_mode_flag(served):
    loop, eng, _ = served
    c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=30)
    c.request("POST", "/v1/chat/completions", body=json.dumps(
        {"messages": [{"role": "user", "content": "x"}], "tools": TOOLS, "max_tokens": 200, "stream": True,
         "response_format": {"type": "json_object"}}))
    r = c.getresponse()
    events = [line[6:] for line in r.read().decode().split("\n") if line.startswith("data: ")]
    c.close()
    assert events[-1] == "[DONE]"
    last = json.loads(events[-2])
    assert last["choices"][0]["finish_reason"] == "tool_calls"
    assert last["choices"][0]["delta"]["tool_calls"][0]["function"]["name"] == "get_weather"
    assert eng.params[-1].json_mode


def test_hawking_native_routes(served):
    loop, eng, tok = served
    st, body = call(loop, "GET", "/v1/hawking/context")
    assert st == 200
    ctx = json.loads(body)
    assert ctx["ctx_len_native"] == 4096 and ctx["max_batch"] == 4 and "free_slots" in ctx
    st, body = call(loop, "GET", "/v1/hawking/surface")
    sf = json.loads(body)
    assert "POST /v1/hawking/generate" in sf["routes"] and sf["features"]["tool_calls"]
    st, body = call(loop, "POST", "/v1/hawking/generate", {"prompt": "hi", "max_tokens": 5})
    assert st == 200, body
    g = json.loads(body)
    assert g["stats"]["completion_tokens"] == 5 and g["stats"]["prompt_tokens"] >= 1
    assert g["text"] == tok.decode(eng.script[:5])
    c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=30)
    c.request("POST", "/v1/hawking/tokens", body=json.dumps({"prompt": "hi", "max_tokens": 4}))
    r = c.getresponse()
    events = [line[6:] for line in r.read().decode().split("\n") if line.startswith("data: ")]
    c.close()
    assert events[-1] == "[DONE]"
    assert [json.loads(e)["token"] for e in events[:-1]] == eng.script[:4]
    assert eng.params[-1].temperature == 0.0
    st, _ = call(loop, "POST", "/v1/hawking/generate", {"prompt": ""})
    assert st == 400


class Failing(Scripted):
    """Raises on its third step (a failed collective, say)."""

    def __init__(self, tok, script):
        super().__init__(tok, script)
        self.n = 0

    def step(self):
        self.n += 1
        if self.n == 3:
            raise RuntimeError("tensor-parallel collective reported device error 3 (peer timeout)")
        return super().step()


def test_engine_failure_drains_and_reports_unhealthy(native):
    tok = native.Tokenizer.from_spec(bpe_spec(native))
    eng = Failing(tok, " hello world hello there hello")
    loop = ServeLoop(eng, tok, port=0, model_id="m").start()
    th = loop.run_in_thread()
    try:
        assert call(loop, "GET", "/healthz")[0] == 200
        st, body = call(loop, "POST", "/v1/completions", {"prompt": "hi", "max_tokens": 50})
        assert st == 503 and "peer timeout" in body
        st, body = call(loop, "GET", "/healthz")
        assert st == 503 and json.loads(body)["status"] == "unhealthy"
        assert call(loop, "POST", "/v1/completions", {"prompt": "again", "max_tokens": 5})[0] == 503
        assert not eng.reqs  # the in-flight request was aborted in the engine
    finally:
        loop.stop()
        th.join(timeout=5)


def test_latency_quantiles_on_metrics(served):
    loop, _, _ = served
    for _ in range(3):
        assert call(loop, "POST", "/v1/completions", {"prompt": "hi", "max_tokens": 6})[0] == 200
    loop._latency_metrics()
    st, text = call(loop, "GET", "/metrics")
    assert st == 200
    for name in ("hawking_ttft_ms_p50", "hawking_ttft_ms_p99", "hawking_itl_ms_p95"):
        assert name in text, text
