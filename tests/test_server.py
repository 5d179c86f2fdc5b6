"""OpenAI-compatible HTTP server end to end on the CPU: native server + ServeLoop + a scripted engine.

Parity: crates/hawking-serve/src/http.rs (routes :265-281, healthz :307, metrics :329-365, chat
:610, completions :673, SSE [DONE] :828, embeddings :1410, 501 stubs :290-305, error body :43-91).
"""
import http.client
import json
import threading

import pytest

from hawking_b200.serve import ServeLoop
from test_tokenizer import bpe_spec

SCRIPT = " hello world hello there"


class ScriptedEngine:
    """Emits the tokens of SCRIPT in order (cycling), one per step per request; finishes on
    max_tokens (finish 1 = length)."""

    max_batch = 8

    def __init__(self, tok):
        self.script = tok.encode(SCRIPT, False)
        self.reqs = {}
        self.aborted = []
        self.next_id = 1
        self.lock = threading.Lock()

    def add_request(self, prompt, params):
        rid = self.next_id
        self.next_id += 1
        self.reqs[rid] = {"n": 0, "max": params.max_tokens, "prompt": list(prompt)}
        return rid

    def abort(self, rid):
        self.reqs.pop(rid, None)
        self.aborted.append(rid)

    def has_work(self):
        return bool(self.reqs)

    def step(self):
        out = []
        for rid, r in list(self.reqs.items()):
            tok = self.script[r["n"] % len(self.script)]
            r["n"] += 1
            fin = 1 if r["n"] >= r["max"] else 0
            out.append((rid, tok, fin))
            if fin:
                del self.reqs[rid]
        return out

    def embed(self, ids):
        n = float(len(ids))
        return [n / (n * n + 1) ** 0.5, 1 / (n * n + 1) ** 0.5]


@pytest.fixture(scope="module")
def server(native):
    tok = native.Tokenizer.from_spec(bpe_spec(native))
    eng = ScriptedEngine(tok)
    loop = ServeLoop(eng, tok, port=0, model_id="test-model", max_context=4096).start()
    th = loop.run_in_thread()
    yield loop, eng, tok
    loop.stop()
    th.join(timeout=5)


def request(loop, method, path, body=None, raw=None):
    c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=30)
    data = raw if raw is not None else (json.dumps(body) if body is not None else None)
    c.request(method, path, body=data, headers={"Content-Type": "application/json"})
    r = c.getresponse()
    payload = r.read().decode()
    c.close()
    return r.status, r.getheader("Content-Type"), payload


def expected_text(tok, n):
    script = tok.encode(SCRIPT, False)
    return tok.decode([script[i % len(script)] for i in range(n)])


def test_health_models_metrics(server):
    loop, _, _ = server
    assert request(loop, "GET", "/healthz")[::2] == (200, "ok")
    st, _, body = request(loop, "GET", "/v1/models")
    assert st == 200 and json.loads(body)["data"][0]["id"] == "test-model"
    st, ct, body = request(loop, "GET", "/metrics")
    assert st == 200 and ct.startswith("text/plain") and "hawking_requests_admitted_total" in body


def test_completion_json(server):
    loop, _, tok = server
    st, _, body = request(loop, "POST", "/v1/completions", {"prompt": "hi there", "max_tokens": 5})
    assert st == 200
    o = json.loads(body)
    assert o["object"] == "text_completion"
    assert o["choices"][0]["text"] == expected_text(tok, 5)
    assert o["choices"][0]["finish_reason"] == "length"
    assert o["usage"]["completion_tokens"] == 5
    assert o["usage"]["prompt_tokens"] == len(tok.encode("hi there"))


def test_chat_stream_sse(server):
    loop, _, tok = server
    c = http.client.HTTPConnection("127.0.0.1", loop.port, timeout=30)
    c.request("POST", "/v1/chat/completions",
              body=json.dumps({"messages": [{"role": "user", "content": "hey"}], "max_tokens": 7, "stream": True}))
    r = c.getresponse()
    assert r.status == 200 and r.getheader("Content-Type") == "text/event-stream"
    text, events, done, finish = "", [], False, None
    for line in r.read().decode().split("\n\n"):
        if not line.startswith("data: "):
            continue
        data = line[6:]
        if data == "[DONE]":
            done = True
            continue
        ev = json.loads(data)
        events.append(ev)
        ch = ev["choices"][0]
        text += ch["delta"].get("content", "")
        finish = ch["finish_reason"] or finish
    c.close()
    assert done and finish == "length"
    assert events[0]["choices"][0]["delta"]["role"] == "assistant"
    assert events[0]["object"] == "chat.completion.chunk"
    assert text == expected_text(tok, 7)


def test_stop_string_truncates_and_aborts(server):
    loop, eng, tok = server
    st, _, body = request(loop, "POST", "/v1/completions", {"prompt": "x", "max_tokens": 40, "stop": ["world"]})
    o = json.loads(body)
    assert st == 200 and o["choices"][0]["finish_reason"] == "stop"
    assert o["choices"][0]["text"] == " hello "
    for _ in range(100):
        if eng.aborted:
            break
        import time
        time.sleep(0.01)
    assert eng.aborted  # the engine request was cancelled


def test_errors(server):
    loop, _, _ = server
    st, _, body = request(loop, "POST", "/v1/chat/completions", raw="{not json")
    assert st == 400 and json.loads(body)["error"]["code"] == "invalid_json"
    st, _, body = request(loop, "POST", "/v1/chat/completions", {"messages": []})
    assert st == 400 and json.loads(body)["error"]["code"] == "missing_required_parameter"
    st, _, body = request(loop, "POST", "/v1/responses", {"input": "x"})
    assert st == 501 and json.loads(body)["error"]["type"] == "not_implemented"
    assert request(loop, "GET", "/nope")[0] == 404
    assert request(loop, "GET", "/v1/completions")[0] == 405


def test_embeddings(server):
    loop, _, tok = server
    st, _, body = request(loop, "POST", "/v1/embeddings", {"input": ["a b c", "hello"]})
    assert st == 200
    o = json.loads(body)
    assert [d["index"] for d in o["data"]] == [0, 1]
    for d in o["data"]:
        v = d["embedding"]
        assert abs(sum(x * x for x in v) - 1.0) < 1e-5


def test_concurrent_streams(server):
    loop, _, tok = server
    results = [None] * 6

    def one(i):
        st, _, body = request(loop, "POST", "/v1/completions", {"prompt": f"p{i}", "max_tokens": 3 + i})
        results[i] = json.loads(body)["choices"][0]["text"]

    ths = [threading.Thread(target=one, args=(i,)) for i in range(6)]
    for t in ths:
        t.start()
    for t in ths:
        t.join(30)
    assert results == [expected_text(tok, 3 + i) for i in range(6)]


def test_chat_templates(native):
    tok = native.Tokenizer.from_spec(bpe_spec(native))
    o = native.ServeOptions()
    o.port = 0
    srv = native.HttpServer(o, tok)
    msgs = json.dumps([{"role": "system", "content": "be brief"}, {"role": "user", "content": [{"type": "text", "text": "hi"}]}])
    assert srv.render_chat(msgs) == ("<|start_header_id|>system<|end_header_id|>\n\nbe brief<|eot_id|>"
                                     "<|start_header_id|>user<|end_header_id|>\n\nhi<|eot_id|>"
                                     "<|start_header_id|>assistant<|end_header_id|>\n\n")
    assert srv.render_chat(msgs, "chatml") == ("<|im_start|>system\nbe brief<|im_end|>\n<|im_start|>user\nhi<|im_end|>\n"
                                               "<|im_start|>assistant\n")
