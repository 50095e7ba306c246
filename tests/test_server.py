"""OpenAI-compatible server on the CPU engine (tiny model)."""
import json

import pytest


@pytest.fixture(scope="module")
def client():
    from fastapi.testclient import TestClient
    from b200ds import EngineConfig, load_engine
    from b200ds.engine.tokenizer import ByteTokenizer
    from b200ds.server.openai import EngineWorker, create_app
    eng = load_engine("tiny", ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu")
    tok = ByteTokenizer()
    eng.tokenizer = tok
    worker = EngineWorker(eng, tok).start()
    with TestClient(create_app(worker, "tiny")) as c:
        yield c
    worker.stop()


def test_completion_greedy_matches_engine(client):
    r = client.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 6, "temperature": 0})
    assert r.status_code == 200
    body = r.json()
    ids = body["choices"][0]["token_ids"]
    assert len(ids) == 6 and body["usage"]["completion_tokens"] == 6
    # greedy is deterministic: the same request gives the same tokens
    r2 = client.post("/v1/completions", json={"prompt": [5, 6, 7, 8], "max_tokens": 6, "temperature": 0})
    assert r2.json()["choices"][0]["token_ids"] == ids


def test_completion_stream(client):
    with client.stream("POST", "/v1/completions",
                       json={"prompt": "hello", "max_tokens": 5, "temperature": 0, "stream": True}) as r:
        events = [l for l in r.iter_lines() if l.startswith("data: ")]
    assert events[-1] == "data: [DONE]"
    toks = sum((json.loads(e[6:])["choices"][0].get("token_ids") or [] for e in events[:-1]), [])
    assert len(toks) == 5


def test_chat_and_models_and_metrics(client):
    r = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                  "max_tokens": 4, "temperature": 0.8, "seed": 3})
    assert r.status_code == 200
    assert r.json()["choices"][0]["message"]["role"] == "assistant"
    assert client.get("/v1/models").json()["data"][0]["id"] == "tiny"
    m = client.get("/metrics").text
    assert "b200ds_requests_completed_total" in m
    assert "b200ds_engine_decode_tokens_total" in m and 'b200ds_switch{name="moe_fused"}' in m
    assert "b200ds_kv_pages_free" in m and "b200ds_prefix_cache_hit_ratio" in m and "b200ds_preemptions_total" in m
    assert "b200ds_cp_queue 0" in m


def test_stop_strings(client):
    """A stop string ends the completion (text cut before it, finish_reason
    stop) in both the plain and the streamed response."""
    from b200ds.engine.tokenizer import ByteTokenizer
    tok = ByteTokenizer()
    base = client.post("/v1/completions", json={"prompt": [9, 10, 11], "max_tokens": 8, "temperature": 0}).json()
    ids = base["choices"][0]["token_ids"]
    text = tok.decode(ids)
    stop = tok.decode(ids[3:5])
    k = text.find(stop)
    assert k >= 0
    r = client.post("/v1/completions", json={"prompt": [9, 10, 11], "max_tokens": 8, "temperature": 0,
                                             "stop": stop}).json()
    assert r["choices"][0]["finish_reason"] == "stop" and r["choices"][0]["text"] == text[:k]
    with client.stream("POST", "/v1/completions", json={"prompt": [9, 10, 11], "max_tokens": 8, "temperature": 0,
                                                        "stop": [stop], "stream": True}) as s:
        events = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: ") and l != "data: [DONE]"]
    assert "".join(e["choices"][0]["text"] for e in events) == text[:k]
    assert events[-1]["choices"][0]["finish_reason"] == "stop"


def test_n_choices(client):
    r = client.post("/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 4, "temperature": 0.9,
                                             "seed": 11, "n": 3}).json()
    assert [c["index"] for c in r["choices"]] == [0, 1, 2]
    assert all(len(c["token_ids"]) == 4 for c in r["choices"]) and r["usage"]["completion_tokens"] == 12
    again = client.post("/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 4, "temperature": 0.9,
                                                 "seed": 11, "n": 3}).json()
    assert [c["token_ids"] for c in again["choices"]] == [c["token_ids"] for c in r["choices"]]


def test_logprobs_fields(client):
    """OpenAI log-probability fields: completions (`logprobs: n` -> tokens /
    token_logprobs / top_logprobs / text_offset), chat (`logprobs: true`,
    `top_logprobs` -> content entries), and per chunk when streaming."""
    r = client.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4, "temperature": 0,
                                             "logprobs": 2}).json()
    c = r["choices"][0]
    lp = c["logprobs"]
    assert len(lp["tokens"]) == len(lp["token_logprobs"]) == len(lp["top_logprobs"]) == 4
    assert all(v <= 0 for v in lp["token_logprobs"]) and all(len(t) <= 2 for t in lp["top_logprobs"])
    assert lp["text_offset"][0] == 0
    ch = client.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3,
                                                   "temperature": 0, "logprobs": True, "top_logprobs": 2}).json()
    content = ch["choices"][0]["logprobs"]["content"]
    assert len(content) == 3 and all(len(e["top_logprobs"]) == 2 for e in content)
    assert content[0]["top_logprobs"][0]["token_id"] == content[0]["token_id"]     # greedy
    plain = client.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4, "temperature": 0}).json()
    assert "logprobs" not in plain["choices"][0] and plain["choices"][0]["token_ids"] == c["token_ids"]
    with client.stream("POST", "/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4, "temperature": 0,
                                                        "logprobs": 1, "stream": True}) as s:
        events = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: ") and l != "data: [DONE]"]
    streamed = sum((e["choices"][0].get("logprobs", {}).get("token_logprobs", []) for e in events), [])
    assert len(streamed) == 4 and abs(streamed[0] - lp["token_logprobs"][0]) < 1e-5
    bad = client.post("/v1/completions", json={"prompt": [5], "max_tokens": 1, "logprobs": 50})
    assert bad.status_code == 400


def _fresh_client(**kw):
    from fastapi.testclient import TestClient
    from b200ds import EngineConfig, load_engine
    from b200ds.engine.tokenizer import ByteTokenizer
    from b200ds.server.openai import EngineWorker, create_app
    eng = load_engine("tiny", ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu")
    tok = ByteTokenizer()
    eng.tokenizer = tok
    worker = EngineWorker(eng, tok, **kw)
    return eng, worker, TestClient(create_app(worker, "tiny"))


def test_engine_failure_fails_requests_and_health():
    """A step that raises fails every pending request (500, or an error event
    when streaming) instead of leaving it waiting; /health turns 503 and new
    requests are refused."""
    eng, worker, client = _fresh_client()
    calls = {"n": 0}
    orig = eng.step

    def flaky():
        calls["n"] += 1
        if calls["n"] == 3:
            raise RuntimeError("injected step failure")
        return orig()
    eng.step = flaky
    worker.start()
    with client as c:
        assert c.get("/health").json() == {"status": "ok"}
        r = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 8, "temperature": 0})
        assert r.status_code == 500 and "injected step failure" in r.json()["detail"]
        h = c.get("/health")
        assert h.status_code == 503 and "injected" in h.json()["error"]
        assert c.post("/v1/completions", json={"prompt": [1], "max_tokens": 2}).status_code == 503
    worker.stop()


def test_watchdog_marks_a_long_step_stalled():
    """A step running past the watchdog limit turns /health 503 ("stalled")
    while it runs (stacks dumped once); the server recovers when it ends."""
    import threading
    import time
    from b200ds.utils.watchdog import Watchdog
    fired = []
    wd = Watchdog(0.1, on_expire=fired.append, dump=False)
    with wd.guard():
        time.sleep(0.4)
        assert wd.stalled
    assert not wd.stalled and len(fired) == 1 and fired[0] >= 0.1
    with wd.guard():
        pass
    time.sleep(0.2)
    assert len(fired) == 1
    wd.stop()

    eng, worker, client = _fresh_client(watchdog_s=0.2)
    worker.watchdog.dump = False
    gate = threading.Event()
    orig = eng.step

    def slow():
        gate.wait(5)
        return orig()
    eng.step = slow
    worker.start()
    with client as c:
        res = {}
        t = threading.Thread(target=lambda: res.update(r=c.post("/v1/completions", json={
            "prompt": [4, 5], "max_tokens": 2, "temperature": 0})))
        t.start()
        deadline = time.time() + 5
        while c.get("/health").status_code == 200 and time.time() < deadline:
            time.sleep(0.05)
        h = c.get("/health")
        assert h.status_code == 503 and h.json()["status"] == "stalled"
        gate.set()
        t.join(10)
        assert res["r"].status_code == 200
        assert c.get("/health").status_code == 200
    worker.stop()


def test_engine_failure_while_streaming():
    eng, worker, client = _fresh_client()
    calls = {"n": 0}
    orig = eng.step

    def flaky():
        calls["n"] += 1
        if calls["n"] == 3:
            raise RuntimeError("injected step failure")
        return orig()
    eng.step = flaky
    worker.start()
    with client as c:
        with c.stream("POST", "/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 8, "temperature": 0,
                                                       "stream": True}) as s:
            lines = [l for l in s.iter_lines() if l.startswith("data: ")]
        assert lines[-1] == "data: [DONE]"
        err = json.loads(lines[-2][6:])
        assert "injected step failure" in err["error"]["message"]
    worker.stop()


def test_penalty_parameters(client):
    ok = client.post("/v1/completions", json={"prompt": [5, 6, 7, 5, 6, 7], "max_tokens": 6, "temperature": 0,
                                              "presence_penalty": 1.5, "frequency_penalty": 0.5,
                                              "repetition_penalty": 1.3, "min_p": 0.05, "min_tokens": 2})
    assert ok.status_code == 200 and len(ok.json()["choices"][0]["token_ids"]) == 6
    for bad in ({"presence_penalty": 3}, {"repetition_penalty": 0}, {"min_p": 1.5}, {"min_tokens": -1}):
        r = client.post("/v1/completions", json=dict({"prompt": [1], "max_tokens": 1}, **bad))
        assert r.status_code == 400, bad


def test_usage_chunk_max_completion_tokens_and_tokenize(client):
    with client.stream("POST", "/v1/chat/completions", json={
            "messages": [{"role": "user", "content": "hi"}], "max_completion_tokens": 3, "temperature": 0,
            "stream": True, "stream_options": {"include_usage": True}}) as s:
        lines = [l for l in s.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    last = json.loads(lines[-2][6:])
    assert last["choices"] == [] and last["usage"]["completion_tokens"] == 3
    t = client.post("/tokenize", json={"prompt": "hello"}).json()
    assert t["count"] == len(t["tokens"]) > 0
    assert client.post("/detokenize", json={"tokens": t["tokens"]}).json()["prompt"] == "hello"
    chat = client.post("/tokenize", json={"messages": [{"role": "user", "content": "hello"}]}).json()
    assert chat["count"] > t["count"]                     # the chat template adds its markers
    assert client.post("/detokenize", json={"tokens": "x"}).status_code == 400


def test_echo_prompt_logprobs_and_zero_max_tokens(client):
    """Completions with echo + logprobs score the prompt (the lm-eval-harness
    loglikelihood request): the prompt's tokens come first in the logprobs,
    the first with no value; max_tokens 0 returns the prompt only."""
    r = client.post("/v1/completions", json={"prompt": [5, 6, 7, 8, 9], "max_tokens": 0, "echo": True,
                                             "logprobs": 1, "temperature": 0}).json()
    c = r["choices"][0]
    lp = c["logprobs"]
    assert c["token_ids"] == [] and len(lp["tokens"]) == 5 and lp["token_logprobs"][0] is None
    assert all(v is not None and v <= 0 for v in lp["token_logprobs"][1:]) and lp["top_logprobs"][0] is None
    assert r["usage"]["completion_tokens"] == 0
    both = client.post("/v1/completions", json={"prompt": [5, 6, 7, 8, 9], "max_tokens": 2, "echo": True,
                                                "logprobs": 0, "temperature": 0}).json()["choices"][0]
    assert len(both["logprobs"]["tokens"]) == 7
    assert both["logprobs"]["token_logprobs"][1:5] == pytest.approx(lp["token_logprobs"][1:5], abs=1e-5)
    with client.stream("POST", "/v1/completions", json={"prompt": "ab", "max_tokens": 2, "echo": True,
                                                        "temperature": 0, "stream": True}) as s:
        events = [json.loads(l[6:]) for l in s.iter_lines() if l.startswith("data: ") and l != "data: [DONE]"]
    assert events[0]["choices"][0]["text"] == "ab"
    assert client.post("/v1/completions", json={"prompt": [1], "max_tokens": -1}).status_code == 400


def test_invalid_requests_are_refused_alone(client):
    """Requests the engine cannot serve get a 400 (empty prompt, ids outside
    the vocabulary, context beyond max_model_len) and the server keeps
    serving; submitted past the HTTP checks, the worker refuses just that
    one."""
    for body in ({"prompt": [], "max_tokens": 2}, {"prompt": [5, 99999], "max_tokens": 2},
                 {"prompt": [5, 6], "max_tokens": 10 ** 6}):
        r = client.post("/v1/completions", json=body)
        assert r.status_code == 400, (body, r.text)
    assert client.get("/health").status_code == 200
    ok = client.post("/v1/completions", json={"prompt": [5, 6], "max_tokens": 3, "temperature": 0})
    assert ok.status_code == 200 and len(ok.json()["choices"][0]["token_ids"]) == 3


def test_worker_refuses_a_bad_request_without_failing():
    import time
    from b200ds.engine.request import SamplingParams
    eng, worker, _ = _fresh_client()

    class Loop:
        def __init__(self):
            self.items = []

        def call_soon_threadsafe(self, fn, item):
            fn(item)

        def put_nowait(self, item):
            self.items.append(item)
    worker.start()
    bad, good = Loop(), Loop()
    worker.submit([], SamplingParams(max_tokens=2), bad, bad)
    worker.submit([4, 5, 6], SamplingParams(max_tokens=2), good, good)
    t0 = time.time()
    while not any(ev[0] == "done" for ev in good.items) and time.time() - t0 < 30:
        time.sleep(0.01)
    worker.stop()
    assert bad.items and bad.items[0][0] == "error" and "empty" in bad.items[0][1]
    assert worker.healthy() and any(ev[0] == "done" for ev in good.items)


def test_guided_fields(client):
    r = client.post("/v1/completions", json={"prompt": "answer:", "max_tokens": 8, "temperature": 0,
                                             "guided_choice": ["left", "right"]}).json()
    assert r["choices"][0]["text"] in ("left", "right")
    r = client.post("/v1/completions", json={"prompt": "id:", "max_tokens": 8, "temperature": 0.7, "seed": 2,
                                             "regex": "[0-9]{4}"}).json()
    t = r["choices"][0]["text"]
    assert len(t) == 4 and t.isdigit()
    assert client.post("/v1/completions", json={"prompt": "x", "guided_regex": "("}).status_code == 400


def test_response_format_json_schema(client):
    schema = {"type": "object", "properties": {"k": {"type": "integer"}, "v": {"enum": ["x", "y"]}}}
    r = client.post("/v1/chat/completions", json={
        "messages": [{"role": "user", "content": "json"}], "max_tokens": 40, "temperature": 0,
        "response_format": {"type": "json_schema", "json_schema": {"name": "t", "schema": schema}}}).json()
    d = json.loads(r["choices"][0]["message"]["content"])
    assert list(d) == ["k", "v"] and isinstance(d["k"], int) and d["v"] in ("x", "y")
    bad = client.post("/v1/completions", json={"prompt": "x", "guided_json": {"type": "tuple"}})
    assert bad.status_code == 400


def test_update_weights_from_disk(tmp_path):
    """POST /update_weights_from_disk loads a checkpoint of the same
    architecture in place; later completions follow the new weights."""
    from b200ds import EngineConfig, load_engine
    from b200ds.config import tiny_config
    from b200ds.models.loader import save_checkpoint_fp8
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    save_checkpoint_fp8(init_weights(cfg, 5), str(tmp_path), cfg)
    want = load_engine(str(tmp_path), ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu").generate(
        [[7, 8, 9]], __import__("b200ds").SamplingParams(max_tokens=4))[0].token_ids
    eng, worker, client = _fresh_client()
    worker.start()
    with client as c:
        before = c.post("/v1/completions", json={"prompt": [7, 8, 9], "max_tokens": 4, "temperature": 0}).json()
        r = c.post("/update_weights_from_disk", json={"model_path": str(tmp_path)})
        assert r.status_code == 200 and r.json()["success"] and r.json()["bytes"] > 0
        after = c.post("/v1/completions", json={"prompt": [7, 8, 9], "max_tokens": 4, "temperature": 0}).json()
        assert after["choices"][0]["token_ids"] == want != before["choices"][0]["token_ids"]
        bad = c.post("/update_weights_from_disk", json={"model_path": str(tmp_path / "missing")})
        assert bad.status_code == 400 and c.get("/health").status_code == 200
    worker.stop()


def test_flush_cache_endpoint(client):
    client.post("/v1/completions", json={"prompt": list(range(3, 40)), "max_tokens": 2, "temperature": 0})
    r = client.post("/flush_cache")
    assert r.status_code == 200 and r.json()["success"] and r.json()["pages"] > 0


def test_logit_bias_field(client):
    r = client.post("/v1/completions", json={"prompt": [5, 6], "max_tokens": 3, "temperature": 0,
                                             "logit_bias": {"77": 100}}).json()
    assert r["choices"][0]["token_ids"] == [77, 77, 77]
    assert client.post("/v1/completions", json={"prompt": [5], "logit_bias": {"5": 1000}}).status_code == 400


def test_stream_n_choices(client):
    """n > 1 with stream: the choices' chunks interleave, each tagged with its
    index, each choice finishes, one [DONE] (and one usage chunk) closes."""
    with client.stream("POST", "/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 4, "temperature": 0.9,
                                                        "seed": 11, "n": 3, "stream": True,
                                                        "stream_options": {"include_usage": True}}) as s:
        lines = [l for l in s.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]" and lines.count("data: [DONE]") == 1
    evs = [json.loads(l[6:]) for l in lines[:-1]]
    usage = evs[-1]
    assert usage["choices"] == [] and usage["usage"]["completion_tokens"] == 12
    toks = {0: [], 1: [], 2: []}
    fins = {}
    for e in evs[:-1]:
        c = e["choices"][0]
        toks[c["index"]].extend(c.get("token_ids") or [])
        if c["finish_reason"]:
            fins[c["index"]] = c["finish_reason"]
    assert all(len(t) == 4 for t in toks.values()) and set(fins) == {0, 1, 2}
    plain = client.post("/v1/completions", json={"prompt": [3, 4, 5], "max_tokens": 4, "temperature": 0.9,
                                                 "seed": 11, "n": 3}).json()
    assert [c["token_ids"] for c in plain["choices"]] == [toks[i] for i in range(3)]


def test_sglang_native_endpoints(client):
    """SGLang's /generate (single, batch, stream) and the info endpoints."""
    r = client.post("/generate", json={"input_ids": [5, 6, 7], "sampling_params": {"max_new_tokens": 4,
                                                                                  "temperature": 0}}).json()
    assert len(r["output_ids"]) == 4 and r["meta_info"]["completion_tokens"] == 4
    assert r["meta_info"]["finish_reason"]["type"] == "length"
    same = client.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4, "temperature": 0}).json()
    assert same["choices"][0]["token_ids"] == r["output_ids"]
    b = client.post("/generate", json={"text": ["hi", "there"], "sampling_params": {"max_new_tokens": 2,
                                                                                    "temperature": 0}}).json()
    assert isinstance(b, list) and len(b) == 2 and all(len(x["output_ids"]) == 2 for x in b)
    g = client.post("/generate", json={"text": "n:", "sampling_params": {"max_new_tokens": 6, "temperature": 0,
                                                                         "regex": "[0-9]{3}"}}).json()
    assert g["text"].isdigit() and len(g["text"]) == 3
    with client.stream("POST", "/generate", json={"input_ids": [5, 6, 7], "stream": True,
                                                  "sampling_params": {"max_new_tokens": 3, "temperature": 0}}) as s:
        lines = [l for l in s.iter_lines() if l.startswith("data: ")]
    assert lines[-1] == "data: [DONE]" and json.loads(lines[-2][6:])["output_ids"] == r["output_ids"][:3]
    lp = client.post("/generate", json={"input_ids": [5, 6, 7], "return_logprob": True, "top_logprobs_num": 2,
                                        "sampling_params": {"max_new_tokens": 3, "temperature": 0}}).json()["meta_info"]
    assert [x[1] for x in lp["output_token_logprobs"]] == r["output_ids"][:3]
    assert all(x[0] <= 0 for x in lp["output_token_logprobs"]) and len(lp["output_top_logprobs"][0]) == 2
    assert client.get("/get_model_info").json()["is_generation"]
    info = client.get("/get_server_info").json()
    assert info["engine_config"]["page_size"] == 8 and info["model_config"]["hidden_size"] == 256
    assert client.post("/generate", json={"input_ids": [], "sampling_params": {}}).status_code == 400


def test_api_key():
    from fastapi.testclient import TestClient
    from b200ds import EngineConfig, load_engine
    from b200ds.engine.tokenizer import ByteTokenizer
    from b200ds.server.openai import EngineWorker, create_app
    eng = load_engine("tiny", ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu")
    worker = EngineWorker(eng, ByteTokenizer()).start()
    with TestClient(create_app(worker, "tiny", api_key="s3cret")) as c:
        body = {"prompt": [5, 6], "max_tokens": 2, "temperature": 0}
        assert c.post("/v1/completions", json=body).status_code == 401
        assert c.post("/v1/completions", json=body, headers={"Authorization": "Bearer nope"}).status_code == 401
        ok = c.post("/v1/completions", json=body, headers={"Authorization": "Bearer s3cret"})
        assert ok.status_code == 200 and c.get("/health").status_code == 200
    worker.stop()
