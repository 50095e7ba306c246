"""Chat output parsers: DeepSeek-R1 reasoning split and DeepSeek-V3 tool
calls; reasoning_content over HTTP."""
import json

from b200ds.server.parsers import CALL_BEGIN, CALL_END, CALLS_BEGIN, CALLS_END, SEP, parse_tool_calls, \
    split_reasoning


def test_split_reasoning():
    assert split_reasoning("<think>a b</think>\n\nanswer") == ("a b", "answer")
    assert split_reasoning("plan</think>ok") == ("plan", "ok")          # template wrote <think>
    assert split_reasoning("no markers") == (None, "no markers")
    assert split_reasoning("<think>still going") == ("still going", "")


def test_parse_tool_calls():
    text = ("Let me check." + CALLS_BEGIN
            + CALL_BEGIN + "function" + SEP + "get_weather\n```json\n{\"city\": \"Paris\"}\n```" + CALL_END
            + CALL_BEGIN + "function" + SEP + "now\n```json\n{}\n```" + CALL_END + CALLS_END)
    content, calls = parse_tool_calls(text)
    assert content == "Let me check." and [c["function"]["name"] for c in calls] == ["get_weather", "now"]
    assert json.loads(calls[0]["function"]["arguments"]) == {"city": "Paris"} and calls[0]["type"] == "function"
    assert parse_tool_calls("plain") == ("plain", [])


def test_reasoning_content_over_http():
    from fastapi.testclient import TestClient
    from b200ds import EngineConfig, load_engine
    from b200ds.engine.tokenizer import ByteTokenizer
    from b200ds.server.openai import EngineWorker, create_app
    eng = load_engine("tiny", ecfg=EngineConfig(page_size=8, cuda_graphs=False), device="cpu")
    eng.tokenizer = ByteTokenizer()
    worker = EngineWorker(eng, eng.tokenizer).start()
    with TestClient(create_app(worker, "tiny", reasoning=True)) as c:
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "q"}], "max_tokens": 40,
                                                 "temperature": 0, "guided_regex": "<think>[a-z]{3}</think>ok"})
        m = r.json()["choices"][0]["message"]
        assert len(m["reasoning_content"]) == 3 and m["content"] == "ok"
        with c.stream("POST", "/v1/chat/completions", json={
                "messages": [{"role": "user", "content": "q"}], "max_tokens": 40, "temperature": 0,
                "guided_regex": "<think>[a-z]{3}</think>ok", "stream": True}) as st:
            evs = [json.loads(l[6:]) for l in st.iter_lines() if l.startswith("data: ") and l != "data: [DONE]"]
        deltas = [e["choices"][0]["delta"] for e in evs]
        assert "".join(d.get("reasoning_content", "") for d in deltas) == m["reasoning_content"]
        assert "".join(d.get("content", "") for d in deltas) == "ok"
        r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "q"}], "max_tokens": 4,
                                                 "temperature": 0, "tools": [{"type": "function", "function": {
                                                     "name": "f", "parameters": {"type": "object"}}}]})
        assert r.status_code == 200 and r.json()["choices"][0]["message"]["role"] == "assistant"
    worker.stop()
