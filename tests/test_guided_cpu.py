"""Guided decoding: outputs constrained to a regular expression or a list of
choices, greedy and sampled, with and without an end-of-sequence id."""
import pytest
import regex
import torch

from b200ds.engine.request import SamplingParams


def _engine(eos=None):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.tokenizer import ByteTokenizer
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False)
    tok = ByteTokenizer()
    return Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu"), ecfg, eos_token_id=eos,
                  tokenizer=tok), tok


def test_guided_choice_and_regex():
    eng, tok = _engine()
    prompt = tok.encode("pick:")
    o = eng.generate([prompt], SamplingParams(max_tokens=10, guided_choice=["yes", "no", "maybe"]))[0]
    assert tok.decode(o.token_ids) in ("yes", "no", "maybe") and o.finish_reason == "stop"
    pat = r"[0-9]{3}-[a-z]{2}"
    for seed in range(3):
        o = eng.generate([prompt], SamplingParams(max_tokens=12, temperature=1.0, seed=seed, guided_regex=pat))[0]
        assert regex.fullmatch(pat, tok.decode(o.token_ids)) and o.finish_reason == "stop"
    # an open-ended pattern runs to max_tokens and stays a prefix of a match
    o = eng.generate([prompt], SamplingParams(max_tokens=6, guided_regex=r"(ab)+"))[0]
    assert o.finish_reason == "length" and tok.decode(o.token_ids) == "ababab"


def test_guided_with_eos_and_validation():
    eng, tok = _engine(eos=1)
    o = eng.generate([tok.encode("q")], SamplingParams(max_tokens=10, guided_regex=r"x{2,4}"))[0]
    text = tok.decode(o.token_ids)
    assert regex.fullmatch(r"x{2,4}", text) and o.finish_reason == "stop"
    with pytest.raises(ValueError):
        eng.add_request([5], SamplingParams(guided_regex="(unclosed"))
    bare, _ = _engine()
    bare.tokenizer = None
    with pytest.raises(ValueError):
        bare.add_request([5], SamplingParams(guided_choice=["a"]))


def test_guided_json_schema_and_object():
    import json
    from b200ds.engine.guided import schema_to_regex
    eng, tok = _engine()
    schema = {"type": "object", "properties": {"name": {"type": "string", "maxLength": 4},
                                               "n": {"type": "integer"}, "ok": {"type": "boolean"},
                                               "tags": {"type": "array", "items": {"enum": ["a", "b"]},
                                                        "maxItems": 2}}}
    for seed in range(3):
        o = eng.generate([tok.encode("json:")], SamplingParams(max_tokens=80, temperature=0.9, seed=seed,
                                                               guided_json=schema))[0]
        d = json.loads(tok.decode(o.token_ids))
        assert list(d) == ["name", "n", "ok", "tags"] and len(d["name"]) <= 4 and isinstance(d["n"], int)
        assert isinstance(d["ok"], bool) and set(d["tags"]) <= {"a", "b"} and len(d["tags"]) <= 2
    o = eng.generate([tok.encode("obj:")], SamplingParams(max_tokens=60, guided_json="object"))[0]
    text = tok.decode(o.token_ids)
    assert text.startswith("{")
    if o.finish_reason == "stop":
        assert isinstance(json.loads(text), dict)
    with pytest.raises(ValueError):
        schema_to_regex({"type": "object", "properties": {"x": {"$ref": "#/defs/y"}}})
