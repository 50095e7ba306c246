"""Speculative decoding (n-gram prompt-lookup drafts, greedy verification in
one forward with logits at every position): same tokens as plain decoding,
fewer steps when the drafts hit."""
import torch


def _run(spec: int):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, spec_ngram=spec, spec_k=4)
    m = build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu")
    eng = Engine(m, ecfg)
    g = torch.Generator().manual_seed(2)
    base = torch.randint(0, cfg.vocab_size, (6,), generator=g).tolist()
    prompts = [base * 4, torch.randint(0, cfg.vocab_size, (20,), generator=g).tolist()]
    outs = eng.generate(prompts, SamplingParams(max_tokens=24))
    return [o.token_ids for o in outs], eng.stats


def test_spec_decode_matches_plain():
    plain, s0 = _run(0)
    spec, s1 = _run(3)
    assert spec == plain
    assert s1.get("spec_proposed", 0) > 0
    assert s1["steps"] <= s0["steps"]
