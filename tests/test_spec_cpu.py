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


def test_verify_batch_layout_matches_unpadded():
    """The fixed-shape verify layout (1 + spec_k rows per request, padding on
    the scratch slot, an absent request) gives the real rows the logits of
    the plain ragged batch."""
    import torch
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.cuda_graph import build_verify_batch
    from b200ds.models.batch import build_batch
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    m = build_model_from(cfg, EngineConfig(page_size=8, cuda_graphs=False), init_weights(cfg, 0), device="cpu")
    m.allocate_kv(16)
    g = torch.Generator().manual_seed(2)
    pa, pb = torch.randint(0, 1000, (13,), generator=g).tolist(), torch.randint(0, 1000, (9,), generator=g).tolist()
    pages_a, pages_b = [1, 2, 3], [4, 5]
    m.forward(build_batch([{"tokens": pa, "start": 0, "pages": pages_a},
                           {"tokens": pb, "start": 0, "pages": pages_b}], 8))
    seqs = [{"tokens": [5, 6, 7], "start": 13, "pages": pages_a}, {"tokens": [8], "start": 9, "pages": pages_b}]
    fb = build_batch(seqs, 8)
    fb.last_idx = torch.arange(fb.num_tokens)
    want = m.forward(fb)
    vb = build_verify_batch(seqs, 4, 3, 8, 4)
    got = m.forward(vb)
    assert got.shape[0] == 15
    assert torch.allclose(got[[0, 1, 2, 5]], want, atol=1e-5)
