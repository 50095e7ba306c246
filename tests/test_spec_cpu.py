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


def test_mtp_speculative_decoding_matches_greedy():
    """MTP drafts (DeepSeek-V3's next-token module as the draft, chained
    for spec_k tokens) verified greedily: the same tokens as plain greedy
    decoding, under chunked prefill; drafts are proposed every step."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    import torch
    cfg = tiny_config(num_nextn_predict_layers=1)
    sd = init_weights(cfg, 0)
    g = torch.Generator().manual_seed(3)
    prompts = torch.randint(0, cfg.vocab_size, (3, 13), generator=g).tolist()

    def run(**kw):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, max_prefill_tokens=7, **kw)
        eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
        outs = eng.generate(prompts, SamplingParams(max_tokens=10))
        return [o.token_ids for o in outs], eng.stats
    base, _ = run()
    spec, stats = run(spec_mtp=True, spec_k=3)
    assert spec == base
    assert stats.get("spec_proposed", 0) > 0


def test_mtp_first_draft_matches_one_shot_computation():
    """The first draft after a chunked prefill equals the MTP module run in
    one pass over z_j = eh_proj[rms(Emb(x_j)); rms(h_{j-1})], j = 1..P
    (x_P = the sampled token), at MTP positions 0..P-1."""
    import torch
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.batch import build_batch
    from b200ds.models.reference import init_weights
    cfg = tiny_config(num_nextn_predict_layers=1)
    sd = init_weights(cfg, 0)
    prompt = torch.randint(0, cfg.vocab_size, (11,), generator=torch.Generator().manual_seed(5)).tolist()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, max_prefill_tokens=4,
                        spec_mtp=True, spec_k=1)
    eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
    r = eng.add_request(prompt, SamplingParams(max_tokens=4))
    while r.t_first is None:
        eng.step()
    x_new, draft = r.output[0], r.mtp_drafts[0]
    # one-shot: main model hiddens over the whole prompt, then the MTP block
    ref_eng = Engine(build_model_from(cfg, EngineConfig(page_size=8, cuda_graphs=False,
                                                        enable_prefix_cache=False), sd, device="cpu"),
                     EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False))
    m = ref_eng.model
    pages = ref_eng.pool.alloc(2)
    m.forward(build_batch([{"tokens": prompt, "start": 0, "pages": pages}], 8))
    H = m.last_residual
    mtp = m.mtp
    mtp.allocate_kv(16)
    toks = prompt[1:] + [x_new]
    fb = build_batch([{"tokens": toks, "start": 0, "pages": pages}], 8)
    logits, _ = mtp.forward(fb, H)
    assert int(logits.argmax(-1)[0]) == draft


def test_extend_batch_layout_matches_ragged():
    """Fixed-shape prefill layout (token bucket with padding on a spare
    sequence row, scratch slot, page 0) gives the ragged batch's last-token
    logits."""
    import torch
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.cuda_graph import build_extend_batch
    from b200ds.models.batch import build_batch
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    m = build_model_from(cfg, EngineConfig(page_size=8, cuda_graphs=False), init_weights(cfg, 0), device="cpu")
    m.allocate_kv(16)
    g = torch.Generator().manual_seed(4)
    a, b = torch.randint(0, 1000, (11,), generator=g).tolist(), torch.randint(0, 1000, (6,), generator=g).tolist()
    seqs = [{"tokens": a, "start": 0, "pages": [1, 2]}, {"tokens": b, "start": 0, "pages": [3]}]
    want = m.forward(build_batch(seqs, 8))
    got = m.forward(build_extend_batch(seqs, 32, 4, 8, 4))
    assert got.shape[0] == 4 and torch.allclose(got[:2], want, atol=1e-5)


def test_speculative_sampling_preserves_distribution():
    """Speculative sampling with a deterministic draft: the first verified
    token follows the sampler's distribution p exactly (accept d with p(d),
    else draw from p without d), and the token after an accepted draft
    follows the next row's distribution."""
    import types
    import torch
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import Request, SamplingParams
    from b200ds.ops.ref import sampling_probs
    g = torch.Generator().manual_seed(0)
    V = 8
    logits = torch.randn(3, V, generator=g) * 2
    params = SamplingParams(max_tokens=10, temperature=0.8, top_k=5, top_p=0.9, seed=1)
    r = Request(0, [1, 2, 3], params)
    eng = types.SimpleNamespace(stats={})
    draft = [int(sampling_probs(logits[0], 0.8, 0.9, 5).argmax()), 4]
    st = types.SimpleNamespace(reqs=[r])
    n = 20000
    first = torch.zeros(V)
    second = torch.zeros(V)
    for _ in range(n):
        toks = Engine._accept_sampled(eng, st, [draft], logits, [0])[0]
        first[toks[0]] += 1
        if toks[0] == draft[0]:
            second[toks[1]] += 1
    p0 = sampling_probs(logits[0], 0.8, 0.9, 5)
    p1 = sampling_probs(logits[1], 0.8, 0.9, 5)
    tv0 = 0.5 * (first / n - p0 / p0.sum()).abs().sum().item()
    tv1 = 0.5 * (second / second.sum() - p1 / p1.sum()).abs().sum().item()
    assert tv0 < 0.02 and tv1 < 0.03, (tv0, tv1)
    assert eng.stats["spec_proposed"] == 2 * n


def test_logprobs_under_speculative_decoding():
    """Log-probabilities of tokens accepted from a draft come from the verify
    forward's row for that position: the same values as plain decoding."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    sd = init_weights(cfg, 0)
    g = torch.Generator().manual_seed(2)
    base = torch.randint(0, cfg.vocab_size, (6,), generator=g).tolist()
    prompts = [base * 4]

    def run(spec):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, spec_ngram=spec, spec_k=4)
        eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
        o = eng.generate(prompts, SamplingParams(max_tokens=16, logprobs=2))[0]
        return o, eng.stats
    plain, _ = run(0)
    spec, stats = run(3)
    assert stats.get("spec_accepted", 0) > 0
    assert spec.token_ids == plain.token_ids and len(spec.logprobs) == len(plain.logprobs)
    for a, b in zip(spec.logprobs, plain.logprobs):
        assert a[0] == b[0] and abs(a[1] - b[1]) < 1e-3 and [t for t, _ in a[2]] == [t for t, _ in b[2]]


def test_mtp_speculative_sampling():
    """MTP drafts with temperature > 0 go through speculative sampling: with
    top_k 1 the sampling distribution is the argmax, so the tokens equal
    greedy decoding; with a wider distribution drafts are still proposed
    and accepted and the outputs are reproducible per seed."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    cfg = tiny_config(num_nextn_predict_layers=1)
    sd = init_weights(cfg, 0)
    g = torch.Generator().manual_seed(3)
    prompts = torch.randint(0, cfg.vocab_size, (2, 13), generator=g).tolist()

    def run(sp, **kw):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, **kw)
        eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
        return [o.token_ids for o in eng.generate(prompts, sp)], eng.stats
    greedy, _ = run(SamplingParams(max_tokens=10))
    top1, st = run(SamplingParams(max_tokens=10, temperature=0.8, top_k=1, seed=1), spec_mtp=True, spec_k=3)
    assert top1 == greedy and st.get("spec_proposed", 0) > 0
    a, st = run(SamplingParams(max_tokens=10, temperature=1.0, seed=7), spec_mtp=True, spec_k=3)
    b, _ = run(SamplingParams(max_tokens=10, temperature=1.0, seed=7), spec_mtp=True, spec_k=3)
    assert a == b and st.get("spec_proposed", 0) > 0 and all(len(t) == 10 for t in a)
