"""DeepSeek-V4 family on CPU: mHC coefficient properties, the E5 prune rule,
Engram hashing through the per-slot token cache, the engine's V4 model
against the fp32 oracle (greedy tokens, logits), and TP=2 over gloo."""
import pytest
import torch

from mp_util import run_ranks


def test_sinkhorn_doubly_stochastic_and_coeff_ranges():
    from b200ds.ops import ref
    g = torch.Generator().manual_seed(0)
    raw = torch.randn(6, 24, generator=g)
    ss = torch.rand(6, generator=g) * 1024 + 512          # rms ~ 1
    pre, post, comb = ref.hc_coeffs(raw, ss, torch.ones(3), torch.zeros(24), 4, 1024, 20, 1e-6)
    # ends on a column pass: columns exact, rows converged
    assert torch.allclose(comb.sum(-1), torch.ones(6, 4), atol=1e-3)
    assert torch.allclose(comb.sum(-2), torch.ones(6, 4), atol=1e-5)
    assert (pre > 0).all() and (pre <= 1 + 1e-5).all() and (post >= 0).all() and (post <= 2).all()


def test_e5_prune_rule():
    from b200ds.ops import ref
    # rows: (0: heavy 5 / light 7), (1: heavy 5 / light 6 shared with row 2), (2: 6 light / 4 heavy)
    ids = torch.tensor([[5, 7], [5, 6], [4, 6]], dtype=torch.int32)
    w = torch.tensor([[0.8, 0.2], [0.7, 0.3], [0.9, 0.1]])
    w2, ids2 = ref.e5_prune(ids, w, budget=0.4, max_count=1)
    # 7: picked once, its run 0.2 <= 0.4 -> dropped; 6: picked twice -> not eligible at max_count 1
    assert ids2.tolist() == [[5, -1], [5, 6], [4, 6]] and float(w2[0, 1]) == 0.0
    w3, ids3 = ref.e5_prune(ids, w, budget=0.4, max_count=2)
    # max_count 2: 6 is eligible in both rows and each pick is within budget -> dropped
    assert ids3.tolist() == [[5, -1], [5, -1], [4, -1]]
    # weights of kept picks are not renormalised
    assert float(w3[0, 0]) == float(w[0, 0])


def test_engram_hash_matches_full_context():
    """Hash ids computed chunk by chunk through the per-slot token cache
    equal the ids from the whole sequence."""
    from b200ds import ops
    from b200ds.config import tiny_v4_config
    from b200ds.models.batch import build_batch
    from b200ds.models.reference_v4 import engram_context
    from b200ds.ops import ref
    cfg = tiny_v4_config()
    toks = list(range(3, 40, 2))
    page = 8
    pages = [5, 2, 9]
    tok_cache = torch.full((16 * page,), -1, dtype=torch.int32)
    mults = torch.tensor([v - (1 << 64) if v >= (1 << 63) else v for v in ref.engram_multipliers(cfg.engram_heads)])
    got = []
    for st, en in ((0, 7), (7, 12), (12, 13), (13, len(toks))):
        fb = build_batch([{"tokens": toks[st:en], "start": st, "pages": pages}], page)
        got.append(ops.engram_ids(fb, tok_cache, cfg, mults, page))
    want = ref.engram_hash(engram_context(torch.tensor(toks), cfg.engram_max_ngram), cfg.engram_heads,
                           cfg.engram_rows, cfg.engram_max_ngram)
    assert torch.equal(torch.cat(got), want)


def _v4_engine(prefix_cache=False, chunk=64, tp=1, ps=None):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_v4_config
    from b200ds.engine.engine import Engine
    from b200ds.models.reference_v4 import init_weights_v4
    cfg = tiny_v4_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=prefix_cache, max_prefill_tokens=chunk,
                        tp_size=tp, ep_size=tp)
    kw = {"ps": ps} if ps is not None else {}
    return Engine(build_model_from(cfg, ecfg, init_weights_v4(cfg, 0), device="cpu", **kw), ecfg), cfg


def _prompts(cfg, n=3, s=11, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab_size, (n, s), generator=g)


def test_v4_engine_matches_oracle_greedy():
    """Paged MQA + sinks + inverse rope + grouped wo_a, mHC kernels' CPU
    references, sqrt-softplus routing with the E5 prune at decode, Engram
    through the token cache under chunked prefill: same greedy tokens and
    close logits as the fp32 oracle."""
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import ReferenceV4Model, init_weights_v4
    eng, cfg = _v4_engine(chunk=7)
    prompts = _prompts(cfg)
    outs = eng.generate(prompts.tolist(), SamplingParams(max_tokens=6))
    oracle = ReferenceV4Model(cfg, init_weights_v4(cfg, 0), 256)
    assert [o.token_ids for o in outs] == oracle.greedy(prompts, 6).tolist()


def test_v4_prefill_logits_match_oracle():
    from b200ds.models.batch import build_batch
    from b200ds.models.reference_v4 import ReferenceV4Model, init_weights_v4
    eng, cfg = _v4_engine()
    prompts = _prompts(cfg, 2, 13, seed=5)
    seqs = [{"tokens": prompts[b].tolist(), "start": 0, "pages": eng.pool.alloc(2)} for b in range(2)]
    logits = eng.model.forward(build_batch(seqs, 8))
    oracle = ReferenceV4Model(cfg, init_weights_v4(cfg, 0), 64)
    oracle.reset(2)
    want = oracle.forward(prompts, 0, decode=False)[:, -1]
    assert torch.allclose(logits, want, rtol=1e-4, atol=1e-4), (logits - want).abs().max()
    assert len(eng.model.aux) == len(cfg.aux_layers) and eng.model.aux[0].shape == (26, cfg.hidden_size)


def test_v4_prefix_cache_transparent():
    from b200ds.engine.request import SamplingParams
    eng, cfg = _v4_engine(prefix_cache=True)
    g = torch.Generator().manual_seed(4)
    shared = torch.randint(0, cfg.vocab_size, (24,), generator=g).tolist()
    p1, p2 = shared + [5, 6, 7], shared + [8, 9]
    first = eng.generate([p1], SamplingParams(max_tokens=5))[0].token_ids
    again = eng.generate([p2], SamplingParams(max_tokens=5))[0].token_ids
    ref_eng, _ = _v4_engine(prefix_cache=False)
    assert ref_eng.generate([p1], SamplingParams(max_tokens=5))[0].token_ids == first
    assert ref_eng.generate([p2], SamplingParams(max_tokens=5))[0].token_ids == again


def _tp_rank(rank, world):
    from b200ds.engine.request import SamplingParams
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo")
    eng, cfg = _v4_engine(tp=world, ps=ps)
    outs = eng.generate(_prompts(cfg).tolist(), SamplingParams(max_tokens=6))
    return [o.token_ids for o in outs]


def test_v4_tp2_gloo_matches_single():
    """Heads / output groups / FFN columns split, experts EP-split, Engram
    table rows sharded (zero rows summed by the all-reduce), vocab-parallel
    head: both ranks produce the single-process tokens."""
    from b200ds.engine.request import SamplingParams
    res = run_ranks(_tp_rank, 2)
    eng, cfg = _v4_engine()
    single = [o.token_ids for o in eng.generate(_prompts(cfg).tolist(), SamplingParams(max_tokens=6))]
    assert res[0] == single and res[1] == single


def test_v4_sparse_indexer_with_window_matches_oracle():
    """V4 with the lightning indexer + sliding window selection (top-6 by
    score, the last 3 positions always kept) over 20+ cached tokens.  8
    indexer heads: a key scores exactly 0 only when every head's ReLU is 0,
    and such ties (ordered differently by the oracle's batched top-k) then
    stay away from the selection boundary."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_v4_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import ReferenceV4Model, init_weights_v4
    cfg = tiny_v4_config(index_n_heads=8, index_head_dim=32, index_topk=6, index_swa=3)
    sd = init_weights_v4(cfg, 0)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, max_prefill_tokens=9)
    eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
    prompts = _prompts(cfg, 2, 21, seed=7)
    outs = eng.generate(prompts.tolist(), SamplingParams(max_tokens=5))
    oracle = ReferenceV4Model(cfg, sd, 128)
    assert [o.token_ids for o in outs] == oracle.greedy(prompts, 5).tolist()


def test_v4_compressed_sparse_attention_matches_oracle():
    """Compressed sparse attention (ratio 2 on layer 1, ratio 4 on layer 2):
    the compressor's gated block means, the indexer over compressed keys and
    attention over the window + top compressed blocks follow the fp32 oracle
    under chunked prefill (blocks completed across chunk boundaries) and
    decode (blocks completed by decode tokens), and the prefix cache reuses
    the compressed rows of cached pages."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_v4_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import ReferenceV4Model, init_weights_v4
    cfg = tiny_v4_config(index_n_heads=8, index_head_dim=32, index_topk=6, index_swa=4, compress_ratios=(0, 2, 4),
                         compress_topk=4)
    assert [cfg.compress_ratio(i) for i in range(3)] == [0, 2, 4]
    sd = init_weights_v4(cfg, 0)
    prompts = _prompts(cfg, 2, 27, seed=9)
    oracle = ReferenceV4Model(cfg, sd, 128)
    want = oracle.greedy(prompts, 7).tolist()
    for prefix in (False, True):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=prefix, max_prefill_tokens=11)
        eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
        outs = eng.generate(prompts.tolist(), SamplingParams(max_tokens=7))
        assert [o.token_ids for o in outs] == want
        if prefix:       # the same prompts again: full pages come from the prefix cache
            again = eng.generate(prompts.tolist(), SamplingParams(max_tokens=7))
            assert [o.token_ids for o in again] == want


def _dp_rank(rank, world):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_v4_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import init_weights_v4
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = tiny_v4_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, max_prefill_tokens=7,
                        tp_size=1, ep_size=world, dp_attention=True)
    eng = Engine(build_model_from(cfg, ecfg, init_weights_v4(cfg, 0), device="cpu", ps=ps), ecfg)
    mine = [i for i in range(3) if i % world == rank]
    prompts = _prompts(cfg, 3, 11, seed=6)
    maxt = [7, 4, 9]
    outs = eng.generate([prompts[i].tolist() for i in mine], [SamplingParams(max_tokens=maxt[i]) for i in mine])
    return mine, [o.token_ids for o in outs]


def test_v4_dp2_ep2_gloo_matches_single():
    """DP attention for the V4 family: each rank runs attention, mHC, Engram
    and the head for its own requests with replicated weights; routed
    experts are EP-split and the MoE exchanges the ranks' rows (uneven
    ranks: rank 1 idles with dummy rows at the end).  Each rank's tokens
    equal a single-process run of its own requests (the E5 prune acts on
    each rank's decode batch)."""
    from b200ds.engine.request import SamplingParams
    res = run_ranks(_dp_rank, 2)
    for mine, toks in res:
        eng, cfg = _v4_engine(chunk=7)
        prompts = _prompts(cfg, 3, 11, seed=6)
        maxt = [7, 4, 9]
        want = [o.token_ids for o in eng.generate([prompts[i].tolist() for i in mine],
                                                  [SamplingParams(max_tokens=maxt[i]) for i in mine])]
        assert toks == want, (mine, toks, want)


def test_v4_window_late_layers_prefill_tail_matches_oracle():
    """Window-only late layers (layers >= late_layer_start attend to the last
    late_window positions, no indexer) with the prefill tail: under chunked
    prefill those layers compute only the rows within reach of each prompt's
    end (whole early chunks skipped there), and the greedy tokens still
    equal the fp32 oracle's, which computes every row; the same holds with
    the tail off and with the prefix cache on (tail off automatically)."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_v4_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import ReferenceV4Model, init_weights_v4
    cfg = tiny_v4_config(late_layer_start=1, late_window=4, index_n_heads=4, index_head_dim=32, index_topk=5,
                         index_swa=2)
    sd = init_weights_v4(cfg, 0)
    prompts = _prompts(cfg, 2, 30, seed=9)
    want = ReferenceV4Model(cfg, sd, 256).greedy(prompts, 6).tolist()
    assert cfg.tail_rows_needed() == 7

    def run(**kw):
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, max_prefill_tokens=7, **kw)
        m = build_model_from(cfg, ecfg, sd, device="cpu")
        skipped = []
        orig = m.forward
        m.forward = lambda fb: (lambda out: skipped.append(m.tail_skipped) or out)(orig(fb))
        toks = [o.token_ids for o in Engine(m, ecfg).generate(prompts.tolist(), SamplingParams(max_tokens=6))]
        return toks, sum(skipped)
    toks, skipped = run(enable_prefix_cache=False)
    assert toks == want and skipped > 0
    toks, skipped = run(enable_prefix_cache=False, prefill_tail=False)
    assert toks == want and skipped == 0
    toks, skipped = run(enable_prefix_cache=True)
    assert toks == want and skipped == 0


def _v4_tbo_cfg(compressed):
    from b200ds.config import tiny_v4_config
    if compressed:
        return tiny_v4_config(index_n_heads=8, index_head_dim=32, index_topk=6, index_swa=4,
                              compress_ratios=(0, 2, 4), compress_topk=4)
    return tiny_v4_config()


def _tbo_rank(rank, world, compressed):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import init_weights_v4
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = _v4_tbo_cfg(compressed)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, max_prefill_tokens=9,
                        tp_size=1, ep_size=world, dp_attention=True, tbo=True, tbo_min_tokens=4)
    eng = Engine(build_model_from(cfg, ecfg, init_weights_v4(cfg, 0), device="cpu", ps=ps), ecfg)
    mine = [i for i in range(4) if i % world == rank]
    prompts = _tbo_prompts(cfg)
    split_decode = []
    orig = eng._tbo_logits

    def spy(seqs, max_tok):
        split_decode.append(bool(seqs) and all(len(q["tokens"]) == 1 for q in seqs) and len(seqs) > 1)
        return orig(seqs, max_tok)
    eng._tbo_logits = spy
    outs = eng.generate([prompts[i] for i in mine], [SamplingParams(max_tokens=TBO_MAXT[i]) for i in mine])
    return mine, [o.token_ids for o in outs], eng.stats.get("tbo_steps", 0), any(split_decode)


TBO_MAXT = [6, 8, 3, 8]


def _tbo_prompts(cfg):
    # rank 0: a 30-token prompt still prefilling while rank 1's two short
    # prompts already decode (a two-row decode batch inside overlapped steps)
    g = torch.Generator().manual_seed(8)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (30, 5, 4, 5)]


@pytest.mark.parametrize("compressed", [False, True])
def test_v4_dp2_two_batch_overlap_gloo(compressed):
    """Two-batch overlap for the V4 family under DP attention: prefill rows
    split in two micro-batches whose layer stacks interleave at the MoE
    exchange (Engram hashes, mHC and, compressed, the block compressor across
    the cut); steps where a rank decodes keep its batch whole (the E5 prune
    routes over the whole decode batch).  Tokens equal a single-process run."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import init_weights_v4
    cfg = _v4_tbo_cfg(compressed)
    res = run_ranks(_tbo_rank, 2, compressed)
    assert sum(r[2] for r in res) >= 1
    assert not any(r[3] for r in res)        # no multi-row decode batch went through the split
    prompts = _tbo_prompts(cfg)
    for mine, toks, _, _ in res:
        ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False, max_prefill_tokens=9)
        eng = Engine(build_model_from(cfg, ecfg, init_weights_v4(cfg, 0), device="cpu"), ecfg)
        want = [o.token_ids for o in eng.generate([prompts[i] for i in mine],
                                                  [SamplingParams(max_tokens=TBO_MAXT[i]) for i in mine])]
        assert toks == want, (mine, toks, want)


def _dp_rank_a2a(rank, world):
    import os
    os.environ["B200_DP_A2A_MIN_ROWS"] = "1"        # every step takes the all-to-all exchange
    return _dp_rank(rank, world)


def test_v4_dp2_all_to_all_exchange_gloo():
    """The V4 family's DP MoE through the all-to-all exchange (rows only to
    their experts' owners; E5-pruned decode routing travels with the rows):
    each rank's tokens equal a single-process run of its own requests."""
    from b200ds.engine.request import SamplingParams
    res = run_ranks(_dp_rank_a2a, 2)
    for mine, toks in res:
        eng, cfg = _v4_engine(chunk=7)
        prompts = _prompts(cfg, 3, 11, seed=6)
        maxt = [7, 4, 9]
        want = [o.token_ids for o in eng.generate([prompts[i].tolist() for i in mine],
                                                  [SamplingParams(max_tokens=maxt[i]) for i in mine])]
        assert toks == want, (mine, toks, want)
