"""Host-side serving components on CPU: page pool reference counting, radix
prefix cache (match / insert / LRU eviction under locks), scheduler
(chunked prefill, preemption by recompute, page accounting), and engine
behaviours (prefix reuse gives identical tokens, stop tokens, sampling
determinism per seed, DP-free single process)."""
import pytest
import torch

from b200ds.engine.request import Request, SamplingParams
from b200ds.engine.scheduler import Scheduler
from b200ds.kv.pool import OutOfPages, PagePool
from b200ds.kv.radix import RadixCache


def test_page_pool_refcounts():
    pool = PagePool(8, 4)
    assert pool.num_free == 7                 # page 0 reserved
    a = pool.alloc(3)
    assert 0 not in a and pool.num_free == 4
    pool.retain(a[:1])
    pool.release(a)
    assert pool.num_free == 6                 # a[0] still referenced once
    pool.release(a[:1])
    assert pool.num_free == 7
    with pytest.raises(OutOfPages):
        pool.alloc(8)
    assert pool.pages_for(9) == 3


def test_radix_match_insert_evict():
    pool = PagePool(16, 2)
    rc = RadixCache(pool)
    toks = [1, 2, 3, 4, 5, 6]
    pages = pool.alloc(3)
    rc.insert(toks, pages)
    pool.release(pages)                       # the tree keeps its own references
    assert pool.num_free == 15 - 3
    got, nodes = rc.match([1, 2, 3, 4, 9, 9])
    assert got == pages[:2] and len(nodes) == 2
    # locked nodes are not evicted; the unlocked leaf is
    assert rc.evict(5) == 1
    assert pool.num_free == 15 - 2
    rc.unlock(nodes)
    assert rc.evict(5) == 2
    assert pool.num_free == 15 and rc.num_nodes == 0


def _req(i, n, max_tokens=4):
    return Request(i, list(range(100 * i, 100 * i + n)), SamplingParams(max_tokens=max_tokens))


def test_scheduler_chunked_prefill_and_decode():
    pool = PagePool(64, 4)
    s = Scheduler(pool, max_num_seqs=4, max_prefill_tokens=10)
    a, b = _req(1, 13), _req(2, 5)
    s.add(a)
    s.add(b)
    st = s.next_step()
    assert st.kind == "prefill" and [len(c) for c in st.chunks] == [10] and st.sample == [False]
    s.commit(st)
    st = s.next_step()                        # b (5, waited for budget) + the rest of a (3)
    assert st.kind == "prefill" and st.reqs == [b, a] and [len(c) for c in st.chunks] == [5, 3]
    assert st.sample == [True, True]
    s.commit(st)
    for r in (a, b):
        r.output.append(7)
    st = s.next_step()
    assert st.kind == "decode" and sorted(st.starts) == [5, 13]
    assert all(len(r.pages) * 4 >= r.cached + 1 for r in (a, b))


def test_scheduler_preempts_when_pages_run_out():
    pool = PagePool(5, 4)                     # 4 usable pages = 16 tokens
    s = Scheduler(pool, max_num_seqs=4, max_prefill_tokens=64)
    a, b = _req(1, 7), _req(2, 7)
    s.add(a)
    s.add(b)
    s.commit(s.next_step())
    for r in (a, b):
        r.output.append(1)
    st = s.next_step()
    s.commit(st)
    for r in (a, b):
        r.output.append(1)
    st = s.next_step()                        # a needs a 3rd page: b is preempted and re-queued
    assert st.kind == "decode" and st.reqs == [a]
    assert b.cached == 0 and b.pages == [] and s.waiting[0] is b


def _engine(prefix_cache=True, **kw):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=prefix_cache, **kw)
    return Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu"), ecfg), cfg


def test_prefix_cache_reuse_is_transparent():
    eng, cfg = _engine(True)
    g = torch.Generator().manual_seed(4)
    shared = torch.randint(0, cfg.vocab_size, (24,), generator=g).tolist()
    p1 = shared + [5, 6, 7]
    p2 = shared + [8, 9]
    first = eng.generate([p1], SamplingParams(max_tokens=6))[0].token_ids
    again = eng.generate([p1, p2], SamplingParams(max_tokens=6))
    assert eng.radix.num_nodes > 0
    ref_eng, _ = _engine(False)
    ref = ref_eng.generate([p1, p2], SamplingParams(max_tokens=6))
    assert again[0].token_ids == first == ref[0].token_ids
    assert again[1].token_ids == ref[1].token_ids


def test_stop_tokens_and_seeded_sampling():
    eng, cfg = _engine(False)
    prompt = list(range(10))
    greedy = eng.generate([prompt], SamplingParams(max_tokens=8))[0].token_ids
    stop = greedy[3]
    out = eng.generate([prompt], SamplingParams(max_tokens=8, stop_token_ids=[stop]))[0]
    assert out.finish_reason == "stop" and out.token_ids == greedy[: greedy.index(stop) + 1]
    sp = SamplingParams(max_tokens=8, temperature=0.9, top_p=0.95, seed=123)
    a = eng.generate([prompt], sp)[0].token_ids
    b = eng.generate([prompt], sp)[0].token_ids
    assert a == b


def test_mixed_steps_same_tokens_and_no_decode_stall():
    """Mixed steps: while a long prompt prefills in chunks, running requests
    keep decoding (one token per step) and every request gets the tokens of
    the prefill-first schedule."""
    def run(mixed):
        eng, cfg = _engine(False, mixed_steps=mixed, max_prefill_tokens=6)
        from b200ds.engine.request import SamplingParams
        a = eng.add_request(list(range(3, 12)), SamplingParams(max_tokens=12))
        for _ in range(3):
            eng.step()
        b = eng.add_request(list(range(100, 140)), SamplingParams(max_tokens=4))
        grew = []
        while not (a.finished and b.finished):
            n = len(a.output)
            eng.step()
            if b.t_first is None and not a.finished:
                grew.append(len(a.output) > n)
        return a.output, b.output, grew
    a0, b0, g0 = run(False)
    a1, b1, g1 = run(True)
    assert a1 == a0 and b1 == b0
    assert all(g1) and not all(g0)          # prefill-first stalls a's decoding; mixed does not


def test_abort_waiting_prefilling_running():
    """Aborting frees the request's pages wherever it is; the others finish
    with their usual tokens."""
    from b200ds.engine.request import SamplingParams
    eng, cfg = _engine(False, max_prefill_tokens=8)
    free0 = eng.pool.num_free
    ref_eng, _ = _engine(False, max_prefill_tokens=8)
    keep_ref = ref_eng.generate([list(range(5, 25))], SamplingParams(max_tokens=6))[0].token_ids
    keep = eng.add_request(list(range(5, 25)), SamplingParams(max_tokens=6))
    mid = eng.add_request(list(range(30, 60)), SamplingParams(max_tokens=6))
    late = eng.add_request(list(range(70, 80)), SamplingParams(max_tokens=6))
    eng.step()                                   # keep is mid-prefill, mid / late wait
    eng.abort(late)                              # waiting
    eng.step()
    eng.abort(mid)                               # prefilling
    while not keep.finished:
        eng.step()
    assert keep.output == keep_ref
    assert late.finish_reason == "abort" and mid.finish_reason == "abort"
    run = eng.add_request(list(range(90, 100)), SamplingParams(max_tokens=50))
    for _ in range(4):
        eng.step()
    eng.abort(run)                               # running
    assert not eng.sched.has_work and eng.pool.num_free == free0


def test_server_cancel_aborts_request():
    """A subscription whose client went away is aborted by the worker."""
    import time as _t
    from b200ds.engine.request import SamplingParams
    from b200ds.server.openai import EngineWorker
    eng, cfg = _engine(False)

    class Loop:
        def __init__(self):
            self.items = []

        def call_soon_threadsafe(self, fn, item):
            fn(item)

        def put_nowait(self, item):
            self.items.append(item)
    w = EngineWorker(eng, None).start()
    lp = Loop()
    w.submit(list(range(40)), SamplingParams(max_tokens=8000), lp, lp)
    t0 = _t.time()
    while not any(ev[0] == "tokens" for ev in lp.items) and _t.time() - t0 < 60:
        _t.sleep(0.01)
    w.cancel(lp)
    while not any(ev[0] == "done" for ev in lp.items) and _t.time() - t0 < 60:
        _t.sleep(0.01)
    w.stop()
    assert ("done", "abort") in lp.items and not eng.sched.has_work


def test_logprobs_match_oracle_and_leave_tokens_unchanged():
    """SamplingParams.logprobs: every output token carries the model's
    log-probability (log-softmax of the raw logits) and the top-n
    alternatives; the values match the fp32 oracle's logits of the prefix,
    and asking for them does not change the tokens."""
    from b200ds.models.reference import ReferenceModel, init_weights
    eng, cfg = _engine(False)
    g = torch.Generator().manual_seed(8)
    prompts = torch.randint(0, cfg.vocab_size, (2, 11), generator=g).tolist()
    plain = [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=5))]
    outs = eng.generate(prompts, SamplingParams(max_tokens=5, logprobs=3))
    assert [o.token_ids for o in outs] == plain
    oracle = ReferenceModel(cfg, init_weights(cfg, 0))
    for p, o in zip(prompts, outs):
        assert len(o.logprobs) == len(o.token_ids)
        seq = torch.tensor([p + o.token_ids])
        oracle.reset(1)
        want = torch.log_softmax(oracle.forward(seq, 0)[0].float(), -1)
        for j, (t, lp, top) in enumerate(o.logprobs):
            row = want[len(p) - 1 + j]
            assert t == o.token_ids[j] and abs(lp - float(row[t])) < 1e-3
            assert [a for a, _ in top] == row.topk(3).indices.tolist()
            assert top[0][0] == t                       # greedy: the sampled token is the top one
    none = eng.generate(prompts[:1], SamplingParams(max_tokens=3))[0]
    assert none.logprobs is None
    zero = eng.generate(prompts[:1], SamplingParams(max_tokens=3, logprobs=0))[0]
    assert all(top == [] for _, _, top in zero.logprobs) and len(zero.logprobs) == 3


def test_lpm_policy_admits_the_longest_cached_prefix_first():
    """schedule_policy lpm: with one free slot, a waiting request whose prompt
    shares a cached prefix goes before an earlier one that shares nothing
    (fcfs keeps arrival order); outputs are unchanged by the order."""
    from b200ds.kv.radix import RadixCache
    for policy, first in (("fcfs", "b"), ("lpm", "c")):
        pool = PagePool(64, 4)
        radix = RadixCache(pool)
        shared = list(range(100, 116))                   # 4 full pages
        pages = pool.alloc(4)
        radix.insert(shared, pages)
        pool.release(pages)
        s = Scheduler(pool, max_num_seqs=1, max_prefill_tokens=64, radix=radix, policy=policy)
        b = Request(1, list(range(1, 19)), SamplingParams())
        c = Request(2, shared + [7, 8], SamplingParams())
        s.add(b)
        s.add(c)
        st = s.next_step()
        assert st.reqs == [b if first == "b" else c]
        if first == "c":
            assert c.cached == 16 and [len(x) for x in st.chunks] == [2]
    import pytest
    with pytest.raises(ValueError):
        Scheduler(PagePool(8, 4), 1, 8, policy="random")
    eng, cfg = _engine(True, schedule_policy="lpm")
    ref_eng, _ = _engine(False)
    g = torch.Generator().manual_seed(12)
    shared = torch.randint(0, cfg.vocab_size, (24,), generator=g).tolist()
    prompts = [shared + [1, 2], torch.randint(0, cfg.vocab_size, (9,), generator=g).tolist(), shared + [3]]
    eng.generate(prompts[:1], SamplingParams(max_tokens=2))
    got = [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=5))]
    want = [o.token_ids for o in ref_eng.generate(prompts, SamplingParams(max_tokens=5))]
    assert got == want


def test_prompt_logprobs_under_chunked_prefill_match_oracle():
    """prompt_logprobs: every prompt token after the first gets the model's
    log-probability (and top-n) from the row before it, across prefill
    chunks and with the prefix cache on (such requests recompute the whole
    prompt); max_tokens=0 returns after the prompt without a token."""
    from b200ds.config import EngineConfig
    from b200ds.models.reference import ReferenceModel, init_weights
    eng, cfg = _engine(True, max_prefill_tokens=7)
    g = torch.Generator().manual_seed(21)
    prompt = torch.randint(0, cfg.vocab_size, (19,), generator=g).tolist()
    eng.generate([prompt], SamplingParams(max_tokens=2))               # the prompt's pages are now cached
    out = eng.generate([prompt, prompt[:9]], [SamplingParams(max_tokens=3, prompt_logprobs=2),
                                              SamplingParams(max_tokens=0, prompt_logprobs=0)])
    oracle = ReferenceModel(cfg, init_weights(cfg, 0))
    for o, p in zip(out, (prompt, prompt[:9])):
        oracle.reset(1)
        want = torch.log_softmax(oracle.forward(torch.tensor([p]), 0)[0].float(), -1)
        assert len(o.prompt_logprobs) == len(p) and o.prompt_logprobs[0] is None
        for j in range(1, len(p)):
            t, lp, top = o.prompt_logprobs[j]
            assert t == p[j] and abs(lp - float(want[j - 1, t])) < 1e-3
            assert [a for a, _ in top] == want[j - 1].topk(len(top)).indices.tolist() if top else True
    assert len(out[0].token_ids) == 3 and out[1].token_ids == [] and out[1].finish_reason == "length"
    plain = eng.generate([prompt], SamplingParams(max_tokens=3))[0]
    assert plain.token_ids == out[0].token_ids and plain.prompt_logprobs is None


def test_gauges_count_prefix_hits():
    eng, cfg = _engine(True)
    p = list(range(40, 72))                                  # 32 tokens = 4 pages of 8
    eng.generate([p], SamplingParams(max_tokens=2))
    g0 = eng.gauges()
    assert g0["admitted_prompt_tokens"] == 32 and g0["prefix_hit_tokens"] == 0
    eng.generate([p + [5]], SamplingParams(max_tokens=2))
    g1 = eng.gauges()
    assert g1["admitted_prompt_tokens"] == 65 and g1["prefix_hit_tokens"] == 32
    assert g1["running"] == 0 and g1["waiting"] == 0 and g1["kv_pages_free"] <= g1["kv_pages_total"]


def test_stream_yields_tokens_as_they_come():
    eng, cfg = _engine(False)
    prompts = [list(range(3, 12)), list(range(30, 35))]
    want = [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=5))]
    got, final = [[], []], None
    for i, toks in eng.stream(prompts, SamplingParams(max_tokens=5)):
        if i == "done":
            final = toks
        else:
            assert toks
            got[i].extend(toks)
    assert got == want and [o.token_ids for o in final] == want


def test_check_request_limits():
    import pytest
    eng, cfg = _engine(False, max_model_len=64)
    for prompt, mt in (([], 1), ([cfg.vocab_size], 1), ([-1], 1), (list(range(60)), 10), ([1, 2], -1)):
        with pytest.raises(ValueError):
            eng.add_request(prompt, SamplingParams(max_tokens=mt))
    assert not eng.sched.has_work
    eng.check_request(list(range(60)), SamplingParams(max_tokens=4))


def test_tensor_prompts_are_accepted():
    eng, cfg = _engine(False)
    p = torch.arange(3, 12)
    a = eng.generate([p], SamplingParams(max_tokens=3))[0].token_ids
    b = eng.generate([p.tolist()], SamplingParams(max_tokens=3))[0].token_ids
    assert a == b


def test_single_group_many_experts_matches_oracle():
    """The Kimi-K2 routing shape (one expert group, top-8 of many experts,
    one dense first layer) on a tiny model: engine tokens equal the oracle's."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, PRESETS, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.models.reference import ReferenceModel, init_weights
    k2 = PRESETS["kimi-k2-1t"]()
    assert k2.n_group == 1 and k2.n_routed_experts == 384 and 1.0e12 < k2.num_params() < 1.1e12
    cfg = tiny_config(n_routed_experts=24, num_experts_per_tok=8, n_group=1, topk_group=1,
                      routed_scaling_factor=2.827)
    sd = init_weights(cfg, 0)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False)
    eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
    g = torch.Generator().manual_seed(17)
    prompts = torch.randint(0, cfg.vocab_size, (2, 12), generator=g)
    outs = eng.generate(prompts.tolist(), SamplingParams(max_tokens=5))
    toks, _ = ReferenceModel(cfg, sd).greedy(prompts, 5)
    assert [o.token_ids for o in outs] == toks.tolist()


def test_priority_policy_admits_lower_priority_values_first():
    pool = PagePool(64, 4)
    s = Scheduler(pool, max_num_seqs=1, max_prefill_tokens=64, policy="priority")
    a = Request(1, list(range(1, 9)), SamplingParams(priority=5))
    b = Request(2, list(range(11, 19)), SamplingParams(priority=-1))
    c = Request(3, list(range(21, 29)), SamplingParams(priority=5))
    for r in (a, b, c):
        s.add(r)
    assert s.next_step().reqs == [b]
    assert [r.rid for r in s.waiting] == [1, 3]          # arrival order within a level


def test_stop_strings_in_engine_api():
    from b200ds.engine.tokenizer import ByteTokenizer
    eng, cfg = _engine(False)
    eng.tokenizer = ByteTokenizer()
    p = eng.tokenizer.encode("go:")
    full = eng.generate([p], SamplingParams(max_tokens=10))[0]
    stop = full.text[3:5]
    o = eng.generate([p], SamplingParams(max_tokens=10, stop=[stop]))[0]
    assert o.finish_reason == "stop" and o.text == full.text[: full.text.find(stop)]
    assert len(o.token_ids) < 10
