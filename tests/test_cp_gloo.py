"""Context-parallel prefill under DP attention on CPU (gloo): a long prompt
prefills on every rank (rows split round-robin, each layer's new cache rows
all-gathered), the owner rank decodes it, and its tokens must equal a
single-process run of the same prompt; the ranks' own requests keep stepping
in lockstep around the context-parallel chunks."""
import dataclasses

import pytest
import torch

from mp_util import run_ranks


def _cfg(sparse: bool):
    from b200ds.config import tiny_config
    cfg = tiny_config()
    if sparse:      # top-8 of up to 45 cached tokens: the gathered indexer keys matter
        cfg = dataclasses.replace(cfg, index_n_heads=4, index_head_dim=32, index_topk=8)
    return cfg


def _prompts(cfg):
    g = torch.Generator().manual_seed(11)
    # the context-parallel prompt (33 tokens: chunks of 16, 16 and 1 at two
    # ranks, so the last chunk leaves one rank without rows) and one ordinary
    # request per rank
    lens = [33, 12, 9]
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]


MAXT = [8, 6, 5]


def _single(cfg, prompts, maxt):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    ecfg = EngineConfig(page_size=8, cuda_graphs=False)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu"), ecfg)
    outs = eng.generate(prompts, [SamplingParams(max_tokens=n) for n in maxt])
    return [o.token_ids for o in outs]


def _rank(rank, world, sparse, owner, a2a=False):
    if a2a:
        import os
        os.environ["B200_DP_A2A_MIN_ROWS"] = "1"    # the chunks' MoE rows go all-to-all
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = _cfg(sparse)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        context_parallel=True, max_prefill_tokens=8)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps), ecfg)
    prompts = _prompts(cfg)
    own = eng.add_request(prompts[1 + rank], SamplingParams(max_tokens=MAXT[1 + rank]))
    cp = eng.add_request(prompts[0], SamplingParams(max_tokens=MAXT[0]), cp_owner=owner)
    while not (own.finished and cp.finished):
        eng.step()
    eng._drain_dp()
    return rank, own.output, cp.output, cp.finish_reason, eng.pool.num_free, eng.stats["prefill_tokens"]


@pytest.mark.parametrize("sparse,a2a", [(False, False), (True, False), (False, True)])
def test_cp2_prefill_matches_single(sparse, a2a):
    cfg = _cfg(sparse)
    prompts = _prompts(cfg)
    ref = _single(cfg, prompts, MAXT)
    owner = 1       # the prompt's last row is computed on rank 0: the row crosses ranks
    res = run_ranks(_rank, 2, sparse, owner, a2a)
    for rank, own, cp, reason, _, _ in res:
        assert own == ref[1 + rank]
        if rank == owner:
            assert cp == ref[0]
            assert reason == "length"
        else:
            assert cp == [] and reason == "context_parallel_peer"
    # each rank prefilled its own prompt plus its half of the long one
    # (33 = 8 + 8 + 1 rows on rank 0, 8 + 8 on rank 1)
    assert {r[0]: r[5] for r in res} == {0: len(prompts[1]) + 17, 1: len(prompts[2]) + 16}


def _rank_abort(rank, world):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = _cfg(False)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        context_parallel=True, max_prefill_tokens=8, enable_prefix_cache=False)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps), ecfg)
    free0 = eng.pool.num_free
    prompts = _prompts(cfg)
    a = eng.add_request(prompts[0], SamplingParams(max_tokens=4), cp_owner=0)
    b = eng.add_request(prompts[0][:20], SamplingParams(max_tokens=3), cp_owner=1)
    eng.step()                      # first chunk of a
    if rank == 0:
        eng.abort(a)                # only the owner learns of the abort; the ranks agree on it
    while not b.finished:
        eng.step()
    eng._drain_dp()
    return rank, a.finish_reason, b.output, b.finish_reason, eng.pool.num_free == free0


def test_cp2_abort_is_agreed():
    cfg = _cfg(False)
    ref = _single(cfg, [_prompts(cfg)[0][:20]], [3])
    res = run_ranks(_rank_abort, 2)
    for rank, ra, bout, rb, pages_back in res:
        assert ra == "abort"
        assert pages_back
        if rank == 1:
            assert bout == ref[0] and rb == "length"
        else:
            assert bout == [] and rb == "context_parallel_peer"


def test_cp_layout_round_robin():
    from b200ds.parallel.cp import build_cp_batch, holder_of_last, layout
    pages = [5, 2, 9, 7]
    lay = layout(3, 10, 3, pages, 4)            # positions 3..12 over 3 ranks
    assert lay.counts == [4, 3, 3] and lay.tmax == 4
    # chunk order: position 3 is rank 0 row 0, 4 is rank 1 row 0, ...
    assert lay.src_rows.tolist() == [0, 4, 8, 1, 5, 9, 2, 6, 10, 3]
    assert lay.dst_slots.tolist() == [pages[p // 4] * 4 + p % 4 for p in range(3, 13)]
    fb = build_cp_batch(list(range(100, 120)), 3, 10, 3, 2, pages, 4)
    assert fb.positions.tolist() == [5, 8, 11] and fb.input_ids.tolist() == [105, 108, 111]
    assert holder_of_last(10, 3) == 0
    empty = build_cp_batch(list(range(20)), 0, 1, 2, 1, pages, 4)     # rank 1 has no rows
    assert empty.out_slots.tolist() == [0] and empty.cp.counts == [1, 0]


def _v4_cfg(compressed: bool):
    from b200ds.config import tiny_v4_config
    if compressed:      # indexer, compressed blocks at ratios 2 / 4, Engram at layer 1
        return tiny_v4_config(index_n_heads=8, index_head_dim=32, index_topk=6, index_swa=4,
                              compress_ratios=(0, 2, 4), compress_topk=4)
    return tiny_v4_config()


def _v4_single(cfg, prompt, maxt):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import init_weights_v4
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False)
    eng = Engine(build_model_from(cfg, ecfg, init_weights_v4(cfg, 0), device="cpu"), ecfg)
    return eng.generate([prompt], SamplingParams(max_tokens=maxt))[0].token_ids


def _v4_rank(rank, world, compressed):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference_v4 import init_weights_v4
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = _v4_cfg(compressed)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        context_parallel=True, max_prefill_tokens=8)
    eng = Engine(build_model_from(cfg, ecfg, init_weights_v4(cfg, 0), device="cpu", ps=ps), ecfg)
    r = eng.add_request(_prompts(cfg)[0], SamplingParams(max_tokens=6), cp_owner=1)
    while not r.finished:
        eng.step()
    eng._drain_dp()
    return rank, r.output, r.finish_reason


@pytest.mark.parametrize("compressed", [False, True])
def test_cp2_v4_prefill_matches_single(compressed):
    """The V4 family under context parallelism: each rank's n-gram hashes
    read the whole chunk's tokens from the token cache, compressed layers
    gather the gate logits with the cache rows and every rank compresses the
    chunk's blocks; the owner's tokens equal a single-process run."""
    cfg = _v4_cfg(compressed)
    want = _v4_single(cfg, _prompts(cfg)[0], 6)
    res = run_ranks(_v4_rank, 2, compressed)
    for rank, out, reason in res:
        if rank == 1:
            assert out == want and reason == "length"
        else:
            assert out == [] and reason == "context_parallel_peer"


def _rank_generate(rank, world):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = _cfg(False)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        context_parallel=True, max_prefill_tokens=8)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps), ecfg)
    prompts = _prompts(cfg)
    outs = eng.generate(prompts[:2], SamplingParams(max_tokens=5), cp_owner=[0, 1])
    return rank, [o.token_ids for o in outs]


def test_cp2_generate_with_owners():
    """Engine.generate with per-prompt owners: both prompts prefill on both
    ranks, prompt i decodes on rank i."""
    cfg = _cfg(False)
    ref = _single(cfg, _prompts(cfg)[:2], [5, 5])
    for rank, toks in run_ranks(_rank_generate, 2):
        assert toks[rank] == ref[rank] and toks[1 - rank] == []
