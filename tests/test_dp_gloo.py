"""DP attention + EP MoE on CPU (gloo, 2 ranks): each rank serves its own
requests, the MoE exchanges tokens between ranks, and every request's tokens
and prefill logits must match a single-process run of all requests."""
import pytest
import torch

from mp_util import run_ranks


def _prompts(cfg):
    g = torch.Generator().manual_seed(7)
    # uneven: rank 0 serves 2 requests, rank 1 one shorter request, so the
    # ranks' token counts differ and rank 1 idles (dummy forwards) at the end
    lens = [20, 13, 9]
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]


def _max_tokens():
    return [10, 6, 14]


def _run(cfg, ecfg, prompts, maxt, ps=None):
    from b200ds import build_model_from
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    m = build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps)
    logs = []
    orig = m.forward
    m.forward = lambda fb: logs.append((fb.num_tokens, orig(fb))) or logs[-1][1]
    eng = Engine(m, ecfg)
    outs = eng.generate(prompts, [SamplingParams(max_tokens=n) for n in maxt])
    return [o.token_ids for o in outs], logs


def _rank(rank, world):
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    assert ps.tp_size == 1 and ps.ep_size == world
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True)
    mine = [i for i in range(3) if i % world == rank]
    prompts = [_prompts(cfg)[i] for i in mine]
    maxt = [_max_tokens()[i] for i in mine]
    toks, logs = _run(cfg, ecfg, prompts, maxt, ps)
    return mine, toks, logs[0][1]


def test_dp2_ep2_matches_single():
    from b200ds.config import EngineConfig, tiny_config
    cfg = tiny_config()
    ref_toks, _ = _run(cfg, EngineConfig(page_size=8, cuda_graphs=False), _prompts(cfg), _max_tokens())
    # single-process prefill logits of each prompt alone (the DP ranks'
    # first forward is their own prompts' prefill)
    res = run_ranks(_rank, 2)
    for mine, toks, first_logits in res:
        assert toks == [ref_toks[i] for i in mine]
        _, logs = _run(cfg, EngineConfig(page_size=8, cuda_graphs=False), [_prompts(cfg)[i] for i in mine],
                       [1] * len(mine))
        assert (first_logits - logs[0][1]).abs().max() < 1e-4


def _spec_rank(rank, world):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        spec_ngram=3, spec_k=3)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps), ecfg)
    mine = [i for i in range(3) if i % world == rank]
    prompts = _spec_prompts(cfg)
    outs = eng.generate([prompts[i] for i in mine], [SamplingParams(max_tokens=(16, 9, 20)[i]) for i in mine])
    return mine, [o.token_ids for o in outs], eng.stats.get("spec_proposed", 0), eng.stats["steps"]


def _spec_prompts(cfg):
    g = torch.Generator().manual_seed(5)
    base = torch.randint(0, cfg.vocab_size, (5,), generator=g).tolist()
    return [base * 4, torch.randint(0, cfg.vocab_size, (11,), generator=g).tolist(), base[:3] * 5]


def test_dp2_speculative_ngram_matches_single():
    """n-gram speculative decoding under DP attention: ranks that verify
    drafts and ranks that decode plainly share one lockstep forward per
    step; every request's tokens equal a single-process run without
    speculation."""
    from b200ds.config import EngineConfig, tiny_config
    cfg = tiny_config()
    ref, _ = _run(cfg, EngineConfig(page_size=8, cuda_graphs=False), _spec_prompts(cfg), [16, 9, 20])
    res = run_ranks(_spec_rank, 2)
    assert sum(r[2] for r in res) > 0                    # drafts were proposed and verified
    for mine, toks, _, _ in res:
        assert toks == [ref[i] for i in mine]


def _tbo_rank(rank, world, idle_rank1=False):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        tbo=True, tbo_min_tokens=4)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps), ecfg)
    mine = [i for i in range(3) if (rank == 0 if idle_rank1 else i % world == rank)]
    if not mine:            # an idle rank: dummy micro-batches in every overlapped step
        eng._drain_dp()
        return mine, [], eng.stats.get("tbo_steps", 0)
    outs = eng.generate([_prompts(cfg)[i] for i in mine], [SamplingParams(max_tokens=_max_tokens()[i]) for i in mine])
    return mine, [o.token_ids for o in outs], eng.stats.get("tbo_steps", 0)


@pytest.mark.parametrize("idle_rank1", [False, True])
def test_dp2_two_batch_overlap_matches_single(idle_rank1):
    """Two-batch overlap of DP prefill steps: each rank's rows run as two
    micro-batches interleaved at the MoE exchange's asynchronous collectives
    (rank 0's 20 + 13 rows split inside the second prompt, so its second half
    reads the first half's cache rows; rank 1's prompt alone); tokens equal a
    single-process run."""
    from b200ds.config import EngineConfig, tiny_config
    cfg = tiny_config()
    ref, _ = _run(cfg, EngineConfig(page_size=8, cuda_graphs=False), _prompts(cfg), _max_tokens())
    res = run_ranks(_tbo_rank, 2, idle_rank1)
    for mine, toks, tbo_steps in res:
        assert tbo_steps >= 1
        assert toks == [ref[i] for i in mine]


def _a2a_rank(rank, world, tbo):
    import os
    os.environ["B200_DP_A2A_MIN_ROWS"] = "1"        # every step takes the all-to-all exchange
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel import ep_a2a
    from b200ds.parallel.state import init_parallel
    calls = []
    orig = ep_a2a.a2a_moe_steps

    def spy(*a, **k):
        calls.append(1)
        return (yield from orig(*a, **k))
    ep_a2a.a2a_moe_steps = spy
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        tbo=tbo, tbo_min_tokens=4)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps), ecfg)
    mine = [i for i in range(3) if i % world == rank]
    outs = eng.generate([_prompts(cfg)[i] for i in mine], [SamplingParams(max_tokens=_max_tokens()[i]) for i in mine])
    return mine, [o.token_ids for o in outs], len(calls)


@pytest.mark.parametrize("tbo", [False, True])
def test_dp2_all_to_all_exchange_matches_single(tbo):
    """The all-to-all MoE exchange (each row only to its experts' owners,
    partial sums back to the source rows), alone and interleaved by two-batch
    overlap: tokens equal a single-process run."""
    from b200ds.config import EngineConfig, tiny_config
    cfg = tiny_config()
    ref, _ = _run(cfg, EngineConfig(page_size=8, cuda_graphs=False), _prompts(cfg), _max_tokens())
    res = run_ranks(_a2a_rank, 2, tbo)
    for mine, toks, calls in res:
        assert calls > 0
        assert toks == [ref[i] for i in mine]


def test_a2a_send_plan():
    """Rows go once to every rank owning one of their experts."""
    import torch
    from b200ds.parallel.ep_a2a import send_plan
    ids = torch.tensor([[0, 5], [1, 2], [7, -1], [6, 4]])     # 8 experts, 2 per rank, 4 ranks
    row, counts = send_plan(ids, 2, 4)
    assert counts.tolist() == [2, 1, 2, 2]
    assert row.tolist() == [0, 1, 1, 0, 3, 2, 3]
