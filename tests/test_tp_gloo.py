"""Tiny DeepSeek-style model, fp32 on CPU, TP=2 over gloo.
Logits of a 2-rank run must match a single-process run to 1e-4."""
import torch

from mp_util import run_ranks


def _prompts(cfg):
    g = torch.Generator().manual_seed(1)
    return torch.randint(0, cfg.vocab_size, (4, 32), generator=g)


def _oracle_rank(rank, world):
    from b200ds.config import tiny_config
    from b200ds.models.reference import ReferenceModel, init_weights, shard_state_dict
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo")
    cfg = tiny_config()
    sd = shard_state_dict(init_weights(cfg, 0), cfg, ps)
    m = ReferenceModel(cfg, sd, ps)
    toks, logits = m.greedy(_prompts(cfg), 16)
    return toks, torch.stack(logits)


def _engine_rank(rank, world):
    from b200ds.config import EngineConfig, tiny_config
    from b200ds import build_model_from
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo")
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=world, ep_size=world)
    m = build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps)
    eng = Engine(m, ecfg)
    # capture logits of each step
    logs = []
    orig = m.forward
    def fwd(fb):
        out = orig(fb)
        logs.append(out.clone())
        return out
    m.forward = fwd
    outs = eng.generate(_prompts(cfg).tolist(), SamplingParams(max_tokens=16))
    return [o.token_ids for o in outs], logs


def test_oracle_tp2_matches_single():
    from b200ds.config import tiny_config
    from b200ds.models.reference import ReferenceModel, init_weights
    cfg = tiny_config()
    single = ReferenceModel(cfg, init_weights(cfg, 0))
    toks1, logits1 = single.greedy(_prompts(cfg), 16)
    res = run_ranks(_oracle_rank, 2)
    for toks, logits in res:
        assert torch.equal(toks, toks1)
        assert (logits - torch.stack(logits1)).abs().max() < 1e-4


def test_engine_tp2_matches_single_and_oracle():
    from b200ds.config import EngineConfig, tiny_config
    from b200ds import build_model_from
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import ReferenceModel, init_weights
    cfg = tiny_config()
    oracle = ReferenceModel(cfg, init_weights(cfg, 0))
    otoks, ologits = oracle.greedy(_prompts(cfg), 16)
    ecfg = EngineConfig(page_size=8, cuda_graphs=False)
    m = build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu")
    single_logs = []
    orig = m.forward
    m.forward = lambda fb: single_logs.append(orig(fb)) or single_logs[-1]
    outs = Engine(m, ecfg).generate(_prompts(cfg).tolist(), SamplingParams(max_tokens=16))
    assert [o.token_ids for o in outs] == otoks.tolist()
    # step 0 is the batched prefill: its last-token logits equal the oracle's
    assert (single_logs[0] - ologits[0]).abs().max() < 1e-4
    res = run_ranks(_engine_rank, 2)
    for toks, logs in res:
        assert toks == otoks.tolist()
        assert len(logs) == len(single_logs)
        for a, b in zip(logs, single_logs):
            assert (a - b).abs().max() < 1e-4
