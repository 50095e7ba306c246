"""Sparse MLA (lightning indexer + top-k) on CPU: the engine's model, with the
indexer projections fused into the attention GEMMs, must reproduce the fp32
oracle's tokens and logits, and so must a 2-rank gloo TP run."""
import dataclasses

import torch

from mp_util import run_ranks


def _cfg():
    from b200ds.config import tiny_config
    # top-8 of up to 48 cached tokens: the selection changes the result
    return dataclasses.replace(tiny_config(), index_n_heads=4, index_head_dim=32, index_topk=8)


def _prompts(cfg):
    g = torch.Generator().manual_seed(3)
    return torch.randint(0, cfg.vocab_size, (3, 24), generator=g)


def _engine(cfg, ps=None, world=1):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.models.reference import init_weights
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=world, ep_size=world)
    m = build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps)
    logs = []
    orig = m.forward
    m.forward = lambda fb: logs.append(orig(fb)) or logs[-1]
    return Engine(m, ecfg), logs


def _rank(rank, world):
    from b200ds.engine.request import SamplingParams
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo")
    cfg = _cfg()
    eng, logs = _engine(cfg, ps, world)
    outs = eng.generate(_prompts(cfg).tolist(), SamplingParams(max_tokens=12))
    return [o.token_ids for o in outs], logs


def test_sparse_engine_matches_oracle():
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import ReferenceModel, init_weights
    cfg = _cfg()
    oracle = ReferenceModel(cfg, init_weights(cfg, 0))
    otoks, ologits = oracle.greedy(_prompts(cfg), 12)
    eng, logs = _engine(cfg)
    outs = eng.generate(_prompts(cfg).tolist(), SamplingParams(max_tokens=12))
    assert [o.token_ids for o in outs] == otoks.tolist()
    assert (logs[0] - ologits[0]).abs().max() < 1e-4
    # the dense model gives different logits: the top-k selection is active
    dense = ReferenceModel(dataclasses.replace(cfg, index_n_heads=0), init_weights(cfg, 0))
    _, dlogits = dense.greedy(_prompts(cfg), 2)
    assert (dlogits[1] - ologits[1]).abs().max() > 1e-3
    res = run_ranks(_rank, 2)
    for toks, rlogs in res:
        assert toks == otoks.tolist()
        for a, b in zip(rlogs, logs):
            assert (a - b).abs().max() < 1e-4


def test_topk_reference_semantics():
    """indexer_scores returns the min(k, n) best causal positions, ascending,
    -1 padded."""
    from b200ds.ops import ref
    T, nh, hd, slots = 3, 2, 8, 64
    g = torch.Generator().manual_seed(0)
    q = torch.randn(T, nh, hd, generator=g)
    w = torch.rand(T, nh, generator=g)
    kc = torch.randn(slots, hd, generator=g)
    ks = torch.ones(slots)
    bt = torch.arange(8, dtype=torch.int32).view(1, 8)
    q_seq = torch.zeros(T, dtype=torch.int32)
    q_pos = torch.tensor([3, 20, 40], dtype=torch.int32)
    out = ref.indexer_scores(q, w, kc, ks, bt, q_seq, q_pos, 8, 6)
    assert out[0].tolist()[:4] == [0, 1, 2, 3] and out[0].tolist()[4:] == [-1, -1]
    for t in (1, 2):
        n = int(q_pos[t]) + 1
        sc = ((q[t] @ kc[:n].T).relu() * w[t].unsqueeze(-1)).sum(0)
        want = sorted(sc.topk(6).indices.tolist())
        assert out[t].tolist() == want
