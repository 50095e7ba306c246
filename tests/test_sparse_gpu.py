"""Sparse-MLA model on one GPU (native kernels: fused indexer projections,
tcgen05 indexer scores, radix top-k, tcgen05 sparse attention) against the
fp32 CPU oracle."""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg(**over):
    from b200ds.config import small_gpu_config
    c = small_gpu_config(index_n_heads=64, index_head_dim=128, index_topk=64, num_hidden_layers=2)
    return dataclasses.replace(c, **over)


def _seqs(cfg):
    g = torch.Generator().manual_seed(5)
    return [torch.randint(0, cfg.vocab_size, (n,), generator=g) for n in (200, 90)]


def _oracle(cfg, wcfg=None):
    from b200ds.models.reference import ReferenceModel, init_weights
    m = ReferenceModel(cfg, init_weights(wcfg or cfg, 0), max_len=256)
    outs = []
    for s in _seqs(cfg):
        m.reset(1)
        outs.append(m.forward(s.view(1, -1), 0)[0, -1])
    return torch.stack(outs)


def _rel(a, b):
    return ((a - b).norm() / b.norm()).item()


def test_sparse_model_matches_oracle():
    from b200ds import ops
    from b200ds.config import EngineConfig
    from b200ds.models.batch import build_batch
    from b200ds.models.loader import build_model
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import ParallelState
    import b200ds._C  # noqa: F401
    ops.set_impl("native")
    cfg = _cfg()
    ps = ParallelState(device=torch.device("cuda", 0))
    m = build_model(cfg, EngineConfig(), ps, init_weights(cfg, 0), device=ps.device)
    m.allocate_kv(16)
    seqs = _seqs(cfg)
    fb = build_batch([{"tokens": seqs[0].tolist(), "start": 0, "pages": [1, 2, 3, 4]},
                      {"tokens": seqs[1].tolist(), "start": 0, "pages": [5, 6]}], 64, device=ps.device)
    out = m.forward(fb).float().cpu()
    oracle = _oracle(cfg)
    dense = _oracle(dataclasses.replace(cfg, index_n_heads=0), cfg)    # same weights, no indexer
    e = _rel(out, oracle)
    # In this random model many keys have near-equal indexer scores, so the
    # e4m3 indexer operands alone move the oracle's logits by ~0.23 (relative)
    # through flipped selections at the top-k boundary.  The GPU run must stay
    # within that noise of the sparse oracle and well away from the dense
    # model (top-64 of up to 200 keys: ~0.74 apart).
    assert e < 0.4, e
    assert _rel(dense, oracle) > 2 * e, (e, _rel(dense, oracle))
