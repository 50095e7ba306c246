"""Prefill (extend) and speculative-verify CUDA graphs on the GPU: the
replayed prefill gives the eager logits; n-gram speculative decoding runs
its verify steps from graphs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _engine(**kw):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, small_gpu_config
    from b200ds.engine.engine import Engine
    from b200ds.models.reference import init_weights
    from b200ds import ops
    ops.set_impl("native")
    cfg = small_gpu_config()
    ecfg = EngineConfig(page_size=64, max_kv_pages=64, max_num_seqs=4, graph_batch_sizes=(4,), **kw)
    return Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cuda"), ecfg), cfg


def test_extend_graph_matches_eager_prefill():
    from b200ds.models.batch import build_batch
    eng, cfg = _engine(cuda_graphs=True, extend_graphs=True)
    from b200ds.engine.cuda_graph import ExtendGraphRunner
    runner = ExtendGraphRunner(eng, eng.graphs.max_pages)
    g = torch.Generator().manual_seed(0)
    seqs = [{"tokens": torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist(), "start": 0,
             "pages": eng.pool.alloc(1)} for n in (40, 17)]
    want = eng.model.forward(build_batch(seqs, 64, device="cuda")).float()
    got = runner.run(seqs).float()
    torch.cuda.synchronize()
    rel = ((got - want).norm() / want.norm()).item()
    assert rel < 1e-2, rel
    runner.release()


def test_spec_decode_with_verify_graphs():
    from b200ds.engine.request import SamplingParams
    eng, cfg = _engine(cuda_graphs=True, spec_ngram=3, spec_k=3, enable_prefix_cache=False)
    prompt = [7, 8, 9, 10, 7, 8, 9, 10, 7, 8, 9, 10, 7, 8]
    outs = eng.generate([prompt, prompt[::-1]], SamplingParams(max_tokens=12))
    torch.cuda.synchronize()
    assert all(len(o.token_ids) == 12 for o in outs)
    assert eng.verify_graphs is not None and eng.verify_graphs_ok and eng.stats.get("spec_proposed", 0) > 0
