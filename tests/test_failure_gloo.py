"""Failure detection on the host (CPU, gloo): a rank that raises in the
middle of serving must not leave its peers hanging - their next collective
ends with an error within the process-group timeout."""
from mp_util import run_ranks


def _faulty_rank(rank, world):
    import torch
    from b200ds.config import EngineConfig, tiny_config
    from b200ds import build_model_from
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo", timeout_s=15)
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=world, ep_size=world)
    m = build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps)
    calls = {"n": 0}
    orig = m.forward

    def fwd(fb):
        calls["n"] += 1
        if rank == 1 and calls["n"] == 4:
            raise RuntimeError("injected fault on rank 1")
        return orig(fb)
    m.forward = fwd
    eng = Engine(m, ecfg)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab_size, (2, 16), generator=g).tolist()
    try:
        eng.generate(prompts, SamplingParams(max_tokens=12))
    except Exception as e:          # the outcome is the test's subject
        return ("error", calls["n"], str(e)[:300])
    return ("ok", calls["n"], "")


def test_rank_fault_does_not_hang_peers():
    import time
    t0 = time.time()
    res = run_ranks(_faulty_rank, 2, timeout=120)
    assert res[1][0] == "error" and "injected fault" in res[1][2], res[1]
    # rank 0 saw its partner vanish at the next all-reduce instead of hanging
    assert res[0][0] == "error", res[0]
    assert res[0][1] <= 5, res[0]
    assert time.time() - t0 < 120
