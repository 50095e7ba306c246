"""DP-attention serving plumbing on 2 gloo ranks: rank 0 assigns requests
round-robin, rank 1 serves its share, tokens of both ranks stream back
through rank 0; stopping ends the follower."""
import threading
import time

import pytest

from mp_util import run_ranks


class _Loop:
    """Stand-in for the asyncio loop and queue of an HTTP handler."""

    def __init__(self):
        self.events = []
        self.lock = threading.Lock()

    def call_soon_threadsafe(self, fn, item):
        with self.lock:
            fn(item)

    def put_nowait(self, item):
        self.events.append(item)


def _rank(rank, world, cp=False):
    import torch
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    from b200ds.parallel.state import init_parallel
    from b200ds.server.openai import DPEngineWorker, follower_loop
    ps = init_parallel(backend="gloo", dp_attention=True)
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, tp_size=1, ep_size=world, dp_attention=True,
                        context_parallel=cp, cp_min_tokens=16, max_prefill_tokens=8)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu", ps=ps), ecfg)
    if rank != 0:
        follower_loop(eng, ps)
        return None
    w = DPEngineWorker(eng, None, ps).start()
    g = torch.Generator().manual_seed(9)
    prompts = torch.randint(0, cfg.vocab_size, (3, 10), generator=g).tolist()
    if cp:      # one long prompt (assigned to rank 1) prefills on both ranks
        prompts[1] = torch.randint(0, cfg.vocab_size, (27,), generator=g).tolist()
    loops = [_Loop() for _ in prompts]
    for p, lp in zip(prompts, loops):
        w.submit(p, SamplingParams(max_tokens=5), lp, lp)
    t0 = time.time()
    while time.time() - t0 < 120:
        if all(any(e[0] == "done" for e in lp.events) for lp in loops):
            break
        time.sleep(0.01)
    w.stop()
    return prompts, [[t for e in lp.events if e[0] == "tokens" for t in e[1]] for lp in loops]


@pytest.mark.parametrize("cp", [False, True])
def test_dp_server_streams_every_ranks_tokens(cp):
    import torch
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    res = run_ranks(_rank, 2, cp)
    prompts, got = [r for r in res if r is not None][0]
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False)
    eng = Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu"), ecfg)
    want = [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=5))]
    assert got == want
