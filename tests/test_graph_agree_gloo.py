"""Rank-agreed CUDA-graph capture verdicts.  A capture that fails on any rank
(an exception of any kind, out of memory) makes every rank drop that graph
and run eagerly from the same step on; an empty capture counts as a success.
Every rank ends with the same transcript of verdicts and step collectives,
and none hangs.  The captures are fakes (no GPU); the agreement is the
engine's own `capture_agreed`."""
import pytest
import torch

from mp_util import run_ranks

# scenario -> {(rank, capture index): exception to raise}
SCENARIOS = {
    "all_ok": {},
    "rank0_first": {(0, 0): RuntimeError("capture invalidated")},
    "rank1_second": {(1, 1): RuntimeError("operation not permitted when stream is capturing")},
    "both_first": {(0, 0): RuntimeError("a"), (1, 0): RuntimeError("b")},
    "oom_rank1": {(1, 0): torch.OutOfMemoryError("graph pool")},
    "bug_rank0_last": {(0, 2): ValueError("not a RuntimeError")},
}


def _rank(rank, world, name):
    import torch.distributed as dist
    from b200ds.engine.cuda_graph import GraphCaptureFailed, capture_agreed
    from b200ds.parallel.state import init_parallel
    ps = init_parallel(backend="gloo")
    fails = SCENARIOS[name]
    enabled, log = True, []
    for i in range(3):
        if enabled:
            def record(i=i):
                if (rank, i) in fails:
                    raise fails[(rank, i)]
                return None if i == 1 else f"graph{i}"      # capture 1 is empty
            try:
                capture_agreed(record, ps.cpu_group, f"graph {i}")
                log.append(("replay", i))
            except GraphCaptureFailed:
                enabled = False
                log.append(("eager-from", i))
        else:
            log.append(("eager", i))
        t = torch.tensor([i + 1], dtype=torch.int64)       # the step's own collective
        dist.all_reduce(t, group=ps.cpu_group)
        log.append(("step", int(t)))
    return log


@pytest.mark.parametrize("name", sorted(SCENARIOS))
def test_capture_verdict_is_agreed(name):
    out = run_ranks(_rank, 2, name, timeout=120)
    assert out[0] == out[1], out
    first_fail = min((i for (_, i) in SCENARIOS[name]), default=None)
    for i in range(3):
        mode = [m for m, j in out[0] if j == i and m != "step"][0]
        if first_fail is None or i < first_fail:
            assert mode == "replay"
        elif i == first_fail:
            assert mode == "eager-from"
        else:
            assert mode == "eager"
    assert [v for m, v in out[0] if m == "step"] == [2, 4, 6]


def test_engine_falls_back_to_eager_when_decode_capture_fails():
    """Engine integration: a decode-graph runner whose capture fails (agreed)
    is disabled at that step and decoding continues eagerly with the same
    tokens as an engine that never had graphs."""
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.cuda_graph import GraphCaptureFailed
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False)
    sd = init_weights(cfg, 0)
    prompts = [list(range(3, 15)), list(range(20, 29))]
    want = [o.token_ids for o in
            Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg).generate(prompts, SamplingParams(max_tokens=6))]

    class FailingRunner:
        enabled, calls, max_pages = True, 0, 64

        def can_run(self, n):
            return self.enabled

        def run(self, step, seqs, bucket=None):
            self.calls += 1
            raise GraphCaptureFailed("decode graph capture failed on a rank")

        def disable(self):
            self.enabled = False

    eng = Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)
    eng.graphs = FailingRunner()
    got = [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=6))]
    assert got == want
    assert eng.graphs.calls == 1 and not eng.graphs.enabled
