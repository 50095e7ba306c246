"""Tracer host logic: phase spans from stamps, per-kind sums, disabled no-op,
and the model's mark sequence (CPU, stamps supplied by the test)."""


def test_tracer_report_and_summary():
    from b200ds.utils.trace import Tracer
    tr = Tracer("cpu", enabled=True)
    for n in ("embed", "L0.attn", "L0.ffn", "L1.attn", "L1.ffn", "head", "end"):
        tr.mark(n)
    st = [0, 1000, 4000, 5000, 9000, 10000, 12000]
    rep = tr.report(st)
    assert rep[0] == ("embed", 1.0) and rep[1] == ("L0.attn", 3.0) and len(rep) == 6
    s = tr.summary(st)
    assert s["attn"] == 7.0 and s["ffn"] == 2.0 and s["head"] == 2.0


def test_model_marks_each_layer_phase():
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.models.batch import build_batch
    from b200ds.models.reference import init_weights
    from b200ds.utils.trace import Tracer
    cfg = tiny_config()
    m = build_model_from(cfg, EngineConfig(page_size=8, cuda_graphs=False), init_weights(cfg, 0), device="cpu")
    m.allocate_kv(8)
    m.tracer = Tracer("cpu", enabled=True)
    m.forward(build_batch([{"tokens": [1, 2, 3], "start": 0, "pages": [1]}], 8))
    assert m.tracer.names == ["embed", "L0.attn", "L0.ffn", "L1.attn", "L1.ffn", "head"]
    off = Tracer("cpu", enabled=False)
    off.mark("x")
    assert off.names == [] and off.report([]) == []
