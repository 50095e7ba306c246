"""Engine features that ride on the GPU kernels, run on a B200: loading an HF
fp8 checkpoint (128 x 128 fp32 or 32 x 32 UE8M0 block scales) with the dequantize / requantize on
the device, the full-logits step path (log-probabilities, penalties, guided
decoding) next to the decode graphs, the host-memory tier of the prefix
cache, and the tactic tuner."""
import json
import os
import subprocess
import sys

import pytest
import regex
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(autouse=True)
def _restore_switches():
    from b200ds.utils import levers
    before = levers.switches()
    yield
    for k, v in before.items():
        levers.set_switch(k, v)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("block,ue8m0", [(128, False), (32, True)])
def test_fp8_checkpoint_loads_on_the_gpu(tmp_path, block, ue8m0):
    """Checkpoint bytes cross the host link as fp8 and are dequantized
    (128 x 128 fp32 or 32 x 32 UE8M0 block scales) and requantized to the
    serving formats on the device; the served model follows the one built
    straight from the same weights."""
    from b200ds import EngineConfig, SamplingParams, build_model_from, load_engine
    from b200ds.config import small_gpu_config
    from b200ds.engine.engine import Engine
    from b200ds.models.loader import save_checkpoint_fp8
    from b200ds.models.reference import init_weights
    from b200ds.ops.quant import dequant_mxfp8
    cfg = small_gpu_config(num_hidden_layers=2)
    sd = init_weights(cfg, 0)
    save_checkpoint_fp8(sd, str(tmp_path), cfg, block=block, ue8m0=ue8m0)
    ecfg = EngineConfig(page_size=64, max_kv_pages=64, cuda_graphs=False)
    eng = load_engine(cfg, weights=str(tmp_path), ecfg=ecfg, device="cuda")
    w = eng.model.layers[0].attn.o_proj.w
    assert w.data.is_cuda
    from b200ds.models.loader import load_checkpoint
    ck = load_checkpoint(str(tmp_path))
    k = "model.layers.0.self_attn.o_proj.weight"
    from b200ds.ops.quant import dequant_blocked
    deq = dequant_blocked(ck[k], ck[k + "_scale_inv"])
    srv = dequant_mxfp8(w.data.cpu(), w.sf.cpu())[: cfg.hidden_size]
    assert _rel(srv, deq) < 0.03
    direct = Engine(build_model_from(cfg, ecfg, sd, device="cuda"), ecfg)
    g = torch.Generator().manual_seed(1)
    prompts = torch.randint(0, cfg.vocab_size, (2, 20), generator=g).tolist()
    a = eng.generate(prompts, SamplingParams(max_tokens=1, logprobs=0))
    b = direct.generate(prompts, SamplingParams(max_tokens=1, logprobs=0))
    # both are MXFP8 models of the same weights (one extra fp8 rounding step apart)
    for x, y in zip(a, b):
        assert abs(x.logprobs[0][1] - y.logprobs[0][1]) < 0.5


def _engine(graphs=True, **kw):
    """Engines whose tokens are compared run with bitwise-reproducible
    kernels (the router logits' split-K fp32 atomics sum in any order, which
    can flip a near-tie expert choice of a random-weight model)."""
    from b200ds import EngineConfig, build_model_from
    from b200ds.utils import levers
    levers.set_switch("deterministic", True)
    from b200ds.config import small_gpu_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.tokenizer import ByteTokenizer
    from b200ds.models.reference import init_weights
    cfg = small_gpu_config()
    ecfg = EngineConfig(page_size=64, max_kv_pages=kw.pop("max_kv_pages", 96), cuda_graphs=graphs,
                        graph_batch_sizes=(1, 2, 4), max_num_seqs=4, **kw)
    return Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cuda"), ecfg,
                  tokenizer=ByteTokenizer()), cfg


def test_logprobs_penalties_and_guided_decoding_on_the_gpu():
    """Steps with log-probabilities / logit adjustments / guides run the
    full-logits forward on the GPU while plain steps replay decode graphs:
    asking for log-probabilities does not change greedy tokens, the values
    are the log-softmax of the step's logits, penalties change the output,
    a guided output matches its pattern."""
    from b200ds.engine.request import SamplingParams
    eng, cfg = _engine()
    g = torch.Generator().manual_seed(8)
    prompts = torch.randint(0, cfg.vocab_size, (2, 30), generator=g).tolist()
    plain = [o.token_ids for o in eng.generate(prompts, SamplingParams(max_tokens=6))]
    outs = eng.generate(prompts, SamplingParams(max_tokens=6, logprobs=3))
    assert [o.token_ids for o in outs] == plain
    for o in outs:
        assert len(o.logprobs) == 6
        for t, lp, top in o.logprobs:
            assert lp <= 0.0 and top[0][0] == t and abs(top[0][1] - lp) < 1e-4
    base = list(range(3, 9)) * 4
    p0 = eng.generate([base], SamplingParams(max_tokens=16))[0].token_ids
    pen = eng.generate([base], SamplingParams(max_tokens=16, presence_penalty=3.0, frequency_penalty=3.0,
                                              repetition_penalty=2.0))[0].token_ids
    assert pen != p0
    forced = eng.generate([[5, 6, 7]], SamplingParams(max_tokens=3, logit_bias={42: 100.0}))[0].token_ids
    assert forced == [42] * 3
    tok = eng.tokenizer
    pat = r"[0-9]{3}-[a-z]{2}"
    o = eng.generate([tok.encode("id:")], SamplingParams(max_tokens=12, guided_regex=pat))[0]
    assert regex.fullmatch(pat, tok.decode(o.token_ids)) and o.finish_reason == "stop"


def test_host_kv_tier_on_the_gpu():
    """Evicted prefix-cache pages move to pinned host memory and come back on
    a match: the same tokens as an engine without the prefix cache."""
    from b200ds.engine.request import SamplingParams
    eng, cfg = _engine(graphs=False, enable_prefix_cache=True, host_kv_pages=32, max_kv_pages=8)
    ref, _ = _engine(graphs=False, enable_prefix_cache=False, max_kv_pages=8)
    g = torch.Generator().manual_seed(31)
    A = torch.randint(0, cfg.vocab_size, (130,), generator=g).tolist()
    others = [torch.randint(0, cfg.vocab_size, (130,), generator=g).tolist() for _ in range(3)]
    seq = [A] + others + [A + [3, 4]]
    # the first token's log-probability of every prompt, computed through the
    # host tier (the last prompt's prefix comes back from host memory) and
    # without a prefix cache: a wrong restored KV row would move it by O(1)
    sp = SamplingParams(max_tokens=1, logprobs=0)
    got = [eng.generate([p], sp)[0].logprobs[0] for p in seq]
    want = [ref.generate([p], sp)[0].logprobs[0] for p in seq]
    for (tg, lg, _), (tw, lw, _) in zip(got, want):
        assert abs(lg - lw) < 0.05, (got, want)
    gg = eng.gauges()
    assert gg["host_offloads"] > 0 and gg["host_restores"] > 0 and gg["prefix_hit_tokens"] >= 128


def test_tactics_tuner_writes_a_loadable_table(tmp_path):
    """benchmarks/kernels.py --tune measures every legal tactic of a decode
    shape and writes a table the engine loads (B200_TACTICS)."""
    out = tmp_path / "tactics.json"
    r = subprocess.run([sys.executable, os.path.join(ROOT, "benchmarks", "kernels.py"), "--tune", str(out),
                        "--tune-quick", "--iters", "3"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    table = json.loads(out.read_text())
    assert table["gemm_splits"] and table["mla_splits"]
    from b200ds.ops import tactics
    tactics.set_table(table)
    try:
        e = table["gemm_splits"][0]
        assert tactics.pick("gemm_splits", 1, N=e["N"], K=e["K"], rows=e["rows"], max_ctas=296) == e["value"]
    finally:
        tactics.set_table(None)
