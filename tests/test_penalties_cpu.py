"""Per-request logit adjustments (repetition / presence / frequency
penalties, min_tokens, min_p): each against its definition on a logits row,
and end to end through the engine."""
import torch

from b200ds.engine.request import Request, SamplingParams


def _req(prompt, output, **kw):
    r = Request(0, list(prompt), SamplingParams(**kw))
    r.output = list(output)
    return r


def test_adjustments_follow_their_definitions():
    from b200ds.engine.penalties import MASKED, adjust_logits
    V = 10
    g = torch.Generator().manual_seed(0)
    lg = torch.randn(1, V, generator=g) * 3
    # repetition: prompt/output tokens, sign-dependent
    r = _req([1, 2], [2, 5], repetition_penalty=2.0)
    out = adjust_logits(lg, [r])[0]
    for t in range(V):
        want = lg[0, t] if t not in (1, 2, 5) else (lg[0, t] / 2 if lg[0, t] > 0 else lg[0, t] * 2)
        assert torch.isclose(out[t], want)
    # presence + frequency over the output only
    r = _req([3], [4, 4, 6], presence_penalty=0.5, frequency_penalty=0.25)
    out = adjust_logits(lg, [r])[0]
    assert torch.isclose(out[4], lg[0, 4] - 0.5 - 0.5) and torch.isclose(out[6], lg[0, 6] - 0.75)
    assert torch.isclose(out[3], lg[0, 3]) and torch.isclose(out[0], lg[0, 0])
    # min_tokens masks eos and stop ids while the output is short
    r = _req([1], [7], min_tokens=2, stop_token_ids=[3])
    out = adjust_logits(lg, [r], eos=9)[0]
    assert out[9] == MASKED and out[3] == MASKED and torch.isclose(out[0], lg[0, 0])
    r.output = [7, 8]
    assert torch.equal(adjust_logits(lg, [r], eos=9)[0], lg[0])
    # min_p on the temperature-scaled distribution; greedy rows untouched
    r = _req([1], [], min_p=0.2, temperature=0.7)
    out = adjust_logits(lg, [r])[0]
    pr = (lg[0] / 0.7).softmax(-1)
    assert torch.equal(out == MASKED, pr < 0.2 * pr.max())
    assert torch.equal(adjust_logits(lg, [_req([1], [], min_p=0.2)])[0], lg[0])
    # rows that do not sample are left alone
    assert torch.equal(adjust_logits(lg, [_req([1], [2], presence_penalty=1.0)], sample=[False])[0], lg[0])


def _engine():
    from b200ds import build_model_from
    from b200ds.config import EngineConfig, tiny_config
    from b200ds.engine.engine import Engine
    from b200ds.models.reference import init_weights
    cfg = tiny_config()
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, enable_prefix_cache=False)
    return Engine(build_model_from(cfg, ecfg, init_weights(cfg, 0), device="cpu"), ecfg)


def test_engine_presence_penalty_and_min_tokens():
    eng = _engine()
    base = list(range(3, 9)) * 3
    plain = eng.generate([base], SamplingParams(max_tokens=24))[0].token_ids
    assert len(set(plain)) < len(plain)              # the tiny model repeats itself greedily
    pen = eng.generate([base], SamplingParams(max_tokens=24, presence_penalty=2.0, frequency_penalty=2.0,
                                              repetition_penalty=1.5))[0].token_ids
    assert pen != plain and len(set(pen)) > len(set(plain))
    # an end-of-sequence id the model emits early is held back until min_tokens
    eng.eos = plain[2]
    early = eng.generate([base], SamplingParams(max_tokens=24))[0]
    assert early.finish_reason == "stop" and len(early.token_ids) == 3
    held = eng.generate([base], SamplingParams(max_tokens=24, min_tokens=6))[0]
    assert plain[2] not in held.token_ids[:5] and len(held.token_ids) >= 6
    # penalties + spec decoding: adjusted requests decode one token per step, same tokens
    from b200ds.config import EngineConfig
    eng.eos = None
    eng.ecfg.spec_ngram = 3
    again = eng.generate([base], SamplingParams(max_tokens=24, presence_penalty=2.0, frequency_penalty=2.0,
                                                repetition_penalty=1.5))[0].token_ids
    assert again == pen


def test_logit_bias():
    from b200ds.engine.penalties import adjust_logits
    lg = torch.zeros(1, 10)
    out = adjust_logits(lg, [_req([1], [], logit_bias={3: 5.0, 7: -100.0})])[0]
    assert out[3] == 5.0 and out[7] == -100.0 and out[0] == 0.0
    eng = _engine()
    forced = eng.generate([[5, 6, 7]], SamplingParams(max_tokens=4, logit_bias={42: 100.0}))[0].token_ids
    assert forced == [42] * 4
