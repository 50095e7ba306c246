"""In-place weight updates: after update_weights the engine produces what a
fresh engine on the new weights produces, every weight tensor keeps its
storage (captured graphs stay valid), and the prefix cache is cleared."""
import pytest
import torch

from b200ds.engine.request import SamplingParams


def _engine(sd, cfg, **kw):
    from b200ds import build_model_from
    from b200ds.config import EngineConfig
    from b200ds.engine.engine import Engine
    ecfg = EngineConfig(page_size=8, cuda_graphs=False, **kw)
    return Engine(build_model_from(cfg, ecfg, sd, device="cpu"), ecfg)


@pytest.mark.parametrize("v4", [False, True])
def test_update_weights_in_place(tmp_path, v4):
    from b200ds.config import tiny_config, tiny_v4_config
    from b200ds.models.reference import init_weights
    from b200ds.models.reference_v4 import init_weights_v4
    from b200ds.models.weights_update import weight_tensors
    cfg = tiny_v4_config() if v4 else tiny_config()
    init = init_weights_v4 if v4 else init_weights
    a, b = init(cfg, 0), init(cfg, 1)
    g = torch.Generator().manual_seed(4)
    prompts = torch.randint(0, cfg.vocab_size, (2, 17), generator=g).tolist()
    sp = SamplingParams(max_tokens=5)
    eng = _engine(a, cfg)
    before = [o.token_ids for o in eng.generate(prompts, sp)]
    assert eng.radix.num_nodes > 0
    ptrs = [t.data_ptr() for _, t in weight_tensors(eng.model)]
    n = eng.update_weights(b)
    assert n > 0 and eng.radix.num_nodes == 0
    assert [t.data_ptr() for _, t in weight_tensors(eng.model)] == ptrs
    after = [o.token_ids for o in eng.generate(prompts, sp)]
    want = [o.token_ids for o in _engine(b, cfg).generate(prompts, sp)]
    assert after == want and after != before
    eng.add_request(prompts[0], sp)
    with pytest.raises(ValueError):
        eng.update_weights(a)
