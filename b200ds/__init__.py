"""b200ds: a Blackwell-native (sm_100a) DeepSeek-V3-family inference engine.

Typical use (one process per GPU under torchrun, or a single process)::

    from b200ds import load_engine, SamplingParams
    eng = load_engine("deepseek-v3-671b", weights="random")      # or a checkpoint dir
    outs = eng.generate([[1, 2, 3]], SamplingParams(max_tokens=32))
"""
from __future__ import annotations

from typing import Optional, Union

import torch

from .config import PRESETS, EngineConfig, ModelConfig
from .engine.engine import Engine, GenerateOutput
from .engine.request import SamplingParams

__all__ = ["Engine", "EngineConfig", "ModelConfig", "SamplingParams", "GenerateOutput", "load_engine", "build_model_from"]


def build_model_from(cfg: ModelConfig, ecfg: EngineConfig, weights: Union[str, dict] = "random",
                     device=None, seed: int = 0, ps=None):
    """Build this rank's model (DeepseekModel, or DeepseekV4Model for
    arch="deepseek_v4").  ``weights`` is "random" (random init of the
    architecture), a checkpoint directory, or a full state dict."""
    from .parallel.state import get_state
    from .models import loader
    from .models.reference import init_weights
    ps = ps or get_state()
    if device is None:
        device = ps.device if ps.device.type == "cuda" else ("cuda" if torch.cuda.is_available() else "cpu")
    if cfg.is_v4:
        from .models.deepseek_v4 import build_model_v4
        from .models.reference_v4 import init_weights_v4
        if isinstance(weights, dict):
            sd = weights
        elif weights == "random":
            from .models import random_init
            if random_init.should_generate_on_device(cfg, device):
                return random_init.build_random_model_v4(cfg, ecfg, ps, device, seed)
            sd = init_weights_v4(cfg, seed=seed)
        else:
            sd = loader.load_checkpoint(weights)
        return build_model_v4(cfg, ecfg, ps, sd, device=device)
    if isinstance(weights, dict):
        sd = weights
    elif weights == "random":
        from .models import random_init
        if random_init.should_generate_on_device(cfg, device):
            return random_init.build_random_model(cfg, ecfg, ps, device, seed)
        sd = init_weights(cfg, seed=seed)
    else:
        sd = loader.load_checkpoint(weights)
    return loader.build_model(cfg, ecfg, ps, sd, device=device)


def load_engine(model: Union[str, ModelConfig] = "tiny", weights: Union[str, dict] = "random",
                ecfg: Optional[EngineConfig] = None, device=None, seed: int = 0, **cfg_over) -> Engine:
    """Create an Engine for a preset name / HF checkpoint dir / ModelConfig."""
    import os
    if isinstance(model, ModelConfig):
        cfg = model
    elif model in PRESETS:
        cfg = PRESETS[model](**cfg_over)
    elif os.path.isdir(model):
        cfg = ModelConfig.from_hf(os.path.join(model, "config.json"))
        if weights == "random":
            weights = model
    else:
        raise ValueError(f"unknown model {model!r}")
    ecfg = ecfg or EngineConfig()
    m = build_model_from(cfg, ecfg, weights, device=device, seed=seed)
    eos, tok = None, None
    if isinstance(model, str) and os.path.isdir(model):
        eos = _eos_id(model)
        from .engine.tokenizer import load_tokenizer
        tok = load_tokenizer(model)
        if eos is None:
            eos = getattr(tok, "eos_token_id", None)
    return Engine(m, ecfg, eos_token_id=eos, tokenizer=tok)


def _eos_id(path: str):
    """End-of-sequence id of a checkpoint directory: generation_config.json,
    else config.json (the first id when a list is given)."""
    import json
    import os
    for f in ("generation_config.json", "config.json"):
        p = os.path.join(path, f)
        if os.path.exists(p):
            with open(p) as fh:
                v = json.load(fh).get("eos_token_id")
            if v is not None:
                return int(v[0] if isinstance(v, list) else v)
    return None
