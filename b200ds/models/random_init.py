"""Random-init weights generated directly on the device, per rank."""
from __future__ import annotations


def should_generate_on_device(cfg, device) -> bool:
    return False


def build_random_model(cfg, ecfg, ps, device, seed):
    raise NotImplementedError
