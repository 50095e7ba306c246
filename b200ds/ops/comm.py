"""Collectives used by the model.

``all_reduce`` runs the fused NVLink kernels when the symmetric workspace is
set up (see b200ds.parallel.symm) and NCCL otherwise (the baseline path).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def all_reduce(x: torch.Tensor, ps) -> torch.Tensor:
    if ps.tp_size <= 1:
        return x
    dist.all_reduce(x, group=ps.tp_group)
    return x
