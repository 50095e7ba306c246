"""Eager collectives used by the model.

``all_reduce`` is the plain NCCL all-reduce over the tensor-parallel group:
the baseline path, and the eager path for prefill chunks larger than the
fused kernels' symmetric slots.  The fused NVLink kernels (GEMM-epilogue
push, combine + all-reduce + norm) are called from `b200ds.ops.cuda` through
`b200ds.parallel.symm`, not from here.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def all_reduce(x: torch.Tensor, ps) -> torch.Tensor:
    if ps.tp_size <= 1:
        return x
    dist.all_reduce(x, group=ps.tp_group)
    return x
