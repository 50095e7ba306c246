"""Process-group topology: tensor-parallel attention, expert-parallel MoE,
data-parallel attention.

One process per GPU.  `ParallelState` owns the torch.distributed groups the
model uses:

* ``tp``  – attention / dense-FFN tensor parallel group (heads and FFN
  columns split, all-reduce after the row-parallel projection);
* ``ep``  – expert parallel group (routed experts split evenly);
* ``dp``  – data-parallel attention (each rank serves its own requests; the
  MoE boundary all-gathers tokens and reduce-scatters them back);
* ``cpu`` – a gloo group over the same ranks for host-side agreement
  (scheduler decisions, failure votes).

Reference parity: the reference runs inside SGLang's GroupCoordinator
(ar.py:1-22, fork_loop.py:86-100) with TP2 and a gloo CPU group
(route_e5.py:529-537).  Here the topology is explicit and testable on CPU
with gloo.
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


@dataclass
class ParallelState:
    world_size: int = 1
    rank: int = 0
    tp_size: int = 1
    tp_rank: int = 0
    ep_size: int = 1
    ep_rank: int = 0
    dp_size: int = 1
    dp_rank: int = 0
    tp_group: Optional[object] = None
    ep_group: Optional[object] = None
    dp_group: Optional[object] = None
    cpu_group: Optional[object] = None
    device: torch.device = torch.device("cpu")
    fused_ar: Optional[object] = None       # parallel.symm.FusedAllReduce when enabled
    fused_ep: Optional[object] = None       # parallel.symm.EPDispatch (DP attention + EP)

    @property
    def distributed(self) -> bool:
        return self.world_size > 1

    # --- collectives used by the torch (baseline / CPU) path -----------------
    def tp_all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.tp_size > 1:
            dist.all_reduce(x, group=self.tp_group)
        return x

    def ep_all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.ep_size > 1:
            dist.all_reduce(x, group=self.ep_group)
        return x

    def ep_all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """[T, ...] per rank -> [ep_size * T, ...] in rank order."""
        if self.ep_size == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.ep_size)]
        dist.all_gather(parts, x.contiguous(), group=self.ep_group)
        return torch.cat(parts, 0)

    def tp_all_gather(self, x: torch.Tensor, dim: int = -1) -> torch.Tensor:
        if self.tp_size == 1:
            return x
        parts = [torch.empty_like(x) for _ in range(self.tp_size)]
        dist.all_gather(parts, x.contiguous(), group=self.tp_group)
        return torch.cat(parts, dim=dim)

    def cpu_min(self, value: int) -> int:
        """Agree on the minimum of an integer over all ranks (host only)."""
        if self.world_size == 1:
            return value
        t = torch.tensor([value], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.cpu_group)
        return int(t.item())


_STATE: Optional[ParallelState] = None


def get_state() -> ParallelState:
    global _STATE
    if _STATE is None:
        _STATE = ParallelState()
    return _STATE


def set_state(s: ParallelState) -> None:
    global _STATE
    _STATE = s


def init_parallel(tp_size: Optional[int] = None, ep_size: Optional[int] = None,
                  dp_attention: bool = False, backend: Optional[str] = None,
                  timeout_s: float = 120.0) -> ParallelState:
    """Initialise torch.distributed from the torchrun environment and build
    the groups.  With WORLD_SIZE unset this returns a single-rank state.

    tp_size defaults to world_size (or 1 with dp_attention); ep_size defaults
    to world_size.  Groups are built on every rank in the same order.
    """
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    device = torch.device("cuda", local_rank) if backend == "nccl" else torch.device("cpu")
    if backend == "nccl":
        torch.cuda.set_device(device)
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        kw = dict(backend=backend, world_size=world, rank=rank,
                  timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = device
        dist.init_process_group(**kw)
    if tp_size is None:
        tp_size = 1 if dp_attention else world
    if ep_size is None:
        ep_size = world
    assert world % tp_size == 0 and world % ep_size == 0, (world, tp_size, ep_size)
    st = ParallelState(world_size=world, rank=rank, tp_size=tp_size, ep_size=ep_size,
                       dp_size=world // tp_size, device=device)
    if world > 1:
        ranks = list(range(world))
        # TP groups: consecutive blocks of tp_size; DP groups: strided.
        for g in range(world // tp_size):
            r = ranks[g * tp_size:(g + 1) * tp_size]
            grp = dist.new_group(r)
            if rank in r:
                st.tp_group, st.tp_rank = grp, r.index(rank)
        for g in range(world // ep_size):
            r = ranks[g * ep_size:(g + 1) * ep_size]
            grp = dist.new_group(r)
            if rank in r:
                st.ep_group, st.ep_rank = grp, r.index(rank)
        for g in range(tp_size):
            r = ranks[g::tp_size]
            grp = dist.new_group(r)
            if rank in r:
                st.dp_group, st.dp_rank = grp, r.index(rank)
        st.cpu_group = dist.new_group(ranks, backend="gloo") if backend != "gloo" else dist.group.WORLD
    set_state(st)
    return st


def shutdown_parallel() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
    set_state(ParallelState())
