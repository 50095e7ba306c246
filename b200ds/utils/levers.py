"""Switch registry, one-shot announcements and fail-closed self-checks.

Every optional fast path of the engine is a named switch here (default on,
overridable by its environment variable), so a run can state which paths it
used and turn any of them off for comparison.  `selfcheck()` runs each
registered check once (the fast path against its reference on a small
input); the verdicts are agreed over the CPU process group with MIN, so a
path that fails on any rank is turned off on every rank and all ranks keep
running the same kernels in the same order.

Reference parity: levers.py:1-589 (switches), levers.py:594-603 (`announce`,
`first`), route_e5.py:529-555 / fin.py:955-963 (first-use checks agreed over
the TP CPU group with gloo MIN, fail-closed).
"""
from __future__ import annotations

import os
import sys
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional


@dataclass
class Switch:
    name: str
    env: str
    default: bool
    doc: str
    value: Optional[bool] = None
    checks: List[Callable[[], bool]] = field(default_factory=list)

    def on(self) -> bool:
        if self.value is None:
            v = os.environ.get(self.env)
            self.value = self.default if v is None else v not in ("0", "false", "False", "")
        return self.value


_REGISTRY: Dict[str, Switch] = {}
_ANNOUNCED: set = set()


def register(name: str, env: str, default: bool, doc: str) -> Switch:
    sw = _REGISTRY.get(name)
    if sw is None:
        sw = _REGISTRY[name] = Switch(name, env, default, doc)
    return sw


def on(name: str) -> bool:
    return _REGISTRY[name].on()


def set_switch(name: str, value: bool) -> None:
    _REGISTRY[name].value = bool(value)


def switches() -> Dict[str, bool]:
    """Current value of every switch (for the bench / server reports)."""
    return {k: s.on() for k, s in sorted(_REGISTRY.items())}


def announce(key: str, msg: str, stream=None) -> bool:
    """Print msg once per key (rank 0 only); returns True the first time."""
    if key in _ANNOUNCED:
        return False
    _ANNOUNCED.add(key)
    if os.environ.get("RANK", "0") == "0":
        print(f"[b200ds] {msg}", file=stream or sys.stderr, flush=True)
    return True


def add_check(name: str, fn: Callable[[], bool]) -> None:
    """Register a self-check of switch `name`: fn() runs the fast path and
    its reference on a small input and returns True when they agree."""
    _REGISTRY[name].checks.append(fn)


def agree_min(values: List[int], group=None) -> List[int]:
    """Elementwise MIN over the ranks of `group` (a gloo CPU group); no group
    (a single-rank parallel state, e.g. a one-GPU model inside a multi-rank
    job) keeps the values local."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.int64)
    if group is not None and dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return [int(v) for v in t.tolist()]


def selfcheck(group=None) -> Dict[str, bool]:
    """Run every registered check of every switch that is on; a switch
    whose check fails (or raises) on any rank is turned off on all ranks.
    Every rank runs the same checks in the same order."""
    names = [n for n in sorted(_REGISTRY) if _REGISTRY[n].on() and _REGISTRY[n].checks]
    local = []
    for n in names:
        ok = True
        for fn in _REGISTRY[n].checks:
            try:
                ok = ok and bool(fn())
            except Exception as e:  # a failing check disables its path, it does not end the run
                announce(f"check-error-{n}", f"self-check of {n} raised {type(e).__name__}: {e}")
                ok = False
        local.append(1 if ok else 0)
    agreed = agree_min(local, group) if names else []
    out = {}
    for n, v in zip(names, agreed):
        if not v:
            set_switch(n, False)
            announce(f"off-{n}", f"{n}: self-check failed on a rank; path turned off on every rank")
        out[n] = bool(v)
    return out


# ---------------------------------------------------------------------------
# the engine's switches
# ---------------------------------------------------------------------------
register("moe_fused", "B200_MOE_FUSED", True,
         "routed experts: FC1 + FC2 in one persistent launch when both use the same token tile")
register("moe_pull", "B200_MOE_PULL", True,
         "fused experts read FC1 rows in place (activations / EP dispatch buffer) instead of a sorted copy")
register("fused_comm", "B200_FUSED_COMM", True,
         "device-initiated NVLink collectives fused into the producing / consuming kernels")
register("nvls", "B200_NVLS", True,
         "tensor-parallel all-reduces through NVLink multicast (multimem.ld_reduce / multimem.st in the switch) on "
         "groups of B200_NVLS_MIN_WORLD or more ranks with multicast support (default 16: off on one 8-GPU "
         "box, where it measured slower than the push protocol and NCCL)")
register("dp_moe_a2a", "B200_DP_MOE_A2A", True,
         "DP-attention steps too large for the fused dispatch buffers exchange MoE rows all-to-all (each row to its "
         "experts' owners only) instead of all-gather + reduce-scatter; rows per rank >= B200_DP_A2A_MIN_ROWS "
         "(default 64), never inside a graph capture")
register("l2_prefetch", "B200_L2_PREFETCH", True,
         "decode layers pull the o-projection (and shared-expert) weights into L2 on a low-priority side stream "
         "while attention runs")
register("ep_combine_epilogue", "B200_EP_COMBINE_EPILOGUE", True,
         "expert parallelism: the experts' FC2 epilogue stores each weighted pair row straight into its token's "
         "owner rank (no separate combine kernel, no local round trip of the FC2 rows)")
register("ep_peer_pull", "B200_EP_PEER_PULL", False,
         "expert parallelism: routed rows stay on their source rank and the fused expert kernel's producer warps read "
         "them over NVLink (only ids / weights are pushed); off: the dispatch stores each row into its owners' "
         "regions")
register("ar_one_kernel", "B200_AR_ONE_KERNEL", True,
         "push-mode all-reduces (and the TP MoE combine) run push + per-CTA arrivals + reduce + norm as one kernel "
         "instead of a push kernel and a reduce kernel")
register("nvls_one_kernel", "B200_NVLS_ONE_KERNEL", False,
         "NVLS groups: one kernel per all-reduce - each CTA's rows stored locally, summed through the switch by "
         "rank c % world and broadcast back, per-CTA flags (off: push kernel + NVLS reduce kernel)")
register("hc_boundary", "B200_HC_BOUNDARY", True,
         "V4 family, decode-sized batches: hc_post + the mHC mixes (fp32, CUDA cores) + coefficients + the next "
         "sublayer's normed input as one kernel, a thread-block cluster per row")
register("deterministic", "B200_DETERMINISTIC", False,
         "bitwise-reproducible steps: split-K GEMMs that sum with fp32 atomics (router logits, mHC stats) run "
         "unsplit")
