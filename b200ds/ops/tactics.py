"""Kernel tactics as data.

A JSON table overrides the built-in per-shape choices of the CUDA op layer,
entry by entry; shapes it does not name keep the heuristics.

    {"gemm_splits": [{"N": 7168, "K": 16384, "rows": [1, 64], "value": 4}],
     "moe_tile":    [{"cap": 64, "rows_per_expert": [0, 8], "value": 32}],
     "mla_splits":  [{"H": 16, "rows": [1, 64], "keys": [0, 4096], "value": 2}]}

An int key must equal the call's value; a [lo, hi] key is an inclusive band.
The first matching entry wins.  Values outside a tactic's legal set (split-K
factors 1 / 2 / 4 / 8 with at least two k-tiles per split, at most 128 rows
and no more CTAs than the caller's cap; token tiles 16..128 up to the caller's cap; KV splits
1..16) are ignored with a one-time notice.  The table comes from the file
named by B200_TACTICS (read once); `benchmarks/kernels.py --tune` measures the
candidates on the GPU and writes one.

Reference parity: FMT / MOET / DT pin a measured tactic per weight shape and
row band (levers.py:30-35, 73-80, 480-484).
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Optional

_TABLE: Optional[Dict[str, List[dict]]] = None
_LEGAL = {
    "gemm_splits": lambda v, ctx: v in (1, 2, 4, 8) and (v == 1 or (
        ctx.get("rows", 0) <= 128 and ctx.get("K", 0) // 128 // v >= 2
        and ctx.get("N", 0) // 128 * v <= ctx.get("max_ctas", 1 << 30))),
    "moe_tile": lambda v, ctx: v in (16, 32, 64, 128) and v <= ctx.get("cap", 128),
    "moe_tile_fc1": lambda v, ctx: v in (16, 32, 64, 128),
    "moe_tile_fc2": lambda v, ctx: v in (16, 32, 64, 128),
    "mla_splits": lambda v, ctx: isinstance(v, int) and 1 <= v <= 16,
}


def load(path: Optional[str] = None) -> Dict[str, List[dict]]:
    """Read (or re-read) the table; {} when none is configured."""
    global _TABLE
    path = path if path is not None else os.environ.get("B200_TACTICS", "")
    if not path:
        _TABLE = {}
        return _TABLE
    with open(path) as f:
        t = json.load(f)
    if not isinstance(t, dict) or not all(isinstance(v, list) for v in t.values()):
        raise ValueError(f"tactics table {path}: expected {{op: [entries]}}")
    unknown = set(t) - set(_LEGAL)
    if unknown:
        raise ValueError(f"tactics table {path}: unknown ops {sorted(unknown)}")
    _TABLE = t
    return _TABLE


def set_table(table: Optional[Dict[str, List[dict]]]) -> None:
    """Install a table directly (None: back to the file / no table)."""
    global _TABLE
    _TABLE = table


def _match(entry: dict, ctx: dict) -> bool:
    for k, want in entry.items():
        if k == "value":
            continue
        if k not in ctx:
            return False
        v = ctx[k]
        if isinstance(want, (list, tuple)):
            if not (want[0] <= v <= want[1]):
                return False
        elif v != want:
            return False
    return True


def pick(op: str, default: int, **ctx) -> int:
    """The table's value for this call, else `default`.  ctx holds the call's
    shape (and limits such as max_ctas / cap, which entries may not name)."""
    table = _TABLE if _TABLE is not None else load()
    entries = table.get(op)
    if not entries:
        return default
    for e in entries:
        if _match(e, ctx):
            v = e.get("value")
            if _LEGAL[op](v, ctx):
                return int(v)
            from ..utils import levers
            levers.announce(f"tactic-illegal-{op}-{v}", f"tactics: {op} value {v} is not legal for {ctx}; "
                            "using the built-in choice")
            return default
    return default


def write(table: Dict[str, List[dict]], path: str) -> None:
    with open(path, "w") as f:
        json.dump(table, f, indent=1)
        f.write("\n")
