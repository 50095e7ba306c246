"""Step tracing: device timestamps at phase boundaries, usable inside CUDA
graphs, plus optional NVTX ranges.

`Tracer.mark(name)` launches a one-thread kernel that writes %globaltimer
into the next slot of a device buffer once the previous kernel in the stream
has completed; names are recorded on the host in launch order.  Marks issued
while a decode graph is captured are replayed with it, so every replay
refreshes the same slots: `report()` after a replay gives the device time of
each phase of that step (all ranks run the same marks; take the max over
ranks for a collective phase).  With tracing off, `mark` does nothing.

Enable with `B200_TRACE=1` (or `EngineConfig.trace`); `B200_NVTX=1` also
opens NVTX ranges named after the marks for external profilers.

Reference parity: route_e5.cu:350-358 / 1050-1056 (%clock64 / %globaltimer
phase stamps written by the leader thread into a `clocks` buffer).
"""
from __future__ import annotations

import os
from typing import Dict, List, Optional, Tuple

import torch


class Tracer:
    def __init__(self, device, capacity: int = 4096, enabled: Optional[bool] = None):
        self.enabled = bool(int(os.environ.get("B200_TRACE", "0"))) if enabled is None else enabled
        self.nvtx = bool(int(os.environ.get("B200_NVTX", "0")))
        self.device = torch.device(device)
        self.capacity = capacity
        self.names: List[str] = []
        self.buf = None
        self._open = False
        if self.enabled and self.device.type == "cuda":
            self.buf = torch.zeros(capacity, dtype=torch.int64, device=self.device)

    def reset(self) -> None:
        """Start a new timeline (call before the marks of one step)."""
        self.names = []
        if self._open:
            torch.cuda.nvtx.range_pop()
            self._open = False

    def mark(self, name: str) -> None:
        if not self.enabled:
            return
        if self.nvtx and self.device.type == "cuda":
            if self._open:
                torch.cuda.nvtx.range_pop()
            torch.cuda.nvtx.range_push(name)
            self._open = True
        idx = len(self.names)
        if idx >= self.capacity:
            return
        self.names.append(name)
        if self.buf is not None:
            from .. import _C
            _C.trace_stamp(self.buf, idx)

    def stamps(self) -> List[int]:
        if self.buf is None:
            return []
        torch.cuda.synchronize(self.device)
        return self.buf[: len(self.names)].tolist()

    def report(self, stamps: Optional[List[int]] = None) -> List[Tuple[str, float]]:
        """[(phase, microseconds)]: phase i spans mark i -> mark i + 1."""
        st = self.stamps() if stamps is None else stamps
        return [(self.names[i], (st[i + 1] - st[i]) / 1e3) for i in range(min(len(st), len(self.names)) - 1)]

    def summary(self, stamps: Optional[List[int]] = None) -> Dict[str, float]:
        """Microseconds per phase kind (the mark name before the first '.')."""
        out: Dict[str, float] = {}
        for name, us in self.report(stamps):
            k = name.split(".", 1)[1] if "." in name else name
            out[k] = out.get(k, 0.0) + us
        return out


_NULL = Tracer("cpu", enabled=False)


def null_tracer() -> Tracer:
    return _NULL
