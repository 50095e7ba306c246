"""Step watchdog: a daemon thread that notices when one engine step runs
longer than a limit (a hung collective, a kernel that never finishes).

On expiry it dumps every thread's stack to stderr once, calls `on_expire`
(the server marks itself unhealthy; with `exit_code` set the process ends so
a supervisor can restart it), and keeps watching; a step that finishes after
all clears the stall.  The limit bounds the host side; device-side waits are
bounded in the kernels themselves and collectives by the process group's
timeout.

Reference parity: the reference's fail-closed design keeps a rank-local
failure from hanging its peers (fg.py RANKS section, ag.py:181-185); serving
stacks add a forward watchdog on top (SGLang's watchdog is absent here).
"""
from __future__ import annotations

import faulthandler
import os
import sys
import threading
import time
from contextlib import contextmanager
from typing import Callable, Optional


class Watchdog:
    def __init__(self, timeout_s: float, on_expire: Optional[Callable[[float], None]] = None,
                 exit_code: Optional[int] = None, poll_s: Optional[float] = None, dump: bool = True):
        self.timeout_s = float(timeout_s)
        self.on_expire = on_expire
        self.exit_code = exit_code
        self.poll_s = poll_s if poll_s is not None else max(0.01, min(1.0, self.timeout_s / 10))
        self.dump = dump
        self._armed_at: Optional[float] = None
        self._fired = False
        self.stalled = False
        self.expirations = 0
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, name="b200ds-watchdog", daemon=True)
        self._t.start()

    @contextmanager
    def guard(self):
        """Arm for the duration of one step."""
        with self._lock:
            self._armed_at, self._fired = time.monotonic(), False
        try:
            yield
        finally:
            with self._lock:
                self._armed_at = None
                self.stalled = False

    def _run(self) -> None:
        while not self._stop.wait(self.poll_s):
            with self._lock:
                t0, fired = self._armed_at, self._fired
                if t0 is None or fired:
                    continue
                elapsed = time.monotonic() - t0
                if elapsed < self.timeout_s:
                    continue
                self._fired, self.stalled = True, True
                self.expirations += 1
            print(f"[b200ds] watchdog: engine step running for {elapsed:.1f} s (limit {self.timeout_s:.1f} s)",
                  file=sys.stderr, flush=True)
            if self.dump:
                faulthandler.dump_traceback(file=sys.stderr, all_threads=True)
            if self.on_expire is not None:
                self.on_expire(elapsed)
            if self.exit_code is not None:
                os._exit(self.exit_code)

    def stop(self) -> None:
        self._stop.set()
        self._t.join(timeout=5)
