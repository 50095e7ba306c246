"""Continuous-batching scheduler with chunked prefill, radix prefix reuse and
preemption by recompute.

Each step is either a prefill step (waiting requests admitted under a token
budget; a prompt longer than the budget is split into chunks) or a decode
step (one token for every running request).  The schedule depends only on
the request stream, so every rank of an SPMD job computes the same batches.

Reference parity: scheduling is SGLang's (absent); the reference tunes the
chunked-prefill size 16384 (levers.py:14).
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from typing import Deque, List, Optional

from ..kv.pool import OutOfPages, PagePool
from ..kv.radix import RadixCache
from .request import Request


@dataclass
class Step:
    kind: str                      # "prefill" | "decode"
    reqs: List[Request]
    chunks: List[List[int]]        # new tokens per request
    starts: List[int]              # cached length before the step
    sample: List[bool]             # whether the step's last logits produce a token
    decode_rows: int = 0           # mixed prefill step: its last rows are running requests' decode tokens


def prefill_target(r: Request) -> int:
    """Tokens that must be cached before decoding resumes.  A preempted
    request re-caches everything except its newest token (the next decode
    input)."""
    return len(r.prompt) if not r.output else r.total_len - 1


LPM_MAX_QUEUE = 128


class Scheduler:
    def __init__(self, pool: PagePool, max_num_seqs: int, max_prefill_tokens: int,
                 radix: Optional[RadixCache] = None, mixed: bool = False, policy: str = "fcfs"):
        if policy not in ("fcfs", "lpm", "priority"):
            raise ValueError(f"schedule policy {policy!r}: fcfs, lpm or priority")
        self.pool = pool
        # lpm: admit the waiting requests with the longest cached prefix first
        # (more prefix-cache hits before those pages are evicted); arrival
        # order breaks ties, and queues longer than LPM_MAX_QUEUE stay FCFS.
        # priority: lower SamplingParams.priority first, arrival order within
        # a level (admission only: running requests are not preempted for it)
        self.policy = policy
        # mixed = True: a prefill step also carries one decode token of every
        # running request, so decoding does not stall behind long prompts
        self.mixed = mixed
        self.radix = radix
        self.max_num_seqs = max_num_seqs
        self.max_prefill_tokens = max_prefill_tokens
        self.waiting: Deque[Request] = deque()
        # counters for the metrics endpoint
        self.admitted_prompt_tokens = 0         # tokens to cache at admission (prompts, recomputes)
        self.prefix_hit_tokens = 0              # of those, found in the prefix cache
        self.preemptions = 0
        self.prefilling: List[Request] = []      # admitted, prompt not fully cached
        self.running: List[Request] = []

    def add(self, r: Request) -> None:
        self.waiting.append(r)

    @property
    def has_work(self) -> bool:
        return bool(self.waiting or self.prefilling or self.running)

    # ------------------------------------------------------------------
    def _ensure_pages(self, r: Request, upto_tokens: int) -> bool:
        need = self.pool.pages_for(upto_tokens) - len(r.pages)
        if need <= 0:
            return True
        if self.pool.num_free < need and self.radix is not None:
            self.radix.evict(need - self.pool.num_free)
        if self.pool.num_free < need:
            return False
        r.pages.extend(self.pool.alloc(need))
        return True

    def _admit(self, r: Request) -> None:
        if self.radix is not None and not r.pages and r.params.prompt_logprobs is None:
            # leave at least one token to compute so the step yields logits
            pages, nodes = self.radix.match(r.all_tokens[: prefill_target(r) - 1] if r.output
                                            else r.prompt[:-1])
            r.pages = list(pages)
            r.prefix_nodes = nodes
            r.prefix_pages = len(pages)
            r.cached = len(pages) * self.pool.page_size
        self.admitted_prompt_tokens += prefill_target(r)
        self.prefix_hit_tokens += r.cached

    def release(self, r: Request, cache_prefix: bool = True) -> None:
        if self.radix is not None and cache_prefix:
            full = r.cached // self.pool.page_size
            self.radix.insert(r.all_tokens[: full * self.pool.page_size], r.pages[:full])
        if self.radix is not None and r.prefix_nodes:
            self.radix.unlock(r.prefix_nodes)
        self.pool.release(r.pages[r.prefix_pages:])
        r.pages, r.prefix_nodes, r.prefix_pages = [], [], 0

    def _preempt(self) -> bool:
        """Free the most recently admitted running request (recompute later)."""
        if not self.running:
            return False
        v = self.running.pop()
        self.preemptions += 1
        self.release(v)
        v.cached = 0
        self.waiting.appendleft(v)
        return True

    # ------------------------------------------------------------------
    def next_step(self) -> Optional[Step]:
        budget = self.max_prefill_tokens
        if self.mixed and self.running:
            # the running requests' decode tokens ride along: reserve them
            budget = max(1, budget - len(self.running))
        if self.prefilling or (self.waiting and len(self.running) + len(self.prefilling) < self.max_num_seqs):
            reqs, chunks, starts, sample = [], [], [], []
            cands = list(self.prefilling)
            self.prefilling = []
            if self.policy == "lpm" and self.radix is not None and 1 < len(self.waiting) <= LPM_MAX_QUEUE:
                order = sorted(self.waiting, key=lambda r: -self.radix.match_len(
                    r.all_tokens[: prefill_target(r) - 1] if r.output else r.prompt[:-1]))
                self.waiting = deque(order)
            elif self.policy == "priority" and len(self.waiting) > 1:
                self.waiting = deque(sorted(self.waiting, key=lambda r: r.params.priority))
            while self.waiting and len(self.running) + len(cands) < self.max_num_seqs:
                r = self.waiting.popleft()
                self._admit(r)
                cands.append(r)
            for r in cands:
                target = prefill_target(r)
                if budget <= 0:
                    self.prefilling.append(r)
                    continue
                n = min(target - r.cached, budget)
                if not self._ensure_pages(r, r.cached + n):
                    if len(r.pages) == r.prefix_pages:
                        self.release(r, cache_prefix=False)
                        r.cached = 0
                        self.waiting.appendleft(r)
                    else:
                        self.prefilling.append(r)
                    continue
                toks = r.all_tokens
                reqs.append(r)
                chunks.append(toks[r.cached:r.cached + n])
                starts.append(r.cached)
                sample.append(r.cached + n == target and not r.output)
                budget -= n
            if reqs:
                nd = 0
                if self.mixed:
                    for r in self.running:
                        if not self._ensure_pages(r, r.cached + 1):
                            continue
                        reqs.append(r)
                        chunks.append([r.all_tokens[r.cached]])
                        starts.append(r.cached)
                        sample.append(True)
                        budget -= 1
                        nd += 1
                return Step("prefill", reqs, chunks, starts, sample, decode_rows=nd)
        if not self.running:
            if self.has_work:
                raise OutOfPages("no request fits in the KV pool")
            return None
        while True:
            ok = True
            for r in self.running:
                if not self._ensure_pages(r, r.cached + 1):
                    ok = False
                    break
            if ok:
                break
            if not self._preempt():
                raise OutOfPages("cannot fit a single decode step")
        reqs = list(self.running)
        return Step("decode", reqs, [[r.all_tokens[r.cached]] for r in reqs],
                    [r.cached for r in reqs], [True] * len(reqs))

    def commit(self, step: Step) -> None:
        """Advance cached lengths after the forward ran."""
        n_pre = len(step.reqs) - step.decode_rows
        for i, (r, ch) in enumerate(zip(step.reqs, step.chunks)):
            r.cached += len(ch)
            if step.kind == "prefill" and i < n_pre:
                if r.cached >= prefill_target(r):
                    self.running.append(r)
                else:
                    self.prefilling.append(r)

    def abort(self, r: Request) -> None:
        """Drop a request wherever it is (waiting, mid-prefill, running) and
        free its pages (fully computed pages still enter the prefix cache)."""
        for lst in (self.running, self.prefilling):
            if r in lst:
                lst.remove(r)
        if r in self.waiting:
            self.waiting.remove(r)
        if r.pages:
            self.release(r)

    def finish(self, r: Request) -> None:
        if r in self.running:
            self.running.remove(r)
        self.release(r)
