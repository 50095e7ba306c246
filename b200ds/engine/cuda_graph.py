"""CUDA-graph capture and replay of the decode step, one graph per padded
batch size.

Static device buffers hold the step's metadata (token ids, positions, KV
slots, block table, sequence lengths).  Each replay: the host fills pinned
staging buffers, one async copy per buffer moves them to the device, the
graph replays the whole forward (all layers, collectives included) plus
greedy argmax, and the sampled ids come back to the host.  Padded rows use
the reserved scratch page 0 so they never touch live KV.

Capture verdicts are agreed over the CPU process group (`capture_agreed`):
a graph is kept only if every rank recorded its own, else every rank drops
it and runs that forward eagerly, so ranks never split between graph replay
and eager launches.

Reference parity: decode/verify forwards are captured by SGLang's graph
runner (absent); the reference adds per-bucket eager graphs (fg.py, ag.py)
whose capture failures are agreed over the TP CPU group so every rank falls
back together (fg.py:1890-1900, ag.py:2309-2320).
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional

import torch

from ..models.batch import ForwardBatch


class _Graph:
    pass


class GraphCaptureFailed(RuntimeError):
    """A capture failed on at least one rank; every rank runs eagerly."""


def capture_agreed(record: Callable[[], object], group=None, what: str = "graph"):
    """Run `record()` (one graph capture) and agree on its verdict over the
    CPU group with MIN.  Returns record()'s result when every rank succeeded;
    otherwise raises GraphCaptureFailed on every rank.

    A capture records kernels and collectives without executing them, so a
    rank whose capture failed has run nothing its peers did not: after the
    agreement all ranks take the same path (replay or eager) and issue the
    same collectives in the same order.  Warm-up forwards, which do execute
    collectives, run before this on every rank."""
    from ..utils import levers
    try:
        out, ok, err = record(), 1, ""
    except Exception as e:      # any local failure is agreed, never raised alone
        out, ok, err = None, 0, f"{type(e).__name__}: {e}"
    if levers.agree_min([ok], group)[0]:
        return out
    raise GraphCaptureFailed(f"{what} capture failed on a rank" + (f" (here: {err})" if err else ""))


class DecodeGraphRunner:
    def __init__(self, engine, batch_sizes=None, max_pages: Optional[int] = None):
        self.eng = engine
        self.model = engine.model
        self.dev = engine.device
        ecfg = engine.ecfg
        self.page_size = ecfg.page_size
        self.batch_sizes = sorted(batch_sizes or [b for b in ecfg.graph_batch_sizes if b <= ecfg.max_num_seqs])
        if not self.batch_sizes or self.batch_sizes[-1] < ecfg.max_num_seqs:
            self.batch_sizes.append(ecfg.max_num_seqs)
        self.max_pages = max_pages or (ecfg.max_model_len + self.page_size - 1) // self.page_size
        self.graphs: Dict[int, _Graph] = {}
        self.pool = None
        self.enabled = True
        self.group = getattr(engine.ps, "cpu_group", None)

    def can_run(self, n: int) -> bool:
        return self.enabled and n <= self.batch_sizes[-1]

    def _bucket(self, n: int) -> int:
        for b in self.batch_sizes:
            if b >= n:
                return b
        raise ValueError(n)

    def _make_static(self, bs: int) -> _Graph:
        g = _Graph()
        d = self.dev
        g.bs = bs
        g.ids = torch.zeros(bs, dtype=torch.int32, device=d)
        g.pos = torch.zeros(bs, dtype=torch.int32, device=d)
        g.q_seq = torch.arange(bs, dtype=torch.int32, device=d)
        g.slots = torch.zeros(bs, dtype=torch.int64, device=d)
        g.lens = torch.ones(bs, dtype=torch.int32, device=d)
        g.bt = torch.zeros(bs, self.max_pages, dtype=torch.int32, device=d)
        g.last = torch.arange(bs, dtype=torch.int64, device=d)
        # pinned host staging
        g.h_ids = torch.zeros(bs, dtype=torch.int32).pin_memory()
        g.h_pos = torch.zeros(bs, dtype=torch.int32).pin_memory()
        g.h_slots = torch.zeros(bs, dtype=torch.int64).pin_memory()
        g.h_lens = torch.ones(bs, dtype=torch.int32).pin_memory()
        g.h_bt = torch.zeros(bs, self.max_pages, dtype=torch.int32).pin_memory()
        g.h_tok = torch.zeros(bs, dtype=torch.int64).pin_memory()
        # per-row sampling parameters (padding rows: greedy)
        g.samp = torch.zeros(4, bs, dtype=torch.float32, device=d)     # temperature, top_p, top_k, uniform
        g.samp[1].fill_(1.0)
        g.temp, g.top_p, g.unif = g.samp[0], g.samp[1], g.samp[3]
        g.top_k = torch.zeros(bs, dtype=torch.int32, device=d)
        g.h_samp = torch.zeros(4, bs, dtype=torch.float32).pin_memory()
        g.fb = ForwardBatch(input_ids=g.ids, positions=g.pos, q_seq=g.q_seq, out_slots=g.slots, seq_lens=g.lens,
                            block_table=g.bt, last_idx=g.last, is_decode=True, max_q_len=1,
                            max_seq_len=self.max_pages * self.page_size, dp_tmax=bs)
        return g

    def capture(self, bs: int) -> _Graph:
        g = self._make_static(bs)
        # the main chain is captured from a high-priority stream (its kernel
        # nodes keep the priority): side-stream prefetches yield to it
        s = torch.cuda.Stream(device=self.dev, priority=-2)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.forward_tokens(g.fb, g.temp, g.top_p, g.top_k, g.unif)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)

        def record():
            # keep_graph: the raw graph stays queryable (kernel-node census)
            g.graph = torch.cuda.CUDAGraph(keep_graph=True)
            if self.pool is None:
                self.pool = torch.cuda.graph_pool_handle()
            with torch.cuda.graph(g.graph, pool=self.pool):
                g.tokens = self.model.forward_tokens(g.fb, g.temp, g.top_p, g.top_k, g.unif)
            g.graph.instantiate()
        capture_agreed(record, self.group, f"decode graph (batch {bs})")
        tr = getattr(self.model, "tracer", None)
        g.trace_names = list(tr.names) if tr is not None and tr.enabled else []
        self.graphs[bs] = g
        return g

    def capture_all(self) -> None:
        for bs in reversed(self.batch_sizes):
            if bs not in self.graphs:
                self.capture(bs)

    def stage(self, g: _Graph, seqs: List[dict]) -> None:
        """Fill the pinned staging buffers for this step and copy them."""
        n = len(seqs)
        ps = self.page_size
        g.h_ids.zero_()
        g.h_pos.zero_()
        g.h_slots.zero_()
        g.h_lens.fill_(1)
        g.h_bt.zero_()
        ids, pos, slots, lens = g.h_ids.numpy(), g.h_pos.numpy(), g.h_slots.numpy(), g.h_lens.numpy()
        bt = g.h_bt.numpy()
        for i, s in enumerate(seqs):
            p = s["start"]
            if len(s["pages"]) > self.max_pages:
                raise ValueError("sequence longer than EngineConfig.max_model_len")
            ids[i] = s["tokens"][0]
            pos[i] = p
            pages = s["pages"]
            slots[i] = pages[p // ps] * ps + p % ps
            lens[i] = p + 1
            bt[i, : len(pages)] = pages
        g.ids.copy_(g.h_ids, non_blocking=True)
        g.pos.copy_(g.h_pos, non_blocking=True)
        g.slots.copy_(g.h_slots, non_blocking=True)
        g.lens.copy_(g.h_lens, non_blocking=True)
        g.bt.copy_(g.h_bt, non_blocking=True)

    def stage_sampling(self, g: _Graph, step) -> None:
        """Per-row temperature / top-p / top-k / uniform for this step."""
        h = g.h_samp.numpy()
        h[0].fill(0.0)
        h[1].fill(1.0)
        h[2].fill(0.0)
        h[3].fill(0.0)
        if step is not None:
            for i, (r, smp) in enumerate(zip(step.reqs, step.sample)):
                p = r.params
                h[0, i] = p.temperature
                h[1, i] = p.top_p
                h[2, i] = p.top_k
                h[3, i] = r.uniform() if (smp and p.temperature > 0) else 0.0
        g.samp.copy_(g.h_samp, non_blocking=True)
        g.top_k.copy_(g.samp[2])

    def run(self, step, seqs: List[dict], bucket: Optional[int] = None) -> Optional[List[int]]:
        """Replay the graph of `bucket` (default: the smallest that fits);
        `step` None replays with padding rows only (an idle DP rank).  The
        graph samples on the device; only the token ids come back."""
        n = len(seqs)
        bs = bucket or self._bucket(n)
        g = self.graphs.get(bs) or self.capture(bs)
        self.stage(g, seqs)
        self.stage_sampling(g, step)
        g.graph.replay()
        if step is None:
            return None
        g.h_tok.copy_(g.tokens, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return g.h_tok[:n].tolist()

    def release(self) -> None:
        """Drop the graphs (before destroying the process group)."""
        self.graphs.clear()
        self.pool = None

    def disable(self) -> None:
        """After a failed (agreed) capture: decode eagerly from now on."""
        self.release()
        self.enabled = False


def build_verify_batch(seqs: List[dict], k: int, rows: int, page_size: int, max_pages: int) -> ForwardBatch:
    """Speculative-verify batch in a fixed layout: `rows` requests x (1 + k)
    token rows.  Request i occupies rows [i (1 + k), (i + 1)(1 + k)): its
    newest token, its draft, then padding.  Padding rows repeat the last
    real position (so they only read pages the request owns) and write their
    latent to the scratch slot 0 of reserved page 0, so they never touch live
    KV; absent requests are all-padding rows on page 0.  All rows return
    logits.  Host tensors (CPU)."""
    w = 1 + k
    T = rows * w
    ids = torch.zeros(T, dtype=torch.int32)
    pos = torch.zeros(T, dtype=torch.int32)
    qs = torch.arange(rows, dtype=torch.int32).repeat_interleave(w)
    slots = torch.zeros(T, dtype=torch.int64)
    lens = torch.ones(rows, dtype=torch.int32)
    bt = torch.zeros(rows, max_pages, dtype=torch.int32)
    for i, s in enumerate(seqs):
        toks, st, pages = s["tokens"], s["start"], s["pages"]
        if len(toks) > w:
            raise ValueError("draft longer than spec_k")
        if len(pages) > max_pages:
            raise ValueError("sequence longer than EngineConfig.max_model_len")
        for j in range(w):
            r = i * w + j
            if j < len(toks):
                p = st + j
                ids[r] = toks[j]
                slots[r] = pages[p // page_size] * page_size + p % page_size
            else:
                p = st + len(toks) - 1       # padding: the last real position (pages exist up to it)
            pos[r] = p
        lens[i] = st + w
        bt[i, : len(pages)] = torch.tensor(pages, dtype=torch.int32)
    return ForwardBatch(input_ids=ids, positions=pos, q_seq=qs, out_slots=slots, seq_lens=lens, block_table=bt,
                        last_idx=torch.arange(T, dtype=torch.int64), is_decode=False, max_q_len=w,
                        max_seq_len=max_pages * page_size)


class VerifyGraphRunner:
    """CUDA graphs of the speculative-verify forward (fixed 1 + spec_k rows
    per request, one graph per request bucket): logits at every row and the
    greedy argmax on the device, only the token ids come back."""

    def __init__(self, engine, k: int, batch_sizes=None, max_pages: Optional[int] = None):
        self.eng = engine
        self.model = engine.model
        self.dev = engine.device
        ecfg = engine.ecfg
        self.k = k
        self.page_size = ecfg.page_size
        self.batch_sizes = sorted(batch_sizes or [b for b in ecfg.graph_batch_sizes if b <= ecfg.max_num_seqs])
        if not self.batch_sizes or self.batch_sizes[-1] < ecfg.max_num_seqs:
            self.batch_sizes.append(ecfg.max_num_seqs)
        self.max_pages = max_pages or (ecfg.max_model_len + self.page_size - 1) // self.page_size
        self.graphs: Dict[int, _Graph] = {}
        self.pool = None

    def can_run(self, n: int) -> bool:
        return n <= self.batch_sizes[-1]

    def _bucket(self, n: int) -> int:
        for b in self.batch_sizes:
            if b >= n:
                return b
        raise ValueError(n)

    def _capture(self, bs: int) -> _Graph:
        g = _Graph()
        host = build_verify_batch([], self.k, bs, self.page_size, self.max_pages)
        g.h = ForwardBatch(**{k: (v.pin_memory() if isinstance(v, torch.Tensor) else v)
                              for k, v in host.__dict__.items()})
        g.fb = ForwardBatch(**{k: (v.to(self.dev) if isinstance(v, torch.Tensor) else v)
                               for k, v in host.__dict__.items()})
        g.h_tok = torch.zeros(host.num_tokens, dtype=torch.int64).pin_memory()
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.forward(g.fb).argmax(-1)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)

        def record():
            g.graph = torch.cuda.CUDAGraph()
            if self.pool is None:
                self.pool = torch.cuda.graph_pool_handle()
            with torch.cuda.graph(g.graph, pool=self.pool):
                g.tokens = self.model.forward(g.fb).argmax(-1)
        capture_agreed(record, getattr(self.eng.ps, "cpu_group", None), f"verify graph (batch {bs})")
        self.graphs[bs] = g
        return g

    def run(self, seqs: List[dict]) -> List[int]:
        """seqs: per request {"tokens": newest + draft, "start", "pages"};
        returns the argmax token of every row, request-major (1 + k each)."""
        bs = self._bucket(len(seqs))
        g = self.graphs.get(bs) or self._capture(bs)
        host = build_verify_batch(seqs, self.k, bs, self.page_size, self.max_pages)
        for name in ("input_ids", "positions", "out_slots", "seq_lens", "block_table"):
            getattr(g.h, name).copy_(getattr(host, name))
            getattr(g.fb, name).copy_(getattr(g.h, name), non_blocking=True)
        g.graph.replay()
        g.h_tok.copy_(g.tokens, non_blocking=True)
        torch.cuda.current_stream(self.dev).synchronize()
        return g.h_tok.tolist()

    def release(self) -> None:
        self.graphs.clear()
        self.pool = None


def build_extend_batch(seqs: List[dict], tokens: int, rows: int, page_size: int, max_pages: int) -> ForwardBatch:
    """Prefill (extend) batch in a fixed shape: `tokens` token rows and
    `rows` sequence rows.  Sequence i's new tokens are consecutive; the
    remaining token rows are padding that belongs to the last sequence row
    (kept free: rows > len(seqs)), sits at position 0 on reserved page 0 and
    writes its latent to the scratch slot 0.  last_idx[i] is sequence i's last
    token (padding rows point at the last token row).  Host tensors."""
    if len(seqs) >= rows:
        raise ValueError("extend graphs keep one sequence row for padding")
    ids = torch.zeros(tokens, dtype=torch.int32)
    pos = torch.zeros(tokens, dtype=torch.int32)
    qs = torch.full((tokens,), rows - 1, dtype=torch.int32)
    slots = torch.zeros(tokens, dtype=torch.int64)
    lens = torch.ones(rows, dtype=torch.int32)
    bt = torch.zeros(rows, max_pages, dtype=torch.int32)
    last = torch.full((rows,), tokens - 1, dtype=torch.int64)
    t = 0
    for i, s in enumerate(seqs):
        toks, st, pages = s["tokens"], s["start"], s["pages"]
        if len(pages) > max_pages:
            raise ValueError("sequence longer than EngineConfig.max_model_len")
        for j, x in enumerate(toks):
            p = st + j
            ids[t], pos[t], qs[t] = x, p, i
            slots[t] = pages[p // page_size] * page_size + p % page_size
            t += 1
        if t > tokens:
            raise ValueError("extend batch larger than its bucket")
        lens[i] = st + len(toks)
        last[i] = t - 1
        bt[i, : len(pages)] = torch.tensor(pages, dtype=torch.int32)
    return ForwardBatch(input_ids=ids, positions=pos, q_seq=qs, out_slots=slots, seq_lens=lens, block_table=bt,
                        last_idx=last, is_decode=False, max_q_len=tokens, max_seq_len=max_pages * page_size)


class ExtendGraphRunner:
    """CUDA graphs of prefill forwards in fixed (token, sequence) buckets:
    every kernel of the step launches from one graph replay instead of the
    host (the chunks of short prompts are launch-bound).  Logits of each
    sequence's last token come back for sampling."""

    TOKEN_BUCKETS = (64, 128, 256, 512, 1024, 2048)

    def __init__(self, engine, max_pages: int):
        self.eng = engine
        self.model = engine.model
        self.dev = engine.device
        ecfg = engine.ecfg
        self.page_size = ecfg.page_size
        self.row_buckets = sorted({b + 1 for b in ecfg.graph_batch_sizes if b <= ecfg.max_num_seqs}
                                  | {ecfg.max_num_seqs + 1})
        self.max_pages = max_pages
        self.graphs: Dict[tuple, _Graph] = {}
        self.pool = None

    def bucket(self, ntok: int, nseq: int):
        tb = next((b for b in self.TOKEN_BUCKETS if b >= ntok), None)
        rb = next((b for b in self.row_buckets if b > nseq), None)
        return None if tb is None or rb is None else (tb, rb)

    def _capture(self, key) -> _Graph:
        tb, rb = key
        g = _Graph()
        host = build_extend_batch([], tb, rb, self.page_size, self.max_pages)
        g.h = ForwardBatch(**{k: (v.pin_memory() if isinstance(v, torch.Tensor) else v)
                              for k, v in host.__dict__.items()})
        g.fb = ForwardBatch(**{k: (v.to(self.dev) if isinstance(v, torch.Tensor) else v)
                               for k, v in host.__dict__.items()})
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.model.forward(g.fb)
        torch.cuda.current_stream(self.dev).wait_stream(s)
        torch.cuda.synchronize(self.dev)

        def record():
            g.graph = torch.cuda.CUDAGraph()
            if self.pool is None:
                self.pool = torch.cuda.graph_pool_handle()
            with torch.cuda.graph(g.graph, pool=self.pool):
                g.logits = self.model.forward(g.fb)
        capture_agreed(record, getattr(self.eng.ps, "cpu_group", None), f"extend graph {key}")
        self.graphs[key] = g
        return g

    def run(self, seqs: List[dict]) -> Optional[torch.Tensor]:
        """Logits [len(seqs), V] of each sequence's last token, or None when
        the step does not fit a bucket."""
        key = self.bucket(sum(len(s["tokens"]) for s in seqs), len(seqs))
        if key is None:
            return None
        g = self.graphs.get(key) or self._capture(key)
        host = build_extend_batch(seqs, key[0], key[1], self.page_size, self.max_pages)
        for name in ("input_ids", "positions", "q_seq", "out_slots", "seq_lens", "block_table", "last_idx"):
            getattr(g.h, name).copy_(getattr(host, name))
            getattr(g.fb, name).copy_(getattr(g.h, name), non_blocking=True)
        g.graph.replay()
        return g.logits[: len(seqs)]

    def release(self) -> None:
        self.graphs.clear()
        self.pool = None
