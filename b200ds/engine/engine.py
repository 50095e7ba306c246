"""`Engine`: the public serving API (`Engine.generate`), one instance per rank.

Every rank of an SPMD job (torchrun, one process per GPU) constructs the
Engine and calls `generate` with the same requests; schedules, page tables
and sampled tokens are identical on every rank, so no host broadcast is
needed between steps.  Under DP attention (EngineConfig.dp_attention) each
rank instead serves its own requests and the ranks step in lockstep.  The server (b200ds.server) drives rank 0 and
forwards requests to the other ranks over the gloo control group.

Per step: the scheduler picks a prefill or decode batch; the host builds the
flat batch metadata in pinned memory and copies it to the device; the model
runs (decode steps replay a captured CUDA graph per padded batch size); the
sampled token ids come back to the host.

Reference parity: Engine.generate / the OpenAI server belong to SGLang
(absent from the reference, which only replaces the forward:
model_node.py:480-482 and the logits processor lgp.py:555).
"""
from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence, Union

import torch

from .. import ops
from ..config import EngineConfig, ModelConfig
from ..kv.pool import PagePool
from ..kv.radix import RadixCache
from ..models.batch import ForwardBatch, build_batch
from ..models.deepseek import DeepseekModel
from ..parallel.state import ParallelState, get_state
from .request import Request, SamplingParams
from .cuda_graph import GraphCaptureFailed
from .penalties import adjust_logits, needs_adjust
from .scheduler import Scheduler, Step


@dataclass
class GenerateOutput:
    rid: int
    prompt_tokens: int
    token_ids: List[int]
    finish_reason: str
    ttft_s: float
    tpot_s: float
    text: Optional[str] = None
    logprobs: Optional[List[tuple]] = None   # per token: (token, logprob, [(alt, logprob), ...])
    prompt_logprobs: Optional[List[Optional[tuple]]] = None   # per prompt token (None for the first)


def _stop_hit(text: str, stops) -> Optional[int]:
    """Index of the earliest stop string in text, or None."""
    hits = [i for i in (text.find(st) for st in stops if st) if i >= 0]
    return min(hits) if hits else None


def _stop_in_tail(tok, output: List[int], stops) -> bool:
    """Whether a stop string ends in the newest tokens of `output`.  Checked
    after every token, so a stop string first completes in the output's tail:
    only the last (longest stop string + 8) tokens are decoded (a token
    decodes to at least one character, except special tokens and partial
    UTF-8 bytes, which the margin covers), keeping the per-step cost
    independent of the output length."""
    w = max(len(st) for st in stops if st) + 8 if any(stops) else 0
    return w > 0 and _stop_hit(tok.decode(output[-w:]), stops) is not None


def _wants_plp(step) -> bool:
    """A prefill step with a request that asked for prompt log-probabilities."""
    return step.kind == "prefill" and any(r.params.prompt_logprobs is not None for r in step.reqs)


def _wants_lp(reqs) -> bool:
    """Any request of the step asked for log-probabilities or logit
    adjustments (those steps run with full logits, not the token-only decode
    graphs)."""
    return any(r.params.logprobs is not None or needs_adjust(r.params) for r in reqs)


class Engine:
    def __init__(self, model: DeepseekModel, ecfg: EngineConfig, num_pages: Optional[int] = None,
                 eos_token_id: Optional[int] = None, tokenizer=None):
        self.model = model
        self.cfg: ModelConfig = model.cfg
        self.ecfg = ecfg
        self.ps: ParallelState = model.ps
        self.device = model.device
        if num_pages is None:
            num_pages = ecfg.max_kv_pages or self._auto_pages()
        self.pool = PagePool(num_pages, ecfg.page_size)
        model.allocate_kv(num_pages)
        self.mtp = getattr(model, "mtp", None) if ecfg.spec_mtp else None
        if ecfg.spec_mtp:
            if self.mtp is None:
                raise ValueError("spec_mtp needs a model with an MTP module (num_nextn_predict_layers > 0)")
            if ecfg.enable_prefix_cache:
                # the MTP row of a prefix's last position depends on the token after it
                raise ValueError("spec_mtp runs without the prefix cache")
            self.mtp.allocate_kv(num_pages)
        host = None
        if ecfg.enable_prefix_cache and ecfg.host_kv_pages > 0:
            from ..kv.host_cache import HostKVPool
            host = HostKVPool(model.kv_tensors(), ecfg.host_kv_pages, ecfg.page_size)
        self.radix = RadixCache(self.pool, host) if ecfg.enable_prefix_cache else None
        self.sched = Scheduler(self.pool, ecfg.max_num_seqs, ecfg.max_prefill_tokens, self.radix,
                               mixed=ecfg.mixed_steps and not ecfg.dp_attention and not ecfg.spec_mtp,
                               policy=ecfg.schedule_policy)
        self.eos = eos_token_id
        self.tokenizer = tokenizer
        self._next_rid = 0
        self.graphs = None
        self.verify_graphs, self.verify_graphs_ok = None, True
        self.extend_graphs, self.extend_graphs_ok = None, True
        if self.device.type == "cuda" and ecfg.cuda_graphs:
            from .cuda_graph import DecodeGraphRunner
            self.graphs = DecodeGraphRunner(self)
        self.stats: Dict[str, float] = {"steps": 0, "prefill_tokens": 0, "decode_tokens": 0}
        self._step_lp: Dict[int, list] = {}
        # DP attention: every rank schedules its own requests; ranks agree
        # each step on the mode and on the per-rank token rows of the MoE
        # exchange (gloo, host only), and an idle rank joins with a dummy.
        self.dp = bool(ecfg.dp_attention) and self.ps.ep_size > 1
        # context-parallel prefill: every rank holds the same queue of long
        # prompts (added on all ranks in the same order) and prefills its
        # head together, chunk by chunk, ahead of the ranks' own steps
        if ecfg.context_parallel and not self.dp:
            raise ValueError("context_parallel needs dp_attention over more than one rank")
        self.cp = bool(ecfg.context_parallel)
        self._cp_wait: Deque[Request] = deque()
        self._cp_cur: Optional[Request] = None
        self._cp_seq = 0
        import os
        if ecfg.trace or os.environ.get("B200_TRACE", "0") == "1":
            from ..utils.trace import Tracer
            model.tracer = Tracer(self.device, enabled=True)
        self.selfcheck = {}
        if self.device.type == "cuda" and ecfg.selfcheck:
            from .. import ops
            if ops.get_impl() == "native":
                from ..ops import cuda as _cuda
                from ..utils import levers
                _cuda.register_selfchecks()
                self.selfcheck = levers.selfcheck(getattr(self.ps, "cpu_group", None))

    def _auto_pages(self) -> int:
        if self.device.type != "cuda":
            return 1024
        free, _ = torch.cuda.mem_get_info(self.device)
        per_page = self.model.kv_bytes_per_token() * self.ecfg.page_size
        return max(16, int(free * self.ecfg.kv_cache_fraction) // per_page)

    # ------------------------------------------------------------------
    def add_request(self, prompt: Union[str, Sequence[int]], params: Optional[SamplingParams] = None,
                    cp_owner: Optional[int] = None) -> Request:
        """Queue a request.  cp_owner (context_parallel engines): prefill the
        prompt on every rank and decode it on rank cp_owner; every rank must
        add it between the same two steps, in the same order relative to its
        other context-parallel requests.  On the other ranks the returned request finishes after the
        prefill with finish_reason "context_parallel_peer" and no tokens."""
        if isinstance(prompt, str):
            assert self.tokenizer is not None, "text prompts need a tokenizer"
            prompt = self.tokenizer.encode(prompt)
        params = params or SamplingParams()
        prompt = [int(t) for t in prompt]      # python ints (tensor / numpy rows accepted)
        self.check_request(prompt, params)
        if cp_owner is not None:
            self._cp_check(params, int(cp_owner))
        r = Request(self._next_rid, prompt, params)
        self._next_rid += 1
        if cp_owner is not None:
            r.cp_owner, r.cp_seq = int(cp_owner), self._cp_seq
            self._cp_seq += 1
            self._cp_wait.append(r)
            return r
        self.sched.add(r)
        return r

    def check_request(self, prompt_ids: Sequence[int], params: SamplingParams) -> None:
        """Raise ValueError for a request the engine cannot serve (checked
        before it is queued, so one bad request never reaches a step): empty
        prompt, ids outside the vocabulary, prompt + max_tokens beyond
        max_model_len or beyond the whole KV pool."""
        n = len(prompt_ids)
        if n == 0:
            raise ValueError("the prompt is empty")
        V = self.cfg.vocab_size
        bad = next((t for t in prompt_ids if not (isinstance(t, int) and 0 <= t < V)), None)
        if bad is not None:
            raise ValueError(f"token id {bad!r} is outside the vocabulary [0, {V})")
        if params.max_tokens < 0:
            raise ValueError("max_tokens must be >= 0")
        if params.logit_bias and any(not 0 <= int(t) < V for t in params.logit_bias):
            raise ValueError("logit_bias names a token id outside the vocabulary")
        if params.guided_regex is not None or params.guided_choice or params.guided_json is not None:
            if self.tokenizer is None:
                raise ValueError("guided decoding needs a tokenizer")
            from .guided import Guide, guide_pattern
            try:
                Guide(guide_pattern(params))
            except Exception as e:
                raise ValueError(f"guided pattern does not compile: {e}")
        total = n + params.max_tokens
        if total > self.ecfg.max_model_len:
            raise ValueError(f"the maximum context length is {self.ecfg.max_model_len} tokens; the request needs "
                             f"{total} ({n} in the prompt, {params.max_tokens} to generate)")
        if self.pool.pages_for(total) > self.pool.num_pages - 1:       # page 0 is the scratch page
            raise ValueError(f"the request needs {total} tokens of KV cache; the pool holds "
                             f"{(self.pool.num_pages - 1) * self.pool.page_size}")

    def abort(self, r: Request) -> None:
        """Stop a request now (client gone): it leaves the schedule, its pages
        are freed, finish_reason becomes "abort".  Call between steps; SPMD
        ranks must abort the same requests in the same order."""
        if r.finished:
            return
        if r.cp_seq >= 0 and (r is self._cp_cur or r in self._cp_wait):
            r.cp_abort = True          # dropped on every rank at the next agreed step
            return
        self.sched.abort(r)
        r.finished, r.finish_reason = True, "abort"
        r.t_done = time.perf_counter()

    def _forward(self, step: Step) -> List[int]:
        seqs = [{"tokens": ch, "start": st, "pages": r.pages}
                for r, ch, st in zip(step.reqs, step.chunks, step.starts)]
        if (step.kind == "decode" and self.graphs is not None and self.graphs.can_run(len(seqs))
                and not _wants_lp(step.reqs)):      # the decode graph returns token ids only
            try:
                return self.graphs.run(step, seqs)
            except GraphCaptureFailed as e:    # agreed on every rank: eager decode from now on
                self._graphs_off("decode", e)
        if (step.kind == "prefill" and self.graphs is not None and self.ecfg.extend_graphs and self.mtp is None
                and self.extend_graphs_ok and not _wants_plp(step)):
            if self.extend_graphs is None:
                from .cuda_graph import ExtendGraphRunner
                self.extend_graphs = ExtendGraphRunner(self, self.graphs.max_pages)
            try:
                logits = self.extend_graphs.run(seqs)
            except GraphCaptureFailed as e:    # agreed on every rank: eager prefill from now on
                self._graphs_off("extend", e)
                logits = None
            if logits is not None:
                toks = self._sample(step, logits)
                self._note_lp(step.reqs, logits, range(len(toks)), [[t] for t in toks], step.sample)
                return toks
        logits = self._eager_logits(step, seqs)
        toks = self._sample(step, logits)
        self._note_lp(step.reqs, logits, range(len(toks)), [[t] for t in toks], step.sample)
        if self.mtp is not None and step.kind == "prefill":
            self._mtp_prefill(step, toks)
        return toks

    def _dp_forward(self, step: Optional[Step]) -> Optional[List[int]]:
        """One lockstep DP-attention forward.  All ranks run the same kind of
        forward: the decode graph of the largest rank's bucket when every
        rank decodes, else eager with dp_tmax = the largest rank's tokens.
        Speculative drafts (n-gram) join the agreement: when any rank
        verifies, every rank runs eagerly and the verifying ranks score their
        drafts in the same forward.  Returns None when no rank has work, else
        (tokens, accepted lists): ([], None) for an idle rank that joined with
        a dummy forward, (tokens, None) after a plain step, (None, accepted
        tokens per request) after a verify."""
        import torch.distributed as dist
        drafts = self._propose_drafts(step)
        ntok = 0 if step is None else sum(len(c) for c in step.chunks) + sum(len(d) for d in drafts or [])
        nseq = 0 if step is None else len(step.reqs)
        prefill = step is not None and step.kind == "prefill"
        lp = step is not None and (_wants_lp(step.reqs) or _wants_plp(step))
        decoding = step is not None and not prefill
        v = torch.tensor([int(prefill), ntok, nseq, int(step is not None), int(lp), int(drafts is not None),
                          int(decoding)], dtype=torch.int64)
        dist.all_reduce(v, op=dist.ReduceOp.MAX, group=self.ps.cpu_group)
        any_prefill, max_tok, max_seq, any_work, any_lp, any_verify, any_decode = (int(x) for x in v)
        if not any_work:
            return None
        # a rank's decode batch is split between the micro-batches only where
        # the routing does not depend on the batch (the E5 prune does)
        if (self.ecfg.tbo and any_prefill and not any_lp and not any_verify and self.mtp is None
                and max_tok >= max(2, self.ecfg.tbo_min_tokens) and getattr(self.model, "supports_tbo", False)
                and (not any_decode or getattr(self.model, "tbo_splits_decode", True))):
            # every rank splits its rows into two micro-batches the same way
            self.stats["tbo_steps"] = self.stats.get("tbo_steps", 0) + 1
            seqs = [] if step is None else [{"tokens": ch, "start": st, "pages": r.pages}
                                            for r, ch, st in zip(step.reqs, step.chunks, step.starts)]
            logits = self._tbo_logits(seqs, max_tok)
            if step is None:
                return [], None
            toks = self._sample(step, logits)
            self._note_lp(step.reqs, logits, range(len(toks)), [[t] for t in toks], step.sample)
            return toks, None
        seqs = [] if step is None else [{"tokens": ch, "start": st, "pages": r.pages}
                                        for r, ch, st in zip(step.reqs, step.chunks, step.starts)]
        if (not any_prefill and not any_lp and not any_verify and self.graphs is not None
                and self.graphs.can_run(max_seq)):
            try:
                toks = self.graphs.run(step, seqs, bucket=self.graphs._bucket(max_seq))
                return [] if toks is None else toks, None
            except GraphCaptureFailed as e:    # agreed on every rank: eager decode from now on
                self._graphs_off("decode", e)
        if step is None:      # idle rank: one dummy token on the scratch page
            fb = build_batch([{"tokens": [0], "start": 0, "pages": [0]}], self.ecfg.page_size, device="cpu")
            fb.dp_tmax = max(max_tok, 1)
            self.model.forward(self._to_device(fb))
            return [], None
        if drafts is not None:  # this rank verifies its drafts in the same lockstep forward
            seqs = [{"tokens": ch + d, "start": s, "pages": r.pages}
                    for r, ch, s, d in zip(step.reqs, step.chunks, step.starts, drafts)]
            return None, self._verify_eager(step, seqs, drafts, dp_tmax=max(max_tok, 1))
        logits = self._eager_logits(step, seqs, dp_tmax=max(max_tok, 1))
        toks = self._sample(step, logits)
        self._note_lp(step.reqs, logits, range(len(toks)), [[t] for t in toks], step.sample)
        return toks, None

    def _tbo_logits(self, seqs: List[dict], max_tok: int) -> Optional[torch.Tensor]:
        """Two-batch overlap: this rank's rows split in two halves (a
        sequence crossing the cut continues in the second micro-batch, whose
        queries then read the first half's cache rows, written earlier in the
        same layer); micro-batch k exchanges up to the agreed ceil / floor
        half of the largest rank's rows; an empty half runs one dummy token on
        the scratch page.  Returns the logits of each sequence's last row."""
        T_r = sum(len(s["tokens"]) for s in seqs)
        cut = (T_r + 1) // 2
        halves: List[List[dict]] = [[], []]
        ends = []
        off = 0
        for s in seqs:
            toks, st, n = s["tokens"], s["start"], len(s["tokens"])
            if off + n <= cut:
                halves[0].append(s)
            elif off >= cut:
                halves[1].append(s)
            else:
                k = cut - off
                halves[0].append({"tokens": toks[:k], "start": st, "pages": s["pages"]})
                halves[1].append({"tokens": toks[k:], "start": st + k, "pages": s["pages"]})
            m = 0 if off + n <= cut else 1
            ends.append((m, len(halves[m]) - 1))
            off += n
        dummy = {"tokens": [0], "start": 0, "pages": [0]}
        tmax = ((max_tok + 1) // 2, max_tok // 2)
        fbs = []
        for half, tm in zip(halves, tmax):
            fb = build_batch(half or [dummy], self.ecfg.page_size, device="cpu")
            fb.dp_tmax = max(tm, 1)
            fbs.append(self._to_device(fb))
        outs = self.model.forward_tbo(fbs)
        if not seqs:
            return None
        return torch.stack([outs[m][j] for m, j in ends])

    def _eager_logits(self, step: Step, seqs: List[dict], dp_tmax: int = 0) -> torch.Tensor:
        """Eager forward of a step; returns the logits of each sequence's last
        row.  Prefill chunks of requests that asked for prompt log-probabilities
        get logits at every row, recorded here."""
        fb = build_batch(seqs, self.ecfg.page_size, device="cpu")
        fb.dp_tmax = dp_tmax
        fb.tail_from = self._tail_from(step)
        sel = None
        if _wants_plp(step):
            idx, sel, off = [], [], 0
            for r, ch in zip(step.reqs, step.chunks):
                n = len(ch)
                idx.extend(range(off, off + n) if r.params.prompt_logprobs is not None else [off + n - 1])
                sel.append(len(idx) - 1)
                off += n
            fb.last_idx = torch.tensor(idx, dtype=torch.int64)
        fb = self._to_device(fb)
        logits = self.model.forward(fb)
        if sel is None:
            return logits
        self._note_prompt_lp(step, logits)
        return logits[torch.tensor(sel, device=logits.device)]

    def _note_prompt_lp(self, step: Step, logits: torch.Tensor) -> None:
        """Row j of a prompt-logprob request's chunk (position p = start + j)
        scores prompt token p + 1; positions already recorded (a recompute
        after preemption) are skipped."""
        row = 0
        for r, ch, st in zip(step.reqs, step.chunks, step.starts):
            m = r.params.prompt_logprobs
            if m is None:
                row += 1
                continue
            if not r.prompt_lp:
                r.prompt_lp.append(None)
            lp = torch.log_softmax(logits[row: row + len(ch)].float(), -1)
            tv, ti = lp.topk(m, -1) if m > 0 else (None, None)
            for j in range(len(ch)):
                p = st + j
                if p + 1 >= len(r.prompt) or len(r.prompt_lp) != p + 1:
                    continue
                t = r.prompt[p + 1]
                top = list(zip(ti[j].tolist(), tv[j].tolist())) if m > 0 else []
                r.prompt_lp.append((t, float(lp[j, t]), top))
            row += len(ch)

    def _tail_from(self, step: Step) -> Optional[torch.Tensor]:
        """Prefill tail of a step (window-only late layers, V4 family): per
        sequence, the first position those layers must compute - a prompt
        needs only its last `tail_rows_needed()` positions there, a decode
        row in a mixed step needs its row.  None when off: no window layers,
        EngineConfig.prefill_tail off, or the prefix cache / MTP draft on
        (both reuse rows a tail would leave out)."""
        c = self.model.cfg
        if (step.kind != "prefill" or not c.is_v4 or c.late_layer_start is None or c.late_window <= 0
                or not self.ecfg.prefill_tail or self.radix is not None or self.mtp is not None
                or _wants_plp(step)):
            return None
        from .scheduler import prefill_target
        n_pre = len(step.reqs) - step.decode_rows
        need = c.tail_rows_needed()
        return torch.tensor([max(0, prefill_target(r) - need) if k < n_pre else 0
                             for k, r in enumerate(step.reqs)], dtype=torch.int32)

    def _note_lp(self, reqs, logits: torch.Tensor, rows, emitted: List[List[int]], sample=None) -> None:
        """Log-probabilities of this step's emitted tokens for requests that
        asked for them: token emitted[i][j] was produced from logits row
        rows[i] + j.  The values are the model's (log-softmax of the raw
        logits, before temperature / top-k / top-p), with the request's top-n
        alternatives; they are kept until the tokens are appended."""
        sel = [(r, int(r0) + j, t) for k, (r, r0, em) in enumerate(zip(reqs, rows, emitted))
               if r.params.logprobs is not None and (sample is None or sample[k]) for j, t in enumerate(em)]
        if not sel:
            return
        dev = logits.device
        lp = torch.log_softmax(logits[torch.tensor([i for _, i, _ in sel], device=dev)].float(), -1)
        chosen = lp.gather(1, torch.tensor([[t] for _, _, t in sel], device=dev))[:, 0].tolist()
        n = max(r.params.logprobs for r, _, _ in sel)
        tv, ti = lp.topk(n, -1) if n > 0 else (None, None)
        tv, ti = (tv.tolist(), ti.tolist()) if n > 0 else (None, None)
        for k, (r, _, t) in enumerate(sel):
            m = r.params.logprobs
            top = list(zip(ti[k][:m], tv[k][:m])) if m > 0 else []
            self._step_lp.setdefault(r.rid, []).append((int(t), float(chosen[k]), top))

    def _graphs_off(self, kind: str, err: Exception) -> None:
        """A capture of `kind` failed on some rank (the verdict is agreed, so
        every rank gets here at the same step): drop those graphs and run
        that kind of forward eagerly from now on."""
        from ..utils import levers
        levers.announce(f"{kind}-graphs-off", f"{kind} graphs off ({err}); eager {kind}")
        if kind == "decode":
            self.graphs.disable()
        elif kind == "verify":
            self.verify_graphs.release()
            self.verify_graphs, self.verify_graphs_ok = None, False
        else:
            self.extend_graphs.release()
            self.extend_graphs, self.extend_graphs_ok = None, False

    def _to_device(self, fb: ForwardBatch) -> ForwardBatch:
        if self.device.type == "cpu":
            return fb
        kw = {}
        for k, v in fb.__dict__.items():
            if isinstance(v, torch.Tensor):
                kw[k] = v.pin_memory().to(self.device, non_blocking=True)
            else:
                kw[k] = v
        return ForwardBatch(**kw)

    def _sample(self, step: Step, logits: torch.Tensor) -> List[int]:
        if any(needs_adjust(r.params) for r in step.reqs):
            logits = adjust_logits(logits, step.reqs, step.sample, self.eos, self.tokenizer)
        B = logits.shape[0]
        temp = torch.tensor([r.params.temperature for r in step.reqs], dtype=torch.float32)
        if bool((temp <= 0).all()):
            return logits.argmax(-1).tolist()
        top_p = torch.tensor([r.params.top_p for r in step.reqs], dtype=torch.float32)
        top_k = torch.tensor([r.params.top_k for r in step.reqs], dtype=torch.int32)
        u = torch.tensor([r.uniform() if s else 0.0 for r, s in zip(step.reqs, step.sample)],
                         dtype=torch.float32)
        dev = logits.device
        return ops.sample(logits, temp.to(dev), top_p.to(dev), top_k.to(dev), u.to(dev)).tolist()

    def step(self) -> List[Request]:
        """Run one scheduler step; returns requests that finished."""
        if self._cp_pending() and self._cp_agree():
            self._step_lp = {}
            return self._cp_step()
        st = self.sched.next_step()
        multi = None
        self._step_lp: Dict[int, list] = {}
        if self.dp:
            res = self._dp_forward(st)
            if st is None:
                return []
            toks, multi = res
        elif st is None:
            return []
        else:
            multi = None
            if st.kind == "decode" and self.mtp is not None:
                multi = self._mtp_decode(st)
            elif st.kind == "decode" and self.ecfg.spec_ngram > 0:
                multi = self._spec_decode(st)
            toks = None if multi is not None else self._forward(st)
        if multi is None:
            self.sched.commit(st)
            multi = [[t] for t in toks]
        else:
            for r, new in zip(st.reqs, multi):     # newest token + accepted drafts are cached now
                r.cached += len(new)
        self._check_device_errors()
        now = time.perf_counter()
        self.stats["steps"] += 1
        if st.kind == "prefill":
            n_pre = len(st.chunks) - st.decode_rows
            self.stats["prefill_tokens"] += sum(len(c) for c in st.chunks[:n_pre])
            self.stats["decode_tokens"] += st.decode_rows
        else:
            self.stats["decode_tokens"] += sum(len(m) for m in multi)
        return self._emit(st, multi, now)

    def _emit(self, st: Step, multi, now: float) -> List[Request]:
        """Append each sampled request's new tokens, apply the stop rules and
        release finished requests; returns those."""
        done = []
        for r, smp, new in zip(st.reqs, st.sample, multi):
            if not smp:
                continue
            if r.params.max_tokens <= 0 or getattr(r, "guide_done", False):
                # prompt only (e.g. prompt log-probabilities), or a guided output
                # that no token can extend: no token
                r.finished, r.t_done = True, now
                r.finish_reason = "stop" if r.params.max_tokens > 0 else "length"
                self.sched.finish(r)
                done.append(r)
                continue
            lps = self._step_lp.get(r.rid)
            for k, t in enumerate(new):
                r.output.append(int(t))
                if lps is not None:
                    r.logprobs.append(lps[k])
                r.token_times.append(now)
                if r.t_first is None:
                    r.t_first = now
                p = r.params
                if len(r.output) >= p.max_tokens:
                    r.finished, r.finish_reason = True, "length"
                elif not p.ignore_eos and ((self.eos is not None and t == self.eos) or t in p.stop_token_ids):
                    r.finished, r.finish_reason = True, "stop"
                elif p.stop and self.tokenizer is not None and _stop_in_tail(self.tokenizer, r.output, p.stop):
                    r.finished, r.finish_reason = True, "stop"
                if r.finished:
                    r.t_done = now
                    self.sched.finish(r)
                    done.append(r)
                    break
        return done

    # ------------------------------------------------------------------
    # Speculative decoding (greedy): n-gram drafts verified in one forward
    def _ngram_draft(self, r: Request) -> List[int]:
        """Up to spec_k tokens that followed the most recent earlier occurrence
        of the context's last n tokens (n = spec_ngram .. 1)."""
        ctx = r.all_tokens[: r.cached + 1]
        k = self.ecfg.spec_k
        for n in range(min(self.ecfg.spec_ngram, len(ctx) - 1), 0, -1):
            pat = ctx[-n:]
            for j in range(len(ctx) - n - 1, -1, -1):
                if ctx[j:j + n] == pat:
                    d = ctx[j + n: j + n + k]
                    if d:
                        return d
        return []

    def _spec_decode(self, st: Step) -> Optional[List[List[int]]]:
        """Verify per-request drafts with one forward over [newest token + draft]
        (logits at every position).  Returns the accepted tokens per request
        (accepted draft prefix + the model's next token), or None when no
        request has a draft (plain decode then)."""
        if self.dp:
            return None       # DP ranks verify inside the lockstep forward (_dp_forward)
        drafts = self._propose_drafts(st)
        if drafts is None:
            return None
        sampling = any(r.params.temperature > 0 for r in st.reqs)
        want_lp = _wants_lp(st.reqs)
        seqs = [{"tokens": ch + d, "start": s, "pages": r.pages}
                for r, ch, s, d in zip(st.reqs, st.chunks, st.starts, drafts)]
        k = self.ecfg.spec_k
        if self.graphs is not None and self.verify_graphs_ok and not sampling and not want_lp:
            # fixed (1 + spec_k) rows per request: one captured graph per bucket
            if self.verify_graphs is None:
                from .cuda_graph import VerifyGraphRunner
                self.verify_graphs = VerifyGraphRunner(self, k, max_pages=self.graphs.max_pages)
            if self.verify_graphs.can_run(len(seqs)):
                try:
                    pred = self.verify_graphs.run(seqs)
                except GraphCaptureFailed as e:    # agreed on every rank: verify eagerly from now on
                    self._graphs_off("verify", e)
                else:
                    starts = [i * (1 + k) for i in range(len(seqs))]
                    return self._accept(st, drafts, pred, starts)
        return self._verify_eager(st, seqs, drafts)

    def _propose_drafts(self, st: Step) -> Optional[List[List[int]]]:
        """n-gram drafts of a decode step's requests (pages reserved for them),
        or None when no request has one or a request needs adjusted logits
        (drafts are verified against the raw logits)."""
        if (st is None or st.kind != "decode" or self.ecfg.spec_ngram <= 0 or self.mtp is not None or not st.reqs
                or any(needs_adjust(r.params) for r in st.reqs)):
            return None
        drafts = []
        for r in st.reqs:
            room = r.params.max_tokens - len(r.output) - 1
            d = self._ngram_draft(r)[: max(0, room)]
            if d and not self.sched._ensure_pages(r, r.cached + 1 + len(d)):
                d = []
            drafts.append(d)
        return drafts if any(drafts) else None

    def _verify_eager(self, st: Step, seqs: List[dict], drafts, dp_tmax: int = 0) -> List[List[int]]:
        """One forward over [newest token + draft] per request with logits at
        every row, then greedy or speculative-sampling acceptance."""
        fb = build_batch(seqs, self.ecfg.page_size, device="cpu")
        fb.last_idx = torch.arange(fb.num_tokens, dtype=torch.int64)     # logits at every position
        fb.dp_tmax = dp_tmax
        fb = self._to_device(fb)
        logits = self.model.forward(fb)
        starts, off = [], 0
        for d in drafts:
            starts.append(off)
            off += 1 + len(d)
        if any(r.params.temperature > 0 for r in st.reqs):
            out = self._accept_sampled(st, drafts, logits, starts)
        else:
            out = self._accept(st, drafts, logits.argmax(-1).tolist(), starts)
        self._note_lp(st.reqs, logits, starts, out)
        return out

    def _accept_sampled(self, st: Step, drafts, logits: torch.Tensor, starts: List[int]) -> List[List[int]]:
        """Speculative sampling with deterministic (n-gram) drafts: draft token
        d at a row is kept with probability p(d) under the request's sampling
        distribution (temperature / top-k / top-p as the sampler applies
        them); on rejection the row's token is drawn from p with d removed;
        after a fully accepted draft the last row is sampled as usual.  The
        accepted tokens follow the same distribution as plain sampling."""
        from ..ops.ref import sampling_probs
        out = []
        lg = logits.float().cpu()
        for r, d, off in zip(st.reqs, drafts, starts):
            p = r.params
            if p.temperature <= 0:
                row = lg[off: off + 1 + len(d)].argmax(-1).tolist()
                a = 0
                while a < len(d) and row[a] == d[a]:
                    a += 1
                toks = d[:a] + [row[a]]
            else:
                toks = []
                for j in range(len(d) + 1):
                    probs = sampling_probs(lg[off + j], p.temperature, p.top_p, p.top_k)
                    probs = probs / probs.sum()
                    if j < len(d):
                        if r.uniform() < float(probs[d[j]]):
                            toks.append(d[j])
                            continue
                        probs = probs.clone()
                        probs[d[j]] = 0.0
                    c = probs.cumsum(0)
                    u = r.uniform() * float(c[-1])
                    toks.append(int(torch.searchsorted(c, torch.tensor([u])).clamp(max=probs.numel() - 1)))
                    break
                a = len(toks) - 1
            out.append(toks)
            self.stats["spec_proposed"] = self.stats.get("spec_proposed", 0) + len(d)
            self.stats["spec_accepted"] = self.stats.get("spec_accepted", 0) + a
        return out

    def _accept(self, st: Step, drafts, pred: List[int], starts: List[int]) -> List[List[int]]:
        """Greedy acceptance: the longest draft prefix the model reproduces,
        then the model's own next token."""
        out = []
        for r, d, off in zip(st.reqs, drafts, starts):
            p = pred[off: off + 1 + len(d)]
            a = 0
            while a < len(d) and p[a] == d[a]:
                a += 1
            out.append(d[:a] + [p[a]])
            self.stats["spec_proposed"] = self.stats.get("spec_proposed", 0) + len(d)
            self.stats["spec_accepted"] = self.stats.get("spec_accepted", 0) + a
        return out

    # ------------------------------------------------------------------
    # Speculative decoding with the model's MTP module as the draft
    def _mtp_run(self, rows, prev_h):
        """One MTP forward over `rows` (see models/mtp.py::mtp_batch);
        returns (greedy draft token, MTP hidden) of each request's last row."""
        from ..models.mtp import mtp_batch
        fb = mtp_batch(rows, self.ecfg.page_size, "cpu")
        fb = self._to_device(fb)
        logits, hid = self.mtp.forward(fb, prev_h)
        return logits.argmax(-1).tolist(), hid

    def _mtp_chain(self, reqs, first, hid, n_next) -> None:
        """Drafts 2..spec_k: the module applied to its own hidden state.
        reqs[i]'s newest draft sits at token position n_next[i]."""
        drafts = [[t] for t in first]
        for _ in range(self.ecfg.spec_k - 1):
            rows = []
            for r, d, n in zip(reqs, drafts, n_next):
                j = n + len(d) - 1            # token position of the newest draft
                if not self.sched._ensure_pages(r, j):
                    return self._mtp_store(reqs, drafts, hid)
                rows.append({"tokens": [d[-1]], "j0": j, "pages": r.pages})
            nxt, hid = self._mtp_run(rows, hid)
            for d, t in zip(drafts, nxt):
                d.append(t)
        self._mtp_store(reqs, drafts, hid)

    @staticmethod
    def _mtp_store(reqs, drafts, hid) -> None:
        for r, d in zip(reqs, drafts):
            r.mtp_drafts = d

    def _mtp_prefill(self, st: Step, toks: List[int]) -> None:
        """After a prefill chunk: MTP rows for the chunk's positions (and, when
        the prompt is done, the sampled token's), from the main model's
        hidden states; finished prompts get their first drafts."""
        H = self.model.last_residual
        rows, prev, fin, fin_pos = [], [], [], []
        off = 0
        for i, (r, ch, s) in enumerate(zip(st.reqs, st.chunks, st.starts)):
            n = len(ch)
            Hr = H[off: off + n]
            off += n
            toks_j, prev_j = [], []
            j0 = max(s, 1)
            for j in range(j0, s + n):
                toks_j.append(ch[j - s])
                prev_j.append(Hr[j - 1 - s] if j - 1 >= s else getattr(r, "mtp_h_prev", None))
            if st.sample[i]:
                if not toks_j:
                    j0 = s + n
                toks_j.append(toks[i])
                prev_j.append(Hr[n - 1])
            r.mtp_h_prev = Hr[n - 1].clone()
            if toks_j and all(p is not None for p in prev_j):
                rows.append({"tokens": toks_j, "j0": j0, "pages": r.pages, "req": r, "fin": st.sample[i]})
                prev.extend(prev_j)
        if not rows:
            return
        draft, hid = self._mtp_run(rows, torch.stack(prev))
        reqs = [row["req"] for row in rows if row["fin"]]
        if not reqs:
            return
        idx = [k for k, row in enumerate(rows) if row["fin"]]
        n_next = [row["j0"] + len(row["tokens"]) for row in rows if row["fin"]]
        self._mtp_chain(reqs, [draft[k] for k in idx], hid[idx], n_next)

    def _mtp_decode(self, st: Step) -> Optional[List[List[int]]]:
        """Verify the MTP drafts in one main-model forward with logits and
        hidden states at every row (greedy acceptance, or speculative sampling
        for temperature > 0: the drafts are the module's argmax, a
        deterministic function of the context), then run the MTP module over
        the accepted tokens for the next drafts."""
        if any(needs_adjust(r.params) for r in st.reqs):
            for r in st.reqs:
                r.mtp_drafts = []
            return None
        drafts = []
        for r in st.reqs:
            room = r.params.max_tokens - len(r.output) - 1
            d = list(getattr(r, "mtp_drafts", []))[: max(0, room)]
            if d and not self.sched._ensure_pages(r, r.cached + 1 + len(d)):
                d = []
            drafts.append(d)
        seqs = [{"tokens": ch + d, "start": s, "pages": r.pages}
                for r, ch, s, d in zip(st.reqs, st.chunks, st.starts, drafts)]
        fb = build_batch(seqs, self.ecfg.page_size, device="cpu")
        fb.last_idx = torch.arange(fb.num_tokens, dtype=torch.int64)     # logits at every position
        fb = self._to_device(fb)
        logits = self.model.forward(fb)
        H = self.model.last_residual
        starts, off = [], 0
        for d in drafts:
            starts.append(off)
            off += 1 + len(d)
        if any(r.params.temperature > 0 for r in st.reqs):
            out = self._accept_sampled(st, drafts, logits, starts)
        else:
            out = self._accept(st, drafts, logits.argmax(-1).tolist(), starts)
        self._note_lp(st.reqs, logits, starts, out)
        rows, prev = [], []
        for r, o, s0, n in zip(st.reqs, out, starts, st.starts):
            # token positions n + 1 .. n + len(o) hold the accepted tokens
            rows.append({"tokens": o, "j0": n + 1, "pages": r.pages})
            prev.extend(H[s0 + k] for k in range(len(o)))
            r.mtp_h_prev = H[s0 + len(o) - 1].clone()
        if not all(self.sched._ensure_pages(r, n + len(o)) for r, o, n in zip(st.reqs, out, st.starts)):
            self._mtp_store(st.reqs, [[] for _ in st.reqs], None)
            return out
        draft, hid = self._mtp_run(rows, torch.stack(prev))
        self._mtp_chain(st.reqs, draft, hid, [n + len(o) + 1 for o, n in zip(out, st.starts)])
        return out

    def update_weights(self, weights, seed: int = 0) -> int:
        """Load new weights of the same architecture (a checkpoint directory,
        a full state dict, or "random" with a seed) into the live model in
        place; returns the bytes copied.  Captured graphs stay valid (same
        buffers); the prefix cache, whose rows came from the old weights, is
        cleared.  Call with no requests in flight; every rank of an SPMD job
        makes the same call."""
        if self.sched.has_work:
            raise ValueError("update_weights needs an idle engine (no queued or running requests)")
        from .. import build_model_from
        from ..models.weights_update import copy_weights
        new = build_model_from(self.cfg, self.ecfg, weights, device=self.device, seed=seed, ps=self.ps)
        n = copy_weights(self.model, new)
        del new
        self.flush_cache()
        return n

    def flush_cache(self) -> int:
        """Clear the prefix cache (both tiers); returns the device pages
        freed.  Only when no request holds cached pages (an idle engine)."""
        if self.radix is None:
            return 0
        if self.sched.has_work:
            raise ValueError("flush_cache needs an idle engine")
        return self.radix.clear()

    def gauges(self) -> Dict[str, float]:
        """Current queue and KV-pool state and the scheduler's counters."""
        sc = self.sched
        return {"running": len(sc.running), "prefilling": len(sc.prefilling), "waiting": len(sc.waiting),
                "kv_pages_total": self.pool.num_pages, "kv_pages_free": self.pool.num_free,
                "admitted_prompt_tokens": sc.admitted_prompt_tokens, "prefix_hit_tokens": sc.prefix_hit_tokens,
                "preemptions": sc.preemptions, "cp_queue": len(self._cp_wait) + (self._cp_cur is not None),
                "host_offloads": self.radix.offloads if self.radix is not None else 0,
                "host_restores": self.radix.restores if self.radix is not None else 0}

    def _check_device_errors(self) -> None:
        """Every device-side wait in the fused collectives is bounded; a wait
        that ran out (a peer that stopped pushing) leaves an error word on
        the device instead of hanging the GPU.  Surface it after each step."""
        for obj in (getattr(self.ps, "fused_ar", None), getattr(self.ps, "fused_ep", None)):
            if obj is not None:
                obj.check()
        if self.device.type == "cuda" and ops.get_impl() == "native":
            from ..ops import cuda as _cuda
            _cuda.check_device_errors()

    def generate(self, prompts: Sequence[Union[str, Sequence[int]]],
                 params: Union[SamplingParams, Sequence[SamplingParams], None] = None,
                 cp_owner: Union[int, Sequence[Optional[int]], None] = None) -> List[GenerateOutput]:
        """Run the prompts to completion and return one output per prompt
        (in order).  Identical calls on every rank of an SPMD job produce
        identical results.  cp_owner (context_parallel engines; one rank for
        all prompts or one per prompt, None = ordinary): the prompts prefill
        on every rank and decode on their owner, so every rank passes the
        same prompts; the other ranks' outputs are empty."""
        if params is None or isinstance(params, SamplingParams):
            params = [params or SamplingParams()] * len(prompts)
        owners = cp_owner if isinstance(cp_owner, (list, tuple)) else [cp_owner] * len(prompts)
        reqs = [self.add_request(p, sp, cp_owner=o) for p, sp, o in zip(prompts, params, owners)]
        while any(not r.finished for r in reqs):
            self.step()
        self._drain_dp()
        return [self._output(r) for r in reqs]

    def stream(self, prompts: Sequence[Union[str, Sequence[int]]],
               params: Union[SamplingParams, Sequence[SamplingParams], None] = None):
        """Like generate, but yields (prompt index, new token ids) after every
        step that produced tokens for that prompt, then ("done", outputs)."""
        if params is None or isinstance(params, SamplingParams):
            params = [params or SamplingParams()] * len(prompts)
        reqs = [self.add_request(p, sp) for p, sp in zip(prompts, params)]
        sent = [0] * len(reqs)
        while any(not r.finished for r in reqs):
            self.step()
            for i, r in enumerate(reqs):
                if len(r.output) > sent[i]:
                    yield i, list(r.output[sent[i]:])
                    sent[i] = len(r.output)
        self._drain_dp()
        yield "done", [self._output(r) for r in reqs]

    def _drain_dp(self) -> None:
        if self.dp:
            # keep stepping (as an idle rank) until every rank is done
            while True:
                if self._cp_pending() and self._cp_agree():
                    self._cp_step()
                    continue
                if self._dp_forward(None) is None:
                    break

    # ------------------------------------------------------------------
    # Context-parallel prefill (DP attention): one long prompt on all ranks
    def _cp_check(self, params: SamplingParams, owner: int) -> None:
        if not self.cp:
            raise ValueError("context-parallel requests need EngineConfig(context_parallel=True)")
        if not getattr(self.model, "supports_cp", False):
            raise ValueError("this model family has no context-parallel prefill")
        if self.mtp is not None:
            raise ValueError("context-parallel prefill runs without the MTP draft module")
        if params.prompt_logprobs is not None:
            raise ValueError("context-parallel requests do not return prompt log-probabilities")
        if not 0 <= owner < self.ps.ep_size:
            raise ValueError(f"cp_owner {owner} is not a rank of the {self.ps.ep_size}-rank group")

    def _cp_pending(self) -> bool:
        """Whether the context-parallel queue holds a request.  The queue is
        the same on every rank (requests are added on all ranks between the
        same two steps and leave together), so ranks with an empty queue skip
        the agreement together and steps without context-parallel work cost
        no extra collective."""
        return self.cp and (self._cp_cur is not None or bool(self._cp_wait))

    def _cp_all(self) -> List[Request]:
        return ([self._cp_cur] if self._cp_cur is not None else []) + list(self._cp_wait)

    def _cp_drop(self, seq: int) -> None:
        """Drop the context-parallel request `seq` (an agreed abort)."""
        for r in self._cp_all():
            if r.cp_seq == seq:
                if r is self._cp_cur:
                    self._cp_cur = None
                else:
                    self._cp_wait.remove(r)
                if r.pages:
                    self.pool.release(r.pages)
                    r.pages = []
                r.finished, r.finish_reason, r.t_done = True, "abort", time.perf_counter()
                return

    def _cp_agree(self) -> bool:
        """Host agreement before each step: do all ranks hold the same
        context-parallel queue, does the head's prompt fit every rank's pool,
        is an abort pending.  True: this step prefills the head's next chunk."""
        import torch.distributed as dist
        from ..kv.pool import OutOfPages
        head = self._cp_cur or (self._cp_wait[0] if self._cp_wait else None)
        fail = 0
        if head is not None and not head.pages:
            need = self.pool.pages_for(len(head.prompt))
            if self.pool.num_free < need and self.radix is not None:
                self.radix.evict(need - self.pool.num_free)
            if self.pool.num_free < need:
                fail = 1
            else:
                head.pages = self.pool.alloc(need)
        n = len(self._cp_wait) + (self._cp_cur is not None)
        ab = max([r.cp_seq + 1 for r in self._cp_all() if r.cp_abort], default=0)
        v = torch.tensor([n, -n, fail, ab, int(self.sched.has_work)], dtype=torch.int64)
        dist.all_reduce(v, op=dist.ReduceOp.MAX, group=self.ps.cpu_group)
        n_max, n_min, any_fail, ab, busy = int(v[0]), -int(v[1]), int(v[2]), int(v[3]), int(v[4])
        if n_max != n_min:
            raise RuntimeError(f"ranks disagree on the context-parallel queue ({n_min} .. {n_max} requests): "
                               "every rank must add each context-parallel request")
        if ab:
            self._cp_drop(ab - 1)
            return False
        if n_max == 0:
            return False
        if any_fail:
            if head is not None and head is not self._cp_cur and head.pages:
                self.pool.release(head.pages)      # let this rank's running requests use them meanwhile
                head.pages = []
            if not busy:
                raise OutOfPages("a context-parallel prompt does not fit in some rank's KV pool")
            return False
        if self._cp_cur is None:
            self._cp_cur = self._cp_wait.popleft()
        return True

    def _cp_step(self) -> List[Request]:
        """Prefill the next chunk of the context-parallel head on every rank
        (this rank's rows: positions start + rank + k * W); after the last
        chunk the owner samples the first token and the request joins its
        running set (which may then hold max_num_seqs plus the
        context-parallel requests it decodes), the other ranks release their
        copy of the cache."""
        from ..parallel.cp import build_cp_batch, holder_of_last
        r = self._cp_cur
        W, me = self.ps.ep_size, self.ps.ep_rank
        start = r.cached
        n = min(len(r.prompt) - start, self.ecfg.max_prefill_tokens * W)
        fb = build_cp_batch(r.prompt, start, n, W, me, r.pages, self.ecfg.page_size)
        own = fb.cp.counts[me]
        m = self.model
        fb = self._to_device(fb)
        h = m._hidden(fb)
        if isinstance(h, tuple):          # the V4 family returns (hidden, batch)
            h, fb = h
        r.cached = start + n
        self.stats["steps"] += 1
        self.stats["prefill_tokens"] += own
        final = r.cached >= len(r.prompt)
        row = m._last_hidden(h, fb) if final else None
        self._check_device_errors()
        if not final:
            return []
        # the prompt's last row: broadcast from the rank that computed it
        row = self.ps.ep_all_gather(row.contiguous())[holder_of_last(n, W)].unsqueeze(0)
        self._cp_cur = None
        now = time.perf_counter()
        if me == r.cp_owner:
            logits = ops.lm_head_logits(row, m.lm_head, self.ps)
            st = Step("prefill", [r], [r.prompt[start:start + n]], [start], [True])
            toks = self._sample(st, logits)
            self._note_lp(st.reqs, logits, range(1), [toks[:1]], st.sample)
            self.sched.running.append(r)
            return self._emit(st, [toks[:1]], now)
        # a peer: its cache of the prompt goes to the prefix cache (or is freed)
        self.sched.release(r, cache_prefix=True)
        r.finished, r.finish_reason, r.t_done = True, "context_parallel_peer", now
        return [r]

    def _output(self, r: Request) -> GenerateOutput:
        n = len(r.output)
        tpot = (r.t_done - r.t_first) / (n - 1) if n > 1 else 0.0
        text = self.tokenizer.decode(r.output) if self.tokenizer is not None else None
        if text is not None and r.params.stop:
            cut = _stop_hit(text, r.params.stop)
            text = text if cut is None else text[:cut]
        return GenerateOutput(r.rid, len(r.prompt), list(r.output), r.finish_reason or "length",
                              (r.t_first or r.t_arrive) - r.t_arrive, tpot, text,
                              list(r.logprobs) if r.params.logprobs is not None else None,
                              list(r.prompt_lp) if r.params.prompt_logprobs is not None else None)
