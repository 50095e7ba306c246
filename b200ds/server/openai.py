"""OpenAI-compatible HTTP server.

Endpoints: POST /v1/completions, POST /v1/chat/completions (both with
``stream: true`` server-sent events, ``n``, ``stop`` strings and token ids,
``seed``, penalties, ``min_p`` / ``min_tokens``, ``max_completion_tokens``,
``stream_options.include_usage`` and log-probabilities: ``logprobs`` /
``top_logprobs``), POST /tokenize and /detokenize, GET /v1/models, GET
/health (503 after an engine failure or while a step overruns the watchdog),
GET /metrics (Prometheus text).

One engine thread owns the Engine and runs `step()` whenever requests are
pending; HTTP handlers enqueue requests and await their tokens through
per-request asyncio queues.  In a multi-GPU job rank 0 serves HTTP and, each
step, broadcasts newly admitted requests to the other ranks over the gloo
control group (`follower_loop` on ranks > 0), so every rank schedules the same
batches.

    python -m b200ds.server.openai --model deepseek-v3-671b --port 8000
    torchrun --nproc-per-node 8 -m b200ds.server.openai --model <ckpt dir>

Reference parity: the reference serves through SGLang's OpenAI server
(absent); request metrics mirror its TTFT / TPOT reporting (fg.py:68-73).
"""


import argparse
import asyncio
import json
import os
import queue
import threading
import time
import uuid
from typing import Dict, List, Optional

from ..engine.request import SamplingParams


class EngineWorker:
    """Runs Engine.step() on a background thread; thread-safe submission."""

    def __init__(self, engine, tokenizer, ps=None, watchdog_s: float = 0.0, watchdog_exit: bool = False):
        self.engine = engine
        self.tok = tokenizer
        self.ps = ps
        self.error: Optional[str] = None          # set when a step raised: the worker stops serving
        self.watchdog = None
        if watchdog_s > 0:
            from ..utils.watchdog import Watchdog
            self.watchdog = Watchdog(watchdog_s, exit_code=70 if watchdog_exit else None)
        self.inbox: "queue.Queue" = queue.Queue()
        self.cancels: "queue.Queue" = queue.Queue()     # subscription queues whose client went away
        self.commands: "queue.Queue" = queue.Queue()    # engine commands (kind, arg, loop, q): update / flush
        self.pending_update = None
        self.subs: Dict[int, tuple] = {}     # rid -> (loop, asyncio.Queue, emitted count)
        self._stop = threading.Event()
        self.t = threading.Thread(target=self._run, daemon=True)
        self.metrics = _Metrics()

    def start(self):
        self.t.start()
        return self

    def stop(self):
        self._stop.set()
        self.t.join(timeout=10)
        if self.watchdog is not None:
            self.watchdog.stop()

    def healthy(self) -> bool:
        return self.error is None and not (self.watchdog is not None and self.watchdog.stalled)

    def health(self) -> dict:
        if self.error is not None:
            return {"status": "error", "error": self.error}
        if self.watchdog is not None and self.watchdog.stalled:
            return {"status": "stalled", "error": f"engine step over {self.watchdog.timeout_s:.0f} s"}
        return {"status": "ok"}

    def submit(self, prompt_ids: List[int], params: SamplingParams, loop, q) -> None:
        if self.error is not None:
            _post(loop, q, ("error", self.error))
            return
        self.inbox.put((prompt_ids, params, loop, q))

    def request_update(self, path: str, loop, q) -> None:
        """Queue a weight update: admission pauses, the update runs on every
        rank once no request is in flight, the result is posted to q."""
        self.commands.put(("update", path, loop, q))

    def request_flush(self, loop, q) -> None:
        """Queue a prefix-cache flush (run like an update: idle, every rank)."""
        self.commands.put(("flush", None, loop, q))

    def _update_due(self) -> bool:
        """Pick up a queued update; True when one is pending and nothing is in flight."""
        if self.pending_update is None:
            try:
                self.pending_update = self.commands.get_nowait()
            except queue.Empty:
                return False
        return not self.subs and not self.engine.sched.has_work

    def _command_msg(self) -> dict:
        kind, arg = self.pending_update[:2]
        return {"new": [], "abort": [], kind: arg if kind == "update" else True}

    def _run_update(self) -> None:
        msg = self._command_msg()
        _, _, loop, q = self.pending_update
        self.pending_update = None
        _post(loop, q, _apply_command(self.engine, msg))

    def _step(self):
        """One engine step under the watchdog (when configured)."""
        if self.watchdog is None:
            return self.engine.step()
        with self.watchdog.guard():
            return self.engine.step()

    def _run(self):
        try:
            self._loop()
        except Exception as e:        # the engine failed: fail every request now instead of leaving it hanging
            import traceback
            traceback.print_exc()
            self._fail(f"{type(e).__name__}: {e}")

    def _fail(self, msg: str) -> None:
        self.error = msg
        for loop, q, *_ in list(self.subs.values()):
            _post(loop, q, ("error", msg))
        self.subs.clear()
        for _, _, loop, q in self._admit():
            _post(loop, q, ("error", msg))

    def cancel(self, q) -> None:
        """The client of subscription q is gone: abort its request."""
        self.cancels.put(q)

    def _cancelled(self) -> List[int]:
        """Keys of self.subs whose client is gone (drained from the cancel
        queue; subscriptions not admitted yet are aborted when they are)."""
        gone = []
        while True:
            try:
                gone.append(self.cancels.get_nowait())
            except queue.Empty:
                break
        if gone:
            self._pending_cancel = getattr(self, "_pending_cancel", []) + gone
        pend = getattr(self, "_pending_cancel", [])
        keys, keep = [], []
        for q in pend:
            k = next((key for key, sub in self.subs.items() if sub[1] is q), None)
            (keys if k is not None else keep).append(k if k is not None else q)
        self._pending_cancel = keep
        return keys

    def _admit(self) -> List[tuple]:
        new = []
        while True:
            try:
                new.append(self.inbox.get_nowait())
            except queue.Empty:
                break
        return new

    def _loop(self):
        eng = self.engine
        while not self._stop.is_set():
            if self._update_due():
                if self.ps is not None and self.ps.world_size > 1:
                    _broadcast_requests(self.ps, self._command_msg())
                self._run_update()
                continue
            new = []
            for prompt, params, loop, q in (self._admit() if self.pending_update is None else []):
                try:
                    r = eng.add_request(prompt, params)
                except ValueError as e:        # refused before it is queued (and never broadcast)
                    _post(loop, q, ("error", str(e)))
                    continue
                new.append((prompt, params, loop, q))
                self.subs[r.rid] = (loop, q, 0, r)
                self.metrics.requests += 1
            aborts = self._cancelled()
            if self.ps is not None and self.ps.world_size > 1:
                # followers mirror admissions in order, so rids agree across ranks
                _broadcast_requests(self.ps, {"new": [(p, sp.__dict__) for p, sp, _, _ in new], "abort": aborts})
            for rid in aborts:
                loop, q, _, r = self.subs.pop(rid)
                eng.abort(r)
                _post(loop, q, ("done", "abort"))
            if not eng.sched.has_work:
                time.sleep(0.002)
                continue
            t0 = time.perf_counter()
            self._step()
            self.metrics.step_time.append(time.perf_counter() - t0)
            for rid, (loop, q, sent, r) in list(self.subs.items()):
                alive = True
                if len(r.output) > sent:
                    new_toks = r.output[sent:]
                    lps = r.logprobs[sent:] if r.params.logprobs is not None else None
                    self.subs[rid] = (loop, q, len(r.output), r)
                    alive = _post(loop, q, ("tokens", new_toks, lps))
                if r.finished:
                    _post(loop, q, ("done", r.finish_reason,
                                    r.prompt_lp if r.params.prompt_logprobs is not None else None))
                    self.metrics.finish(r)
                    del self.subs[rid]
                elif not alive:               # the handler's event loop is gone
                    self.cancel(q)
        if self.ps is not None and self.ps.world_size > 1:
            _broadcast_requests(self.ps, None)      # followers stop


def _apply_command(engine, msg: dict) -> tuple:
    """An engine command on this rank: {"update": path} -> ("updated", bytes),
    {"flush": True} -> ("flushed", pages); ("error", why) on failure."""
    try:
        if msg.get("update"):
            return ("updated", engine.update_weights(msg["update"]))
        return ("flushed", engine.flush_cache())
    except (ValueError, OSError, KeyError) as e:
        return ("error", f"{type(e).__name__}: {e}")


def _post(loop, q, item) -> bool:
    """Hand an event to a request handler's event loop; False when that loop
    has closed (the client is gone)."""
    try:
        loop.call_soon_threadsafe(q.put_nowait, item)
        return True
    except RuntimeError:
        return False


def _broadcast_requests(ps, reqs):
    import torch.distributed as dist
    obj = [reqs]
    dist.broadcast_object_list(obj, src=0, group=ps.cpu_group)
    return obj[0]


class DPEngineWorker(EngineWorker):
    """DP attention serving: rank 0 takes the HTTP requests and assigns each
    to a rank round-robin; every rank serves its own requests and all ranks
    step in lockstep (the engine agrees on each step's shape); each step the
    ranks' new tokens are gathered to rank 0, which streams them out.
    Stopping broadcasts a sentinel that ends the followers' loops."""

    def __init__(self, engine, tokenizer, ps, **kw):
        super().__init__(engine, tokenizer, ps, **kw)
        self.next_gid = 0
        self.own: Dict[int, list] = {}      # gid -> [request, tokens sent]

    def _loop(self):
        eng, ps = self.engine, self.ps
        world = ps.world_size
        while not self._stop.is_set():
            if self._update_due():
                _broadcast_requests(ps, self._command_msg())
                self._run_update()
                continue
            new = self._admit() if self.pending_update is None else []
            batch = []
            for prompt, params, loop, q in new:
                try:
                    eng.check_request(prompt, params)
                except ValueError as e:        # refused before it is assigned to a rank
                    _post(loop, q, ("error", str(e)))
                    continue
                gid = self.next_gid
                self.next_gid += 1
                self.subs[gid] = (loop, q, 0, None)
                self.metrics.requests += 1
                batch.append((prompt, params.__dict__, gid % world, gid))
            aborts = self._cancelled()
            _broadcast_requests(ps, {"new": batch, "abort": aborts})
            _dp_admit(eng, ps, batch, self.own)
            _dp_abort(eng, aborts, self.own)
            for gid in aborts:
                loop, q, _, _ = self.subs.pop(gid)
                _post(loop, q, ("done", "abort"))
            t0 = time.perf_counter()
            self._step()
            if eng.sched.has_work:
                self.metrics.step_time.append(time.perf_counter() - t0)
            for upd in _dp_gather(ps, _dp_updates(self.own)):
                for gid, toks, fin, reason, r, lps, plp in upd:
                    if gid not in self.subs:     # aborted meanwhile
                        continue
                    loop, q, sent, _ = self.subs[gid]
                    alive = _post(loop, q, ("tokens", toks, lps)) if toks else True
                    if not alive and not fin:
                        self.cancel(q)
                    if fin and reason and reason.startswith("error: "):
                        _post(loop, q, ("error", reason[len("error: "):]))
                        del self.subs[gid]
                        continue
                    if fin:
                        _post(loop, q, ("done", reason, plp))
                        if r is not None:
                            self.metrics.finish(r)
                        del self.subs[gid]
            if not new and not self.subs:
                time.sleep(0.002)
        _broadcast_requests(ps, None)           # followers stop


def _dp_abort(eng, gids, own) -> None:
    for gid in gids:
        st = own.pop(gid, None)
        if st is not None:
            eng.abort(st[0])


class _Refused:
    """A request its owner rank could not queue (reported back as an error)."""

    def __init__(self, params, msg: str):
        self.params, self.output, self.logprobs, self.prompt_lp = params, [], [], []
        self.finished, self.finish_reason = True, "error: " + msg


def _dp_admit(eng, ps, batch, own) -> None:
    """Queue this rank's share of a broadcast batch.  With context
    parallelism on, prompts of at least cp_min_tokens are queued on every
    rank (all ranks prefill them; the assigned rank decodes and streams)."""
    for prompt, spd, owner, gid in batch:
        cp = getattr(eng, "cp", False) and len(prompt) >= eng.ecfg.cp_min_tokens
        if owner == ps.rank or cp:
            sp = SamplingParams(**spd)
            try:
                r = eng.add_request(prompt, sp, cp_owner=owner) if cp else eng.add_request(prompt, sp)
            except ValueError as e:
                r = _Refused(sp, str(e))
            if owner == ps.rank:
                own[gid] = [r, 0]


def _dp_updates(own) -> list:
    out = []
    for gid, st in list(own.items()):
        r, sent = st
        toks = r.output[sent:]
        lps = list(r.logprobs[sent:]) if r.params.logprobs is not None else None
        st[1] = len(r.output)
        if toks or r.finished:
            plp = list(r.prompt_lp) if r.finished and r.params.prompt_logprobs is not None else None
            out.append((gid, list(toks), r.finished, r.finish_reason, None, lps, plp))
        if r.finished:
            del own[gid]
    return out


def _dp_gather(ps, updates) -> list:
    import torch.distributed as dist
    objs = [None] * ps.world_size if ps.rank == 0 else None
    dist.gather_object(updates, objs, dst=0, group=ps.cpu_group)
    return objs if ps.rank == 0 else []


def dp_follower_loop(engine, ps) -> None:
    """DP ranks > 0: serve the requests assigned to this rank, step in
    lockstep with rank 0 and send it this rank's new tokens every step."""
    own: Dict[int, list] = {}
    while True:
        msg = _broadcast_requests(ps, None)
        if msg is None:
            return
        if msg.get("update") or msg.get("flush"):
            _apply_command(engine, msg)
            continue
        _dp_admit(engine, ps, msg["new"], own)
        _dp_abort(engine, msg["abort"], own)
        engine.step()
        _dp_gather(ps, _dp_updates(own))


def follower_loop(engine, ps) -> None:
    """Ranks > 0: mirror rank 0's admissions and step in lockstep (TP); DP
    attention engines serve their own share (dp_follower_loop)."""
    if getattr(engine, "dp", False):
        return dp_follower_loop(engine, ps)
    reqs_by_rid = {}
    while True:
        msg = _broadcast_requests(ps, None)
        if msg is None:
            return
        if msg.get("update") or msg.get("flush"):
            _apply_command(engine, msg)
            continue
        for prompt, spd in msg["new"]:
            r = engine.add_request(prompt, SamplingParams(**spd))
            reqs_by_rid[r.rid] = r
        for rid in msg["abort"]:
            r = reqs_by_rid.pop(rid, None)
            if r is not None:
                engine.abort(r)
        if len(reqs_by_rid) > 1024:
            reqs_by_rid = {k: r for k, r in reqs_by_rid.items() if not r.finished}
        if engine.sched.has_work:
            engine.step()


class _Metrics:
    def __init__(self):
        self.requests = 0
        self.completed = 0
        self.prompt_tokens = 0
        self.gen_tokens = 0
        self.ttft: List[float] = []
        self.tpot: List[float] = []
        self.step_time: List[float] = []

    def finish(self, r):
        self.completed += 1
        self.prompt_tokens += len(r.prompt)
        self.gen_tokens += len(r.output)
        if r.t_first is not None:
            self.ttft.append(r.t_first - r.t_arrive)
        if r.t_done is not None and len(r.output) > 1:
            self.tpot.append((r.t_done - r.t_first) / (len(r.output) - 1))

    def prometheus(self, engine_stats=None, switches=None, gauges=None) -> str:
        def q(xs, p):
            if not xs:
                return 0.0
            s = sorted(xs)
            return s[min(len(s) - 1, int(p * len(s)))]
        lines = [
            f"b200ds_requests_total {self.requests}",
            f"b200ds_requests_completed_total {self.completed}",
            f"b200ds_prompt_tokens_total {self.prompt_tokens}",
            f"b200ds_generation_tokens_total {self.gen_tokens}",
            f'b200ds_ttft_seconds{{quantile="0.5"}} {q(self.ttft, 0.5)}',
            f'b200ds_ttft_seconds{{quantile="0.99"}} {q(self.ttft, 0.99)}',
            f'b200ds_tpot_seconds{{quantile="0.5"}} {q(self.tpot, 0.5)}',
            f'b200ds_tpot_seconds{{quantile="0.99"}} {q(self.tpot, 0.99)}',
            f'b200ds_step_seconds{{quantile="0.5"}} {q(self.step_time[-1000:], 0.5)}',
        ]
        st = engine_stats or {}
        for k in ("steps", "prefill_tokens", "decode_tokens", "spec_proposed", "spec_accepted", "tbo_steps"):
            if k in st:
                lines.append(f"b200ds_engine_{k}_total {int(st[k])}")
        g = gauges or {}
        for k in ("running", "prefilling", "waiting", "kv_pages_total", "kv_pages_free", "cp_queue"):
            if k in g:
                lines.append(f"b200ds_{k} {int(g[k])}")
        for k in ("admitted_prompt_tokens", "prefix_hit_tokens", "preemptions", "host_offloads", "host_restores"):
            if k in g:
                lines.append(f"b200ds_{k}_total {int(g[k])}")
        if g.get("admitted_prompt_tokens"):
            lines.append(f"b200ds_prefix_cache_hit_ratio {g['prefix_hit_tokens'] / g['admitted_prompt_tokens']:.6f}")
        for k, v in sorted((switches or {}).items()):
            lines.append(f'b200ds_switch{{name="{k}"}} {int(bool(v))}')
        return "\n".join(lines) + "\n"


def _stop_scan(text: str, stops: List[str]):
    """(index of the first stop string in text or None, length of the longest
    text suffix that is a prefix of a stop string: held back from streaming)."""
    cut = None
    for st in stops:
        i = text.find(st)
        if i >= 0 and (cut is None or i < cut):
            cut = i
    hold = 0
    for st in stops:
        for n in range(min(len(st) - 1, len(text)), 0, -1):
            if text.endswith(st[:n]):
                hold = max(hold, n)
                break
    return cut, hold


def _logprobs_param(body: dict, chat: bool) -> Optional[int]:
    """OpenAI: completions take `logprobs` = number of alternatives (0-20);
    chat takes `logprobs: true` and `top_logprobs` (0-20)."""
    if chat:
        if not body.get("logprobs"):
            return None
        n = int(body.get("top_logprobs") or 0)
    else:
        if body.get("logprobs") is None or body.get("logprobs") is False:
            return None
        n = int(body["logprobs"])
    if not 0 <= n <= 20:
        raise ValueError("logprobs / top_logprobs must be between 0 and 20")
    return n


def _max_tokens(body: dict, default: int) -> int:
    """max_completion_tokens or max_tokens (0 allowed: the prompt only, e.g.
    with echo + logprobs to score it)."""
    v = body.get("max_completion_tokens")
    v = body.get("max_tokens") if v is None else v
    if v is None:
        return default
    v = int(v)
    if v < 0:
        raise ValueError("max_tokens must be >= 0")
    return v


def _logit_bias(body: dict):
    """OpenAI logit_bias: {token id (string or int): bias in [-100, 100]}."""
    lb = body.get("logit_bias")
    if not lb:
        return None
    if not isinstance(lb, dict):
        raise ValueError("logit_bias must map token ids to biases")
    out = {}
    for k, v in lb.items():
        v = float(v)
        if not -100.0 <= v <= 100.0:
            raise ValueError("logit_bias values must be in [-100, 100]")
        out[int(k)] = v
    return out


def _json_guide(body: dict):
    """guided_json (a schema) or response_format json_schema / json_object."""
    if body.get("guided_json") is not None:
        return body["guided_json"]
    rf = body.get("response_format") or {}
    if rf.get("type") == "json_schema":
        js = rf.get("json_schema") or {}
        return js.get("schema", js)
    if rf.get("type") == "json_object":
        return "object"
    return None


def _penalty_params(body: dict) -> dict:
    """presence_penalty / frequency_penalty (OpenAI, -2..2), repetition_penalty
    (> 0), min_p (0..1), min_tokens (>= 0)."""
    def num(name, default, lo, hi, cast=float):
        v = body.get(name)
        if v is None:
            return default
        v = cast(v)
        if not lo <= v <= hi:
            raise ValueError(f"{name} must be in [{lo}, {hi}]")
        return v
    return dict(presence_penalty=num("presence_penalty", 0.0, -2.0, 2.0),
                frequency_penalty=num("frequency_penalty", 0.0, -2.0, 2.0),
                repetition_penalty=num("repetition_penalty", 1.0, 1e-3, 100.0),
                min_p=num("min_p", 0.0, 0.0, 1.0),
                min_tokens=num("min_tokens", 0, 0, 1 << 30, int))


def _lp_json(tok, lps, chat: bool, offset: int = 0, prompt=None) -> dict:
    """Engine log-probabilities -> the OpenAI response field (chat: `content`
    entries with token, logprob, bytes, top_logprobs; completions: parallel
    tokens / token_logprobs / top_logprobs / text_offset lists)."""
    if chat:
        def ent(t, lp):
            s = tok.decode([t])
            return {"token": s, "logprob": lp, "bytes": list(s.encode("utf-8")), "token_id": t}
        return {"content": [dict(ent(t, lp), top_logprobs=[ent(a, alp) for a, alp in top]) for t, lp, top in lps]}
    toks, offs, vals, tops = [], [], [], []
    ent = list(lps)
    if prompt is not None:            # echo: the prompt's tokens first (the first one has no log-probability)
        ids, plp = prompt
        plp = plp or [None] * len(ids)
        ent = [(t, None, None) if e is None else e for t, e in zip(ids, plp)] + ent
    for t, lp, top in ent:
        s = tok.decode([t])
        toks.append(s)
        offs.append(offset)
        offset += len(s)
        vals.append(lp)
        tops.append(None if top is None else {tok.decode([a]): alp for a, alp in top})
    return {"tokens": toks, "token_logprobs": vals, "top_logprobs": tops, "text_offset": offs}


def _params(body: dict, default_max: int = 16, chat: bool = False) -> SamplingParams:
    stop_ids = body.get("stop_token_ids") or []
    return SamplingParams(
        max_tokens=_max_tokens(body, default_max),
        temperature=float(body.get("temperature", 1.0) if body.get("temperature") is not None else 1.0),
        top_p=float(body.get("top_p", 1.0) or 1.0),
        top_k=int(body.get("top_k", 0) or 0),
        seed=body.get("seed"),
        ignore_eos=bool(body.get("ignore_eos", False)),
        stop_token_ids=list(stop_ids),
        logprobs=_logprobs_param(body, chat),
        prompt_logprobs=(_logprobs_param(body, chat) if body.get("echo") and not chat else None),
        priority=int(body.get("priority") or 0),
        logit_bias=_logit_bias(body),
        guided_regex=body.get("guided_regex", body.get("regex")),
        guided_choice=body.get("guided_choice"),
        guided_json=_json_guide(body),
        **_penalty_params(body),
    )


def create_app(worker: EngineWorker, model_name: str = "b200ds", reasoning: bool = False,
               api_key: Optional[str] = None):
    """The HTTP app.  reasoning: chat answers are split into
    reasoning_content and content at "</think>" (DeepSeek-R1 style; streamed
    as reasoning_content / content deltas)."""
    from .parsers import parse_tool_calls, split_reasoning, stream_reasoning
    from fastapi import FastAPI, HTTPException, Request
    from fastapi.responses import JSONResponse, PlainTextResponse, StreamingResponse

    app = FastAPI(title="b200ds")

    if api_key:
        import hmac

        @app.middleware("http")
        async def _auth(request, call_next):
            """Every endpoint but /health needs `Authorization: Bearer <api key>`."""
            if request.url.path != "/health":
                got = request.headers.get("authorization", "")
                if not hmac.compare_digest(got.encode(), f"Bearer {api_key}".encode()):
                    return JSONResponse({"error": {"message": "invalid API key", "type": "auth_error"}},
                                        status_code=401)
            return await call_next(request)
    tok = worker.tok

    async def _run(prompt_ids, params):
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        worker.submit(prompt_ids, params, loop, q)
        return q

    def _prompt_ids(body, chat: bool):
        if chat:
            msgs = body.get("messages")
            if not isinstance(msgs, list):
                raise HTTPException(400, "messages must be a list")
            return tok.encode_chat(msgs, body.get("tools"))
        p = body.get("prompt")
        if isinstance(p, list) and all(isinstance(i, int) for i in p):
            return p
        if isinstance(p, list) and len(p) == 1 and isinstance(p[0], str):
            p = p[0]
        if not isinstance(p, str):
            raise HTTPException(400, "prompt must be a string or a list of token ids")
        return tok.encode(p)

    async def _collect(q, stops):
        """Tokens of one subscription until it finishes (or a stop string
        appears): (token ids, text, finish reason, log-probabilities, prompt
        log-probabilities)."""
        out: List[int] = []
        lps: List[tuple] = []
        plp = None
        reason = "length"
        text = None
        try:
            while True:
                ev = await q.get()
                kind, val = ev[0], ev[1]
                if kind == "error":
                    raise HTTPException(500, f"engine error: {val}")
                if kind == "tokens":
                    out.extend(val)
                    if len(ev) > 2 and ev[2]:
                        lps.extend(ev[2])
                    if stops:
                        cut, _ = _stop_scan(tok.decode(out), stops)
                        if cut is not None:
                            text, reason = tok.decode(out)[:cut], "stop"
                            worker.cancel(q)
                            break
                else:
                    reason = val
                    plp = ev[2] if len(ev) > 2 else None
                    break
        except HTTPException:
            raise
        except BaseException:              # cancelled (client gone)
            worker.cancel(q)
            raise
        return out, (tok.decode(out) if text is None else text), reason, lps, plp

    async def _handle(request: Request, chat: bool):
        if not worker.healthy():
            raise HTTPException(503, f"engine unavailable: {worker.health().get('error')}")
        body = await request.json()
        ids = _prompt_ids(body, chat)
        try:
            params = _params(body, chat=chat)
            worker.engine.check_request(ids, params)
        except ValueError as e:
            raise HTTPException(400, str(e))
        rid = f"{'chatcmpl' if chat else 'cmpl'}-{uuid.uuid4().hex[:16]}"
        created = int(time.time())
        n = int(body.get("n") or 1)
        if n < 1:
            raise HTTPException(400, "n must be >= 1")
        obj = "chat.completion" if chat else "text_completion"
        stops = body.get("stop") or []
        stops = [stops] if isinstance(stops, str) else [x for x in stops if isinstance(x, str) and x]

        echo = bool(body.get("echo")) and not chat

        tools = chat and bool(body.get("tools"))

        def _choice(i, out, text, reason, lps, plp=None):
            if echo:
                text = tok.decode(ids) + text
            if chat:
                msg = {"role": "assistant", "content": text}
                if tools:                     # the tool-call markers are special tokens: decode them too
                    msg["content"], calls = parse_tool_calls(tok.decode(out, keep_special=True))
                    if calls:
                        msg["tool_calls"] = calls
                        msg["content"] = msg["content"] or None
                        reason = "tool_calls"
                if reasoning and isinstance(msg["content"], str):
                    msg["reasoning_content"], msg["content"] = split_reasoning(msg["content"])
                c = {"index": i, "message": msg, "finish_reason": reason}
            else:
                c = {"index": i, "text": text, "token_ids": out, "finish_reason": reason}
            if params.logprobs is not None:
                c["logprobs"] = _lp_json(tok, lps, chat, prompt=(ids, plp) if echo else None)
            return c
        if n > 1 and not body.get("stream"):
            # n independent samples of the prompt (seed + i when a seed is given)
            import dataclasses
            qs = [await _run(ids, dataclasses.replace(params, seed=None if params.seed is None else params.seed + i))
                  for i in range(n)]
            results = [await _collect(q, stops) for q in qs]
            choices = [_choice(i, *res) for i, res in enumerate(results)]
            gen_tok = sum(len(res[0]) for res in results)
            return JSONResponse({"id": rid, "object": obj, "created": created, "model": model_name,
                                 "choices": choices, "usage": {"prompt_tokens": len(ids), "completion_tokens": gen_tok,
                                                               "total_tokens": len(ids) + gen_tok}})
        if body.get("stream"):
            import dataclasses
            qs = [await _run(ids, params if n == 1 else dataclasses.replace(
                params, seed=None if params.seed is None else params.seed + i)) for i in range(n)]
            counts = [0] * n
            usage = bool((body.get("stream_options") or {}).get("include_usage"))

            def _final() -> str:
                """Closing events: the usage chunk (stream_options.include_usage)
                and [DONE]."""
                tail = "data: [DONE]\n\n"
                if not usage:
                    return tail
                n_out = sum(counts)
                u = {"prompt_tokens": len(ids), "completion_tokens": n_out, "total_tokens": len(ids) + n_out}
                ev = {"id": rid, "object": obj + ".chunk", "created": created, "model": model_name,
                      "choices": [], "usage": u}
                return f"data: {json.dumps(ev)}\n\n" + tail

            def _ev(choice) -> str:
                return f"data: {json.dumps({'id': rid, 'object': obj + '.chunk', 'created': created, 'model': model_name, 'choices': [choice]})}\n\n"

            async def _chunks(q, idx):
                """Events of choice idx until it finishes."""
                ids_all: List[int] = []
                sent = 0                      # characters of the decoded text already streamed
                r_sent = a_sent = 0           # reasoning / answer characters streamed (reasoning parser)
                if echo:                      # the prompt's text first
                    yield _ev({"index": idx, "text": tok.decode(ids), "token_ids": [], "finish_reason": None})
                while True:
                    ev = await q.get()
                    kind, val = ev[0], ev[1]
                    if kind == "error":
                        yield f"data: {json.dumps({'error': {'message': f'engine error: {val}', 'type': 'server_error'}})}\n\n"
                        return
                    if kind == "tokens":
                        lp_field = None
                        if params.logprobs is not None and len(ev) > 2 and ev[2]:
                            lp_field = _lp_json(tok, ev[2], chat, len(tok.decode(ids_all)))
                        ids_all.extend(val)
                        counts[idx] = len(ids_all)
                        full = tok.decode(ids_all)
                        cut, hold = _stop_scan(full, stops)
                        end = cut if cut is not None else len(full) - hold
                        text = full[sent:end] if end > sent else ""
                        sent = max(sent, end)
                        if chat and reasoning:      # deltas split into reasoning_content / content
                            rs, ans = stream_reasoning(full[:end])
                            delta = {}
                            if len(rs) > r_sent:
                                delta["reasoning_content"] = rs[r_sent:]
                            if len(ans) > a_sent:
                                delta["content"] = ans[a_sent:]
                            r_sent, a_sent = max(r_sent, len(rs)), max(a_sent, len(ans))
                            if delta:
                                yield _ev({"index": idx, "delta": delta, "finish_reason": None})
                        elif text or cut is None:
                            choice = ({"index": idx, "delta": {"content": text}, "finish_reason": None} if chat
                                      else {"index": idx, "text": text, "token_ids": val, "finish_reason": None})
                            if lp_field is not None:
                                choice["logprobs"] = lp_field
                            yield _ev(choice)
                        if cut is not None:     # a stop string: finish now and free the request
                            worker.cancel(q)
                            yield _ev({"index": idx, "delta": {}, "finish_reason": "stop"} if chat
                                      else {"index": idx, "text": "", "finish_reason": "stop"})
                            return
                    else:
                        yield _ev({"index": idx, "delta": {}, "finish_reason": val} if chat
                                  else {"index": idx, "text": "", "finish_reason": val})
                        return

            async def gen():
                finished = [False] * n
                try:
                    if n == 1:
                        async for chunk in _chunks(qs[0], 0):
                            yield chunk
                        finished[0] = True
                    else:                     # the choices' events interleaved as they come
                        merged: asyncio.Queue = asyncio.Queue()

                        async def pump(i):
                            async for chunk in _chunks(qs[i], i):
                                await merged.put(chunk)
                            finished[i] = True
                            await merged.put(None)
                        tasks = [asyncio.ensure_future(pump(i)) for i in range(n)]
                        left = n
                        while left:
                            chunk = await merged.get()
                            if chunk is None:
                                left -= 1
                            else:
                                yield chunk
                        await asyncio.gather(*tasks)
                    yield _final()
                finally:
                    for i, q in enumerate(qs):
                        if not finished[i]:   # client disconnected: free the request
                            worker.cancel(q)
            return StreamingResponse(gen(), media_type="text/event-stream")
        q = await _run(ids, params)
        res = await _collect(q, stops)
        out = res[0]
        choice = _choice(0, *res)
        return JSONResponse({"id": rid, "object": obj, "created": created, "model": model_name, "choices": [choice],
                             "usage": {"prompt_tokens": len(ids), "completion_tokens": len(out),
                                       "total_tokens": len(ids) + len(out)}})

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await _handle(request, chat=False)

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        return await _handle(request, chat=True)

    @app.get("/v1/models")
    async def models():
        return {"object": "list", "data": [{"id": model_name, "object": "model", "owned_by": "b200ds"}]}

    # ---- SGLang-native endpoints (the reference's clients talk to SGLang) ----
    def _sgl_params(sp: dict) -> SamplingParams:
        body = {"max_tokens": sp.get("max_new_tokens", 128), "temperature": sp.get("temperature", 1.0),
                "top_p": sp.get("top_p"), "top_k": sp.get("top_k") if (sp.get("top_k") or 0) > 0 else 0,
                "seed": sp.get("sampling_seed", sp.get("seed")), "ignore_eos": sp.get("ignore_eos", False),
                "stop_token_ids": sp.get("stop_token_ids"), "presence_penalty": sp.get("presence_penalty"),
                "frequency_penalty": sp.get("frequency_penalty"),
                "repetition_penalty": sp.get("repetition_penalty"), "min_p": sp.get("min_p"),
                "min_tokens": sp.get("min_new_tokens"), "regex": sp.get("regex"),
                "guided_json": (json.loads(sp["json_schema"]) if isinstance(sp.get("json_schema"), str)
                                else sp.get("json_schema"))}
        return _params({k: v for k, v in body.items() if v is not None}, default_max=128)

    @app.post("/generate")
    async def generate(request: Request):
        """SGLang's /generate: {"text" | "input_ids" (one or a batch),
        "sampling_params": {max_new_tokens, temperature, top_p, top_k, stop,
        stop_token_ids, ignore_eos, penalties, min_new_tokens, regex,
        json_schema}, "stream"} -> {"text", "output_ids", "meta_info"}."""
        if not worker.healthy():
            raise HTTPException(503, f"engine unavailable: {worker.health().get('error')}")
        body = await request.json()
        batch = body.get("input_ids") if body.get("input_ids") is not None else body.get("text")
        single = not (isinstance(batch, list) and batch and isinstance(batch[0], (list, str)))
        items = [batch] if single else batch
        sp = body.get("sampling_params") or {}
        try:
            params = _sgl_params(sp)
            if body.get("return_logprob"):
                import dataclasses
                params = dataclasses.replace(params, logprobs=int(body.get("top_logprobs_num") or 0))
            prompts = [tok.encode(x) if isinstance(x, str) else list(x) for x in items]
            for ids in prompts:
                worker.engine.check_request(ids, params)
        except (ValueError, TypeError) as e:
            raise HTTPException(400, str(e))
        stops = sp.get("stop") or []
        stops = [stops] if isinstance(stops, str) else list(stops)

        def meta(ids, out, reason, lps=None):
            fr = {"type": "stop"} if reason == "stop" else {"type": reason}
            m = {"prompt_tokens": len(ids), "completion_tokens": len(out), "finish_reason": fr}
            if lps is not None and params.logprobs is not None:
                # SGLang's layout: [logprob, token id, text]
                m["output_token_logprobs"] = [[lp, t, None] for t, lp, _ in lps]
                if params.logprobs > 0:
                    m["output_top_logprobs"] = [[[alp, a, None] for a, alp in top] for _, _, top in lps]
            return m
        if body.get("stream"):
            if not single:
                raise HTTPException(400, "stream takes one prompt")
            q = await _run(prompts[0], params)

            async def gen():
                out, done = [], False
                try:
                    while True:
                        ev = await q.get()
                        if ev[0] == "error":
                            yield f"data: {json.dumps({'error': {'message': ev[1]}})}\n\n"
                            break
                        if ev[0] == "tokens":
                            out.extend(ev[1])
                            text = tok.decode(out)
                            cut, _ = _stop_scan(text, stops) if stops else (None, 0)
                            if cut is not None:
                                worker.cancel(q)
                                yield f"data: {json.dumps({'text': text[:cut], 'output_ids': out, 'meta_info': meta(prompts[0], out, 'stop')})}\n\n"
                                break
                            yield f"data: {json.dumps({'text': text, 'output_ids': out, 'meta_info': meta(prompts[0], out, None)})}\n\n"
                        else:
                            yield f"data: {json.dumps({'text': tok.decode(out), 'output_ids': out, 'meta_info': meta(prompts[0], out, ev[1])})}\n\n"
                            break
                    done = True
                    yield "data: [DONE]\n\n"
                finally:
                    if not done:
                        worker.cancel(q)
            return StreamingResponse(gen(), media_type="text/event-stream")
        qs = [await _run(ids, params) for ids in prompts]
        res = []
        for ids, q in zip(prompts, qs):
            out, text, reason, lps, _ = await _collect(q, stops)
            res.append({"text": text, "output_ids": out, "meta_info": meta(ids, out, reason, lps)})
        return res[0] if single else res

    @app.get("/get_model_info")
    async def get_model_info():
        c = worker.engine.cfg
        return {"model_path": model_name, "tokenizer_path": model_name, "is_generation": True,
                "architecture": c.arch, "num_params": c.num_params()}

    @app.get("/get_server_info")
    async def get_server_info():
        import dataclasses
        e = worker.engine
        return {"engine_config": dataclasses.asdict(e.ecfg), "model_config": e.cfg.to_dict(),
                "tp_size": e.ps.tp_size, "ep_size": e.ps.ep_size, "dp_attention": bool(e.dp)}

    @app.post("/update_weights_from_disk")
    async def update_weights(request: Request):
        """{"model_path": checkpoint dir}: new weights of the same architecture,
        loaded in place once the requests in flight have finished."""
        body = await request.json()
        path = body.get("model_path")
        if not isinstance(path, str):
            raise HTTPException(400, "model_path must be a checkpoint directory")
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        worker.request_update(path, loop, q)
        kind, val = await q.get()
        if kind == "error":
            raise HTTPException(400, val)
        return {"success": True, "bytes": int(val)}

    @app.post("/flush_cache")
    async def flush_cache():
        """Clear the prefix cache (on the engine thread, once no request is in
        flight, on every rank)."""
        loop = asyncio.get_running_loop()
        q: asyncio.Queue = asyncio.Queue()
        worker.request_flush(loop, q)
        kind, val = await q.get()
        if kind == "error":
            raise HTTPException(409, val)
        return {"success": True, "pages": int(val)}

    @app.post("/tokenize")
    async def tokenize(request: Request):
        """{"prompt": text} or {"messages": [...]} -> token ids (chat template applied)."""
        body = await request.json()
        ids = _prompt_ids(body, chat="messages" in body)
        return {"tokens": ids, "count": len(ids)}

    @app.post("/detokenize")
    async def detokenize(request: Request):
        body = await request.json()
        t = body.get("tokens")
        if not isinstance(t, list) or not all(isinstance(i, int) for i in t):
            raise HTTPException(400, "tokens must be a list of token ids")
        return {"prompt": tok.decode(t)}

    @app.get("/health")
    async def health():
        h = worker.health()
        return h if h["status"] == "ok" else JSONResponse(h, status_code=503)

    @app.get("/metrics")
    async def metrics():
        from ..utils import levers
        return PlainTextResponse(worker.metrics.prometheus(worker.engine.stats, levers.switches(),
                                                           worker.engine.gauges()))

    return app


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny", help="preset name or HF checkpoint directory")
    ap.add_argument("--weights", default="random")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--max-num-seqs", type=int, default=256)
    ap.add_argument("--no-cuda-graphs", action="store_true")
    ap.add_argument("--dp-attention", action="store_true", help="DP attention + EP experts over all ranks")
    ap.add_argument("--max-model-len", type=int, default=16384)
    ap.add_argument("--no-prefix-cache", action="store_true")
    ap.add_argument("--spec-ngram", type=int, default=0, help="n-gram speculative decoding (max n)")
    ap.add_argument("--spec-mtp", action="store_true", help="speculative decoding with the model's MTP module")
    ap.add_argument("--spec-k", type=int, default=4, help="draft tokens verified per step")
    ap.add_argument("--trace", action="store_true", help="device timestamps per layer phase")
    ap.add_argument("--mixed-steps", action="store_true", help="decode tokens ride along with prefill chunks")
    ap.add_argument("--context-parallel", action="store_true",
                    help="with --dp-attention: long prompts prefill on every rank")
    ap.add_argument("--cp-min-tokens", type=int, default=8192, help="shortest prompt that prefills context-parallel")
    ap.add_argument("--tbo", action="store_true",
                    help="with --dp-attention: two-batch overlap of prefill steps (MoE exchange vs compute)")
    ap.add_argument("--extend-graphs", action="store_true", help="replay prefill chunks from CUDA graphs")
    ap.add_argument("--page-size", type=int, default=64, help="tokens per KV page")
    ap.add_argument("--max-prefill-tokens", type=int, default=16384, help="chunked-prefill budget per step")
    ap.add_argument("--kv-cache-fraction", type=float, default=0.85, help="of free HBM after weights")
    ap.add_argument("--graph-batch-sizes", default="1,2,4,8,16,32,64,128,256",
                    help="decode CUDA-graph batch buckets (comma-separated)")
    ap.add_argument("--no-prefill-tail", action="store_true", help="window-only late layers on every prefill row")
    ap.add_argument("--host-kv-pages", type=int, default=0,
                    help="pinned host pages behind the prefix cache (evicted pages move there)")
    ap.add_argument("--schedule-policy", choices=("fcfs", "lpm", "priority"), default="fcfs",
                    help="admission order: arrival, longest cached prefix first, or request priority")
    ap.add_argument("--comm", choices=("fused", "nccl"), default="fused",
                    help="fused NVLink collectives or the NCCL baseline")
    ap.add_argument("--watchdog-timeout", type=float, default=300.0,
                    help="seconds one engine step may run before /health reports a stall (0: off)")
    ap.add_argument("--watchdog-exit", action="store_true", help="exit the process when the watchdog fires")
    ap.add_argument("--api-key", default=os.environ.get("B200_API_KEY"),
                    help="require `Authorization: Bearer <key>` (also B200_API_KEY)")
    ap.add_argument("--reasoning-parser", choices=("deepseek-r1",), default=None,
                    help="split chat answers into reasoning_content and content")
    args = ap.parse_args(argv)
    import uvicorn
    from .. import load_engine
    from ..config import EngineConfig
    from ..engine.tokenizer import load_tokenizer
    from ..parallel.state import init_parallel
    ps = init_parallel(dp_attention=args.dp_attention)
    ecfg = EngineConfig(tp_size=1 if args.dp_attention else ps.tp_size, ep_size=ps.ep_size,
                        dp_attention=args.dp_attention, max_num_seqs=args.max_num_seqs,
                        cuda_graphs=not args.no_cuda_graphs, max_model_len=args.max_model_len,
                        enable_prefix_cache=not (args.no_prefix_cache or args.spec_mtp),
                        spec_ngram=args.spec_ngram, spec_mtp=args.spec_mtp, spec_k=args.spec_k, trace=args.trace,
                        mixed_steps=args.mixed_steps, extend_graphs=args.extend_graphs, page_size=args.page_size,
                        max_prefill_tokens=args.max_prefill_tokens, kv_cache_fraction=args.kv_cache_fraction,
                        graph_batch_sizes=tuple(int(x) for x in args.graph_batch_sizes.split(",") if x),
                        prefill_tail=not args.no_prefill_tail, comm_impl=args.comm,
                        schedule_policy=args.schedule_policy, host_kv_pages=args.host_kv_pages,
                        context_parallel=args.context_parallel, cp_min_tokens=args.cp_min_tokens, tbo=args.tbo)
    eng = load_engine(args.model, weights=args.weights, ecfg=ecfg)
    tok = load_tokenizer(args.model)
    eng.tokenizer = tok
    eng.eos = getattr(tok, "eos_token_id", None)
    if ps.rank != 0:
        follower_loop(eng, ps)
        return
    wd = dict(watchdog_s=args.watchdog_timeout, watchdog_exit=args.watchdog_exit)
    worker = (DPEngineWorker(eng, tok, ps, **wd) if eng.dp else EngineWorker(eng, tok, ps, **wd)).start()
    uvicorn.run(create_app(worker, model_name=str(args.model), reasoning=args.reasoning_parser is not None,
                           api_key=args.api_key),
                host=args.host, port=args.port, log_level="warning")


if __name__ == "__main__":
    main()
