"""Serving benchmark: concurrent streamed requests against the OpenAI-compatible
server, measured from the client the way serving benchmarks report them.

    python -m b200ds serve --model deepseek-v3-671b ... &      (or torchrun ...)
    python benchmarks/serving.py --url http://127.0.0.1:8000 --num-prompts 256 \
        --concurrency 64 --input-len 1024 --output-len 1024

Prompts are uniform-random token ids (seed 0) sent as token lists to
/v1/completions with stream, ignore_eos and max_tokens = output-len.  Per
request: TTFT (time to the first streamed token), TPOT ((end - first token)
/ (tokens - 1)), end-to-end latency; whole run: output tokens/s, requests/s.
One JSON line on stdout.

Reference parity: the reference quotes engine TTFT measured by an external
client (fg.py:68-73, 139-142); this client measures TTFT / TPOT / output
throughput over HTTP the same way for this server.
"""
from __future__ import annotations

import argparse
import asyncio
import json
import random
import time
from typing import List


def _pct(xs: List[float], p: float) -> float:
    if not xs:
        return 0.0
    xs = sorted(xs)
    return xs[min(len(xs) - 1, int(round(p / 100 * (len(xs) - 1))))]


async def _one(session, url: str, prompt: List[int], out_len: int, temperature: float) -> dict:
    body = {"prompt": prompt, "max_tokens": out_len, "temperature": temperature, "stream": True,
            "ignore_eos": True}
    t0 = time.perf_counter()
    first, n, err = None, 0, None
    async with session.post(url + "/v1/completions", json=body) as r:
        if r.status != 200:
            return {"ok": False, "error": f"HTTP {r.status}: {await r.text()}"}
        async for raw in r.content:
            line = raw.decode().strip()
            if not line.startswith("data: ") or line == "data: [DONE]":
                continue
            ev = json.loads(line[6:])
            if "error" in ev:
                err = ev["error"].get("message")
                break
            k = len(ev["choices"][0].get("token_ids") or [])
            if k and first is None:
                first = time.perf_counter()
            n += k
    t1 = time.perf_counter()
    if err is not None or first is None:
        return {"ok": False, "error": err or "no tokens"}
    return {"ok": True, "ttft": first - t0, "latency": t1 - t0, "tokens": n,
            "tpot": (t1 - first) / (n - 1) if n > 1 else 0.0}


async def run(url: str, num_prompts: int, concurrency: int, input_len: int, output_len: int, vocab: int,
              temperature: float = 0.0, seed: int = 0) -> dict:
    import aiohttp
    rng = random.Random(seed)
    prompts = [[rng.randrange(vocab) for _ in range(input_len)] for _ in range(num_prompts)]
    sem = asyncio.Semaphore(concurrency)
    timeout = aiohttp.ClientTimeout(total=None, sock_read=None)
    async with aiohttp.ClientSession(timeout=timeout) as session:
        async def guarded(p):
            async with sem:
                return await _one(session, url, p, output_len, temperature)
        t0 = time.perf_counter()
        res = await asyncio.gather(*(guarded(p) for p in prompts))
        wall = time.perf_counter() - t0
    ok = [r for r in res if r["ok"]]
    toks = sum(r["tokens"] for r in ok)
    ms = lambda xs, p: round(_pct(xs, p) * 1e3, 3)
    ttft = [r["ttft"] for r in ok]
    tpot = [r["tpot"] for r in ok if r["tokens"] > 1]
    return {"metric": "serving output tok/s (client-measured, streamed)", "output_tok_s": round(toks / wall, 2),
            "requests_s": round(len(ok) / wall, 3), "completed": len(ok), "failed": len(res) - len(ok),
            "output_tokens": toks,
            "errors": sorted({r["error"] for r in res if not r["ok"]})[:3],
            "ttft_ms": {"p50": ms(ttft, 50), "p90": ms(ttft, 90), "p99": ms(ttft, 99)},
            "tpot_ms": {"p50": ms(tpot, 50), "p90": ms(tpot, 90), "p99": ms(tpot, 99)},
            "wall_s": round(wall, 3), "config": {"num_prompts": num_prompts, "concurrency": concurrency,
                                                 "input_len": input_len, "output_len": output_len,
                                                 "temperature": temperature, "data": "uniform-random token ids"}}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--url", default="http://127.0.0.1:8000")
    ap.add_argument("--num-prompts", type=int, default=64)
    ap.add_argument("--concurrency", type=int, default=64)
    ap.add_argument("--input-len", type=int, default=1024)
    ap.add_argument("--output-len", type=int, default=1024)
    ap.add_argument("--vocab", type=int, default=129280)
    ap.add_argument("--temperature", type=float, default=0.0)
    a = ap.parse_args(argv)
    out = asyncio.run(run(a.url.rstrip("/"), a.num_prompts, a.concurrency, a.input_len, a.output_len, a.vocab,
                          a.temperature))
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
