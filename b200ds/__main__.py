"""Command line: `python -m b200ds <command>`.

    generate  --model M [--weights W] --prompt TEXT | --ids 1,2,3  [--max-tokens N]
              [--temperature T] [--top-p P] [--top-k K] [--seed S] [--device cpu|cuda]
    serve     (the OpenAI-compatible server; same options as b200ds.server.openai)
    presets   list the model presets
    switches  list the fast-path switches and their environment variables

Multi-GPU runs go through torchrun (one process per GPU), e.g.
`torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m b200ds serve --model DIR`.
"""
from __future__ import annotations

import argparse
import json
import sys


def _generate(argv) -> int:
    ap = argparse.ArgumentParser(prog="python -m b200ds generate")
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--weights", default="random")
    ap.add_argument("--prompt", default=None)
    ap.add_argument("--ids", default=None, help="comma-separated token ids")
    ap.add_argument("--max-tokens", type=int, default=16)
    ap.add_argument("--temperature", type=float, default=0.0)
    ap.add_argument("--top-p", type=float, default=1.0)
    ap.add_argument("--top-k", type=int, default=0)
    ap.add_argument("--seed", type=int, default=None)
    ap.add_argument("--logprobs", type=int, default=None, help="report each token's log-probability (+ top-n)")
    ap.add_argument("--presence-penalty", type=float, default=0.0)
    ap.add_argument("--frequency-penalty", type=float, default=0.0)
    ap.add_argument("--repetition-penalty", type=float, default=1.0)
    ap.add_argument("--guided-regex", default=None, help="constrain the output to this regular expression")
    ap.add_argument("--guided-choice", default=None, help="comma-separated allowed outputs")
    ap.add_argument("--device", default=None)
    ap.add_argument("--no-cuda-graphs", action="store_true")
    a = ap.parse_args(argv)
    from . import EngineConfig, SamplingParams, load_engine
    from .engine.tokenizer import load_tokenizer
    from .parallel.state import init_parallel
    ps = init_parallel()
    ecfg = EngineConfig(tp_size=ps.tp_size, ep_size=ps.ep_size, cuda_graphs=not a.no_cuda_graphs)
    eng = load_engine(a.model, weights=a.weights, ecfg=ecfg, device=a.device)
    tok = load_tokenizer(a.model)
    eng.tokenizer = eng.tokenizer or tok
    ids = [int(x) for x in a.ids.split(",")] if a.ids else tok.encode(a.prompt or "Hello")
    sp = SamplingParams(max_tokens=a.max_tokens, temperature=a.temperature, top_p=a.top_p, top_k=a.top_k,
                        seed=a.seed, logprobs=a.logprobs, presence_penalty=a.presence_penalty,
                        frequency_penalty=a.frequency_penalty, repetition_penalty=a.repetition_penalty,
                        guided_regex=a.guided_regex,
                        guided_choice=a.guided_choice.split(",") if a.guided_choice else None)
    out = eng.generate([ids], sp)[0]
    if ps.rank == 0:
        res = {"token_ids": out.token_ids, "text": tok.decode(out.token_ids), "finish_reason": out.finish_reason}
        if out.logprobs is not None:
            res["logprobs"] = [lp for _, lp, _ in out.logprobs]
        print(json.dumps(res))
    return 0


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        print(__doc__)
        return 0
    cmd, rest = argv[0], argv[1:]
    if cmd == "generate":
        return _generate(rest)
    if cmd == "serve":
        from .server.openai import main as serve
        serve(rest)
        return 0
    if cmd == "presets":
        from .config import PRESETS
        for name, fn in PRESETS.items():
            c = fn()
            print(f"{name:28s} {c.arch:12s} layers {c.num_hidden_layers:3d}  hidden {c.hidden_size:5d}  "
                  f"experts {c.n_routed_experts:4d}  params {c.num_params() / 1e9:8.1f} B")
        return 0
    if cmd == "switches":
        from .utils import levers
        for name, sw in sorted(levers._REGISTRY.items()):
            print(f"{name:14s} {sw.env:22s} default {'on' if sw.default else 'off':3s}  {sw.doc}")
        return 0
    print(f"unknown command {cmd!r}\n{__doc__}", file=sys.stderr)
    return 2


if __name__ == "__main__":
    sys.exit(main())
