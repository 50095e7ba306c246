#!/usr/bin/env python
"""Headline benchmark: DeepSeek-V3-shaped 671B decoder serving 64 concurrent
requests (1024 uniform-random input tokens each, seed 0, ignore_eos),
random-init fp8 weights, TP=N attention + EP=N MoE on N GPUs of one node.

    python bench.py --gpus 1 --steps 20 --warmup 3
    torchrun --nproc-per-node 8 ... bench.py --gpus 8 --steps 20 --warmup 3

Prints ONE JSON line (rank 0).  `value` = output tokens/s of the whole job
from K back-to-back replays of the captured decode step (CUDA events, max
over ranks, inputs already on the device); `e2e.value` = the same metric
through the public API (Engine.step: host scheduling, pinned H2D of the
step's inputs, graph replay, D2H of the sampled ids) over K further steps.
Prefill of the 64 prompts (untimed for `value`) gives TTFT.

Data / weights: synthetic uniform-random token ids and random-init weights
of the named architecture.  Per-step weights (>= 1.4 GB of routed experts
per MoE layer) and KV exceed the 126 MB L2, so no flush is needed.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HEADLINE_METRIC = "output tok/s/GPU on 8xB200 (device-timed, max over ranks); p50 TPOT, TTFT"


class ClockSampler:
    """Samples SM clocks and clock-event (throttle) reasons of this rank's GPU
    every 20 ms during the timed region through NVML (read-only queries);
    falls back to nvidia-smi every 200 ms without NVML."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown"}

    def __init__(self, index: int):
        self.index = index
        self.samples = []            # (sm_mhz, max_mhz, reason bitmask)
        self._stop = threading.Event()
        self._t = None
        self._nvml = None
        try:
            import pynvml
            pynvml.nvmlInit()
            h = None
            try:
                import torch
                pr = torch.cuda.get_device_properties(index)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self._nvml = (pynvml, h)
        except Exception:
            self._nvml = None

    def _sample_nvml(self):
        nv, h = self._nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        try:
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        except Exception:
            rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
        self.samples.append((float(sm), float(mx), int(rs)))

    def _sample_smi(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={q}", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=5).stdout.strip()
        f = [x.strip() for x in out.split(",")]
        bits = [0x8, 0x40, 0x20, 0x4]
        rs = sum(b for b, v in zip(bits, f[2:6]) if v.lower().startswith("active"))
        self.samples.append((float(f[0]), float(f[1]), rs))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample_nvml() if self._nvml else self._sample_smi()
            except Exception:
                pass
            self._stop.wait(0.02 if self._nvml else 0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [s[0] for s in self.samples]
        reasons = sorted({name for s in self.samples for bit, name in self.REASONS.items() if s[2] & bit})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": reasons, "samples": len(self.samples), "source": "nvml" if self._nvml else "nvidia-smi"}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="native", choices=["native", "baseline", "reference"])
    p.add_argument("--config", default="v3-1k", choices=sorted(BENCH_CONFIGS),
                   help="named workload: v3-1k (headline: 671B, 64 x 1K, TP attention + EP), v32-sparse-32k "
                        "(671B + lightning indexer top-2048, 8 x 32K), v3-dp-2k / v3-nvfp4-dp-2k (DP attention "
                        "+ EP, 256 x 2K; MXFP8 / NVFP4 routed experts), v41-flash-1k (V4.1-Flash-shaped, "
                        "64 x 1K)")
    p.add_argument("--model", default=None)
    p.add_argument("--batch", type=int, default=None)
    p.add_argument("--input-len", type=int, default=None)
    p.add_argument("--output-len", type=int, default=None)
    p.add_argument("--weight-sets", type=int, default=0)
    p.add_argument("--trace", action="store_true",
                   help="device timestamps per layer phase inside the decode graph (adds launches: the step "
                        "time of a traced run is not a clean measurement); adds a per-phase breakdown to the JSON")
    a = p.parse_args()
    d = BENCH_CONFIGS[a.config]
    a.model = a.model or d["model"]
    a.batch = a.batch or d["batch"]
    a.input_len = a.input_len or d["input_len"]
    a.output_len = a.output_len or d["output_len"]
    a.dp = bool(d.get("dp", False))
    return a


# Named workloads (model preset, concurrent requests, input tokens each).
BENCH_CONFIGS = {
    "v3-1k": {"model": "deepseek-v3-671b", "batch": 64, "input_len": 1024, "output_len": 1024},
    "v32-sparse-32k": {"model": "deepseek-v3.2-sparse-671b", "batch": 8, "input_len": 32768, "output_len": 1024},
    # DP attention on every rank + EP over all ranks, 256 requests x 2K in, 512 out
    "v3-dp-2k": {"model": "deepseek-v3-671b", "batch": 256, "input_len": 2048, "output_len": 512, "dp": True},
    "v3-nvfp4-dp-2k": {"model": "deepseek-v3-671b-nvfp4", "batch": 256, "input_len": 2048, "output_len": 512,
                       "dp": True},
    # the reference's served architecture: DeepSeek-V4.1-Flash shape (mHC, MQA + sinks, Engram, E5), NVFP4 experts
    "v41-flash-1k": {"model": "deepseek-v4.1-flash", "batch": 64, "input_len": 1024, "output_len": 1024},
}


def log(msg: str) -> None:
    if os.environ.get("RANK", "0") == "0":
        print(f"[bench] {time.strftime('%H:%M:%S')} {msg}", file=sys.stderr, flush=True)


def main():
    import faulthandler
    faulthandler.enable()
    args = parse()
    if args.impl == "reference":
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference is a forward-pass plug-in for an absent SGLang fork (no setup.py/"
                          "pyproject; needs cacheon/dsv41-tp2-upstream, FlashInfer 0.7.1, DeepGEMM, sm_103); "
                          "pip install of the reference source tree fails: 'Directory is not installable'"}))
        return
    if args.impl == "baseline":
        # FlashInfer's JIT modules of the library arm, prebuilt in-tree (compiling
        # them on a fresh box takes tens of minutes)
        os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", os.path.join(ROOT, "baseline", "_fi"))
    import torch
    import torch.distributed as dist
    from b200ds import ops
    from b200ds.config import PRESETS, EngineConfig
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.random_init import build_random_model
    from b200ds.parallel.state import init_parallel

    world = int(os.environ.get("WORLD_SIZE", "1"))
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE={world}"
    ps = init_parallel(backend="nccl", timeout_s=600, dp_attention=args.dp)
    dev = ps.device if ps.device.type == "cuda" else torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ops.set_impl("torch" if args.impl == "baseline" else "native")
    if args.impl == "native":
        import b200ds._C  # noqa: F401
    cfg = PRESETS[args.model]()
    # KV room for the whole output (1K in + 1K out reaches context 2K): decode is
    # timed at contexts spread over the output (see context_points)
    ctx = args.input_len + args.output_len + 2 * args.warmup + 2 * args.steps + 16
    # DP attention: each rank serves batch / world of the requests
    assert not args.dp or args.batch % world == 0, "DP attention needs batch % gpus == 0"
    local_batch = args.batch // world if args.dp else args.batch
    ecfg = EngineConfig(tp_size=1 if args.dp else world, ep_size=world, page_size=64, max_num_seqs=local_batch,
                        max_prefill_tokens=16384 if not args.dp else 4096, cuda_graphs=True,
                        graph_batch_sizes=(local_batch,), enable_prefix_cache=False, weight_sets=args.weight_sets,
                        max_model_len=max(16384, ctx + 64), dp_attention=args.dp, trace=args.trace)
    t0 = time.time()
    log(f"building {args.model} on {world} GPU(s)")
    kv_per_tok = cfg.num_hidden_layers * (cfg.kv_cache_dim + (cfg.index_head_dim + 4 if cfg.index_n_heads else 0))
    reserve = 24e9 + local_batch * (ctx + 64) * kv_per_tok
    if cfg.is_v4:
        from b200ds.models.random_init import build_random_model_v4
        model = build_random_model_v4(cfg, ecfg, ps, dev, seed=0, reserve_bytes=reserve)
    else:
        model = build_random_model(cfg, ecfg, ps, dev, seed=0, reserve_bytes=reserve)
    torch.cuda.synchronize()
    t_init = time.time() - t0
    pages_per_seq = (ctx + ecfg.page_size - 1) // ecfg.page_size
    eng = Engine(model, ecfg, num_pages=local_batch * pages_per_seq + 8)
    eng.graphs.max_pages = pages_per_seq

    g = torch.Generator().manual_seed(0)
    prompts = torch.randint(0, cfg.vocab_size, (args.batch, args.input_len), generator=g).tolist()
    if args.dp:
        prompts = prompts[ps.rank::world]
    # every request decodes through the warm-up and both timed loops without finishing
    sp = SamplingParams(max_tokens=ctx - args.input_len, ignore_eos=True)
    reqs = [eng.add_request(p, sp) for p in prompts]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- prefill (TTFT) -------------------------------------------------------
    log(f"model ready in {time.time() - t0:.1f}s, weight sets {getattr(model, 'weight_sets', None)}; prefill")
    barrier()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    def pending_prefill() -> bool:
        p = int(any(r.t_first is None for r in reqs))
        if args.dp and world > 1:       # DP ranks step in lockstep until all are done
            t = torch.tensor([p], dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ps.cpu_group)
            p = int(t.item())
        return bool(p)

    while pending_prefill():
        eng.step()
    s1.record()
    barrier()
    ttft_ms = max_over_ranks(s0.elapsed_time(s1))

    # ---- capture + warmup --------------------------------------------------------
    log(f"prefill done ({ttft_ms:.0f} ms); capturing decode graph")
    from b200ds.engine.cuda_graph import GraphCaptureFailed
    graphs_ok = True
    try:
        eng.graphs.capture_all()
    except GraphCaptureFailed as e:
        # the library arm's PyTorch ops may not be capturable: it then runs
        # (and is timed as) eager decode steps; our own arm must capture
        if args.impl == "native":
            raise
        graphs_ok = False
        eng._graphs_off("decode", e)
    log("warmup")
    for _ in range(args.warmup):
        eng.step()
    barrier()

    # ---- timed decode at contexts spread over the 1K output ----------------------
    # The K timed steps are split over three context points (start of the
    # output, its middle, its end), so the step time averages the attention
    # cost over the whole output.  Each point: K_i back-to-back replays of the
    # captured decode step (device-timed, max over ranks), then K_i steps
    # through Engine.step (end to end).  Between points every running request
    # is moved forward to the next context: its KV rows for the skipped
    # positions are copies of its own earlier rows (the work per step depends
    # on the context length only).
    points = context_points(args.input_len, args.output_len, args.steps, args.warmup)
    shares = [args.steps // len(points) + (1 if k < args.steps % len(points) else 0) for k in range(len(points))]
    gr = eng.graphs.graphs[eng.graphs._bucket(len(eng.sched.running))] if graphs_ok else None
    sampler = ClockSampler(dev.index)
    dev_ms, e2e_ms, step_times, per_point = 0.0, 0.0, [], []
    with sampler:
        for ctx_target, k in zip(points, shares):
            if k == 0:
                continue
            advance_context(eng, model, ctx_target, seed=ctx_target)
            seqs = [{"tokens": [r.all_tokens[r.cached]], "start": r.cached, "pages": r.pages}
                    for r in eng.sched.running]
            if gr is not None:
                eng.graphs.stage(gr, seqs)
            barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(k):
                if gr is not None:
                    gr.graph.replay()
                else:
                    eng.step()            # eager library arm: its step is the whole engine step
            e1.record()
            barrier()
            d_ms = max_over_ranks(e0.elapsed_time(e1))
            # end to end through the public API (host scheduling, pinned H2D of
            # the step's inputs, replay, D2H of the sampled ids)
            f0 = torch.cuda.Event(enable_timing=True)
            f1 = torch.cuda.Event(enable_timing=True)
            pt = []
            f0.record()
            for _ in range(k):
                t = time.perf_counter()
                eng.step()
                pt.append(time.perf_counter() - t)
            f1.record()
            barrier()
            f_ms = max_over_ranks(f0.elapsed_time(f1))
            dev_ms += d_ms
            e2e_ms += f_ms
            step_times += pt
            per_point.append({"context": ctx_target, "steps": k, "ms_per_step": round(d_ms / k, 3),
                              "e2e_ms_per_step": round(f_ms / k, 3),
                              "p50_tpot_ms": round(statistics.median(pt) * 1e3, 3)})
    step_ms = dev_ms / args.steps
    trace_us = None
    if args.trace and gr is not None and gr.trace_names:
        tr = model.tracer
        gr.graph.replay()
        st = tr.stamps()
        tr.names = gr.trace_names
        trace_us = {k: round(v, 1) for k, v in tr.summary(st).items()}
    value = args.batch * args.steps / (dev_ms / 1e3)
    log(f"device-timed {step_ms:.2f} ms/step over contexts {points}")
    e2e_value = args.batch * args.steps / (e2e_ms / 1e3)
    tpot_p50 = statistics.median(step_times) * 1e3

    # token id, position, KV slot, length, block-table row, sampling params (4 x 4 B)
    h2d = local_batch * (4 + 4 + 8 + 4 + 16) + local_batch * eng.graphs.max_pages * 4
    d2h = local_batch * 8
    launches, graph_nodes = count_launches(gr) if args.impl == "native" else (None, None)
    if os.environ.get("B200_BENCH_PROFILE") == "1" and gr is not None:
        profile_breakdown(gr, ps.rank)
    clocks = sampler.summary()
    if ps.rank == 0:
        out = {
            "metric": HEADLINE_METRIC,
            "value": round(value, 2),
            "unit": "output tokens/s (whole job)",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(step_ms, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "fp8 weights (MXFP8, UE8M0 per 32) / bf16 activations, fp32 accumulate",
            "data": "synthetic: uniform-random token ids (seed 0), random-init weights",
            "impl": args.impl,
            "tok_s_per_gpu": round(value / world, 2),
            "p50_tpot_ms": round(tpot_p50, 3),
            "ttft_ms_batch_prefill": round(ttft_ms, 2),
            "e2e": {"value": round(e2e_value, 2), "unit": "output tokens/s (whole job) via Engine.step",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            # every kernel node of the decode graph (ours + torch / library glue)
            "graph_kernel_nodes": graph_nodes,
            "clocks": clocks,
            "config": {"name": args.config, "model": args.model, "global_batch": args.batch,
                       "seq_len": args.input_len, "output_len": args.output_len,
                       "context_points": per_point,
                       "parallelism": (f"dp{world}-attn+ep{world}-moe" if args.dp else f"tp{world}-attn+ep{world}-moe"),
                       "expert_format": cfg.expert_format, "weight_sets": getattr(model, "weight_sets", None),
                       "weight_format": weight_format(cfg, args.impl),
                       "switches": __import__("b200ds.utils.levers", fromlist=["switches"]).switches(),
                       "selfcheck": eng.selfcheck,
                       "l2": "no flush: per-step weights+KV >> 126 MB L2", "init_s": round(t_init, 1),
                       "decode": "cuda graph replay" if gr is not None else "eager engine steps (graph capture failed)"},
        }
        if trace_us is not None:
            out["trace_us_per_step"] = trace_us      # traced run: timing includes the stamp launches
        print(json.dumps(out), flush=True)
    # Teardown: drop every reference to the captured graphs (they hold NCCL
    # work) before the process group goes.  The process then ends through the
    # normal interpreter exit (exit handlers run); a daemon watchdog ends it
    # only if the multi-rank teardown stalls, since the result line is out.
    gr = None
    eng.graphs.release()
    import gc
    gc.collect()
    torch.cuda.synchronize()
    sys.stdout.flush()
    sys.stderr.flush()
    if world > 1:
        wd = threading.Timer(60.0, lambda: os._exit(0))
        wd.daemon = True
        wd.start()
        try:
            dist.destroy_process_group()
        except Exception as e:
            log(f"process-group teardown: {e}")
        wd.cancel()


def weight_format(cfg, impl: str) -> str:
    """The weight / activation formats the timed step streams."""
    dense = ("dense and attention weights e4m3 with one UE8M0 scale per 32 K elements (MXFP8; a checkpoint's "
             "128x128 fp32 block scales are converted at load), activations quantized the same way per 32")
    if impl == "baseline":
        return ("routed experts: the same e4m3 bytes with 128x128 fp32 block scales, activations with 1x128 scales "
                "(FlashInfer trtllm-gen DeepSeek FP8); " + dense)
    if cfg.expert_format == "nvfp4":
        return ("routed experts NVFP4 (e2m1 + e4m3 per 16 + fp32 global scale per expert; activations per token); "
                + dense)
    return "routed experts and " + dense


def context_points(input_len: int, output_len: int, steps: int, warmup: int):
    """Contexts at which decode is timed: the output's start (right after
    prefill and warm-up), its middle and its end (input_len + output_len,
    minus the room the timed steps need)."""
    k = steps // 3 + 1
    first = input_len + warmup
    last = input_len + output_len - 2 * k - 1
    mid = (first + last) // 2
    return [first, mid, last] if last > mid > first else [first]


def advance_context(eng, model, target: int, seed: int = 0) -> None:
    """Move every running request forward to `target` cached tokens without
    running the model: output tokens are appended (uniform-random ids), pages
    allocated, and the KV rows (every per-slot cache tensor of the model) of
    the new positions copied from the request's own rows at position
    (p mod cached-so-far).  Decode work per step depends on the context
    length only, so this reaches a later context at no compute cost."""
    import torch
    g = torch.Generator().manual_seed(seed)
    ps = eng.ecfg.page_size
    src, dst = [], []
    for r in eng.sched.running:
        have = r.cached
        if target <= have:
            continue
        n_new = target - have
        r.output.extend(torch.randint(0, eng.cfg.vocab_size, (n_new,), generator=g).tolist())
        if not eng.sched._ensure_pages(r, target + 1):
            raise RuntimeError("KV pool too small for the timed contexts")
        for p in range(have, target):
            q = p % have
            dst.append(r.pages[p // ps] * ps + p % ps)
            src.append(r.pages[q // ps] * ps + q % ps)
        r.cached = target
    if not dst:
        return
    dev = model.device
    si = torch.tensor(src, dtype=torch.int64, device=dev)
    di = torch.tensor(dst, dtype=torch.int64, device=dev)
    for t in model.kv_tensors():
        if t.dim() >= 1 and t.shape[0] >= int(max(max(src), max(dst))) + 1:
            v = t.view(torch.uint8) if t.element_size() == 1 else t    # no fp8 index kernels
            v.index_copy_(0, di, v.index_select(0, si))
    if dev.type == "cuda":
        torch.cuda.synchronize()


def profile_breakdown(gr, rank: int) -> None:
    """Diagnostic only (stderr, never part of the result): per-kernel device
    time of one untimed decode-graph replay."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        gr.graph.replay()
        torch.cuda.synchronize()
    if rank != 0:
        return
    rows = sorted(prof.key_averages(), key=lambda e: -e.device_time_total)
    tot = sum(e.device_time_total for e in rows)
    print(f"[profile] kernel time {tot / 1e3:.2f} ms in one replay", file=sys.stderr)
    for e in rows[:28]:
        print(f"[profile] {e.device_time_total / 1e3:8.3f} ms {100 * e.device_time_total / max(tot, 1):5.1f}% "
              f"n={e.count:4d} {e.key[:100]}", file=sys.stderr)


def count_launches(gr):
    """(kernels of the b200ds extension, all kernel nodes) in one replay of
    the decode graph, read from the captured graph's kernel nodes (no
    profiler)."""
    from b200ds import _C
    total, ours = _C.graph_kernel_count(gr.graph.raw_cuda_graph())
    return int(ours), int(total)


if __name__ == "__main__":
    main()
