"""Prefill cost of the DeepSeek-V3-shaped decoder on one GPU, per layer kind.

Builds a model of the flagship's widths with few layers (one dense layer and
`--moe-layers` MoE layers, random-init MXFP8 weights), runs a batch prefill
of `--batch` prompts x `--input-len` tokens through the engine (the same
chunked path `bench.py` times as TTFT), once cold and then `--iters` times
warm, and prints JSON lines: the cold and warm wall times on the device (CUDA
events) and the warm time per layer, and, with
`--kernels`, the warm chunk's device time per kernel name from the PyTorch
profiler (shares only: numbers under a profiler are not timings).

    python benchmarks/prefill.py --batch 16 --input-len 1024 --moe-layers 3 --kernels

Under DP attention (`--dp-attention`, launched with torchrun, one rank per
GPU) each rank prefills its own `--batch` prompts; `--tbo` turns on the
two-batch overlap of those steps; `--context-parallel` instead prefills each
rank's prompts on all ranks together, one at a time (every rank adds every
prompt, owners round-robin).  The printed times are rank 0's device times,
maxed over the ranks.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 benchmarks/prefill.py --dp-attention \
        --context-parallel --batch 1 --input-len 32768
"""
import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--input-len", type=int, default=1024)
    ap.add_argument("--moe-layers", type=int, default=3)
    ap.add_argument("--chunk", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--kernels", action="store_true")
    ap.add_argument("--dp-attention", action="store_true")
    ap.add_argument("--context-parallel", action="store_true")
    ap.add_argument("--tbo", action="store_true")
    a = ap.parse_args()

    from b200ds import ops
    from b200ds.config import EngineConfig, v3_671b_config
    from b200ds.engine.engine import Engine
    from b200ds.engine.request import SamplingParams
    from b200ds.models.random_init import build_random_model
    from b200ds.parallel.state import init_parallel
    import b200ds._C  # noqa: F401

    ops.set_impl("native")
    import torch.distributed as dist
    dp = a.dp_attention or a.context_parallel or a.tbo
    ps = init_parallel(backend="nccl", timeout_s=300, dp_attention=dp)
    dev = ps.device if ps.device.type == "cuda" else torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    W = ps.world_size
    cfg = v3_671b_config(num_hidden_layers=1 + a.moe_layers, first_k_dense_replace=1)
    ctx = a.input_len + 8
    pages = (ctx + 63) // 64
    n_req = a.batch * (2 + a.iters)
    ecfg = EngineConfig(page_size=64, max_num_seqs=a.batch, max_prefill_tokens=a.chunk, cuda_graphs=False,
                        enable_prefix_cache=False, max_model_len=ctx + 64,
                        tp_size=1 if dp else ps.tp_size, ep_size=ps.ep_size, dp_attention=dp,
                        context_parallel=a.context_parallel, tbo=a.tbo)
    model = build_random_model(cfg, ecfg, ps, dev, seed=0, reserve_bytes=8e9 + n_req * ctx * 700 * cfg.num_hidden_layers)
    eng = Engine(model, ecfg, num_pages=a.batch * pages * (W if a.context_parallel else 1) + 8)
    g = torch.Generator().manual_seed(0)

    def dev_max(ms: float) -> float:
        if W == 1:
            return ms
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=ps.cpu_group)
        return float(t.item())

    def one_batch():
        prompts = torch.randint(0, cfg.vocab_size, (W, a.batch, a.input_len), generator=g).tolist()
        sp = SamplingParams(max_tokens=1, ignore_eos=True)
        if a.context_parallel:      # every rank adds every prompt; owners round-robin
            reqs = [eng.add_request(p, sp, cp_owner=q) for q in range(W) for p in prompts[q]]
        else:
            reqs = [eng.add_request(p, sp) for p in prompts[ps.rank if dp else 0]]
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        while any(r.t_first is None and not r.finished for r in reqs):
            eng.step()
        e1.record()
        torch.cuda.synchronize()
        while any(not r.finished for r in reqs):
            eng.step()
        if dp:
            eng._drain_dp()
        return dev_max(e0.elapsed_time(e1))

    cold = one_batch()
    warm = [one_batch() for _ in range(a.iters)]
    w = min(warm)
    tokens = a.batch * a.input_len * (W if dp else 1)
    if ps.rank == 0:
        print(json.dumps({"bench": "prefill", "gpus": W, "dp_attention": dp, "context_parallel": a.context_parallel,
                          "tbo": a.tbo, "batch": a.batch, "input_len": a.input_len, "layers": cfg.num_hidden_layers,
                          "moe_layers": a.moe_layers, "chunk": a.chunk, "cold_ms": round(cold, 2),
                          "warm_ms": round(w, 2), "warm_all_ms": [round(x, 2) for x in warm],
                          "tokens": tokens, "warm_tok_s": round(tokens / w * 1e3, 1),
                          "warm_ms_per_layer": round(w / cfg.num_hidden_layers, 2)}), flush=True)
    if a.kernels:
        from torch.profiler import ProfilerActivity, profile
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            one_batch()             # every rank: the steps are collective
        if ps.rank != 0:
            return
        rows = []
        for ev in prof.key_averages():
            dt = getattr(ev, "device_time_total", None)
            if dt is None:
                dt = getattr(ev, "cuda_time_total", 0)
            if dt and ev.count:
                rows.append((dt, ev.count, ev.key))
        rows.sort(reverse=True)
        total = sum(r[0] for r in rows) or 1.0
        for dt, cnt, key in rows[:40]:
            print(json.dumps({"kernel": key[:120], "device_us": round(dt, 1), "calls": cnt,
                              "share": round(dt / total, 4)}), flush=True)


if __name__ == "__main__":
    main()
