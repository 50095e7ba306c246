#!/usr/bin/env python
"""Fused-collective microbenchmark sweep, one process per GPU:

    torchrun --nproc-per-node N benchmarks/collectives.py

For each token count M it times, with CUDA events around `iters` back-to-back
calls (max over ranks), on every rank:
  * nccl_ar      NCCL all-reduce of a bf16 [M, 7168] partial;
  * fused_ar     our one-shot NVLink push + reduce(+residual+RMSNorm+MXFP8);
  * gemm_nccl    our MXFP8 GEMM (o_proj shape N=7168, K=16384/N_gpus) + NCCL;
  * gemm_fused   the GEMM whose split-K cluster epilogue pushes its tiles into
                 every rank's slot, + the reduce kernel (M <= 128);
  * lib_nccl     cuBLAS block-scaled GEMM (torch._scaled_mm) + NCCL (baseline).
Roofline per point: max(FLOPs / measured bf16 peak x2 for fp8... reported as
the bf16 figure, weight bytes / measured HBM copy bandwidth, all-reduce bytes
2(W-1)/W x M x 7168 x 2 / 770 GB/s).  Prints one JSON object per M (rank 0).
"""
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch
import torch.distributed as dist

HBM = 6553e9          # measured copy bandwidth (MEASURED_PEAKS.json), bytes/s
BF16 = 1654.4e12      # measured cuBLAS bf16 burst, FLOP/s
NVLINK = 770e9        # measured peer copy per direction, bytes/s


GRAPHS = []


def timed(fn, iters, warmup=3):
    """Device time per call: `iters` calls captured in one CUDA graph (so the
    host launch path is out of the measurement for every arm alike), replayed
    after warm-up; CUDA events on the launching stream, max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(iters):
                fn()
    torch.cuda.current_stream().wait_stream(s)
    GRAPHS.append(g)
    g.replay()
    torch.cuda.synchronize()
    dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / iters * 1e3], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    from b200ds import _C, ops
    from b200ds.ops import cuda as oc
    from b200ds.ops.quant import MXFP8Tensor
    from b200ds.parallel.state import init_parallel
    from b200ds.parallel.symm import FusedAllReduce
    ps = init_parallel(backend="nccl", timeout_s=120)
    W, H = ps.world_size, 7168
    K = 16384 // W
    dev = ps.device
    Ms = [int(x) for x in os.environ.get("MS", "1,8,64,512,4096,16384").split(",")]
    far = FusedAllReduce(ps, H, max_tokens=max(Ms), push_ctas=296)
    wq = torch.empty(H, K, dtype=torch.uint8, device=dev)
    _C.fill_bytes(wq, 11 + ps.rank, 0xBF, 0)
    w = MXFP8Tensor(wq.view(torch.float8_e4m3fn), torch.full((H * K // 32,), 122, dtype=torch.uint8, device=dev))
    ln = torch.ones(H, device=dev)
    for M in Ms:
        iters = 20 if M <= 512 else 5
        x = oc.quant(torch.randn(M, K, device=dev, dtype=torch.bfloat16))
        part = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
        resid = torch.zeros(M, H, device=dev)
        res = {"M": M, "n_gpus": W, "N": H, "K": K}
        res["nccl_ar_us"] = timed(lambda: dist.all_reduce(part), iters)
        res["fused_ar_us"] = timed(lambda: far.allreduce_add_rmsnorm(part, resid, ln, 1e-6, True), iters)
        res["gemm_nccl_us"] = timed(lambda: dist.all_reduce(oc.gemm(x, w)), iters)
        if M <= 128:
            res["gemm_fused_us"] = timed(lambda: far.gemm_allreduce_add_rmsnorm(x, w, resid, ln, 1e-6, True), iters)
        try:
            sa = x.sf.view(torch.float8_e8m0fnu)
            sb = w.sf.view(torch.float8_e8m0fnu)
            res["lib_nccl_us"] = timed(lambda: dist.all_reduce(
                torch._scaled_mm(x.q, w.data.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)), iters)
        except Exception as e:  # library path unavailable for this shape
            res["lib_nccl_us"] = None
            res["lib_error"] = str(e)[:120]
        flops = 2.0 * M * H * K
        ar_bytes = 2.0 * (W - 1) / W * M * H * 2
        roof = max(flops / BF16, (H * K + M * K) / HBM, ar_bytes / NVLINK) * 1e6
        res["roofline_us"] = roof
        best = res.get("gemm_fused_us") or res["gemm_nccl_us"]
        res["fused_fraction_of_roofline"] = roof / best if best else None
        far.check()
        if ps.rank == 0:
            print(json.dumps({k: (round(v, 2) if isinstance(v, float) else v) for k, v in res.items()}), flush=True)
    torch.cuda.synchronize()
    GRAPHS.clear()
    os._exit(0)


if __name__ == "__main__":
    main()
