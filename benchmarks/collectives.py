#!/usr/bin/env python
"""Fused-collective microbenchmark sweep, one process per GPU:

    torchrun --nproc-per-node N benchmarks/collectives.py [--part ar,ep]

Every arm is timed as `iters` back-to-back calls captured in one CUDA graph
(the host launch path is out of every arm alike), replayed after warm-up,
CUDA events on the launching stream, max over ranks.  Per token count M
(rows per rank; default 1, 8, 64, 512, 4096, 16384):

o_proj GEMM + all-reduce (bf16 partial [M, 7168], K = 16384 / N):
  * nccl_ar        NCCL all-reduce of the partial alone;
  * nccl_ar_norm   NCCL all-reduce + residual add + RMSNorm in PyTorch ops
                   (the library chain the fused kernels replace);
  * push_ar        our one-shot NVLink push + reduce (+residual +RMSNorm
                   +MXFP8) as one kernel (per-CTA arrivals);
  * push2_ar       the same as a push kernel + a reduce kernel;
  * push1_c{1,4}_ar the one-kernel variant at any row count with 1 / 4 CTAs
                   per row owner sharing the NVLink stores;
  * nvls1_ar       one-kernel NVLS variant (rows stored locally, summed
                   through the switch by one rank per CTA, broadcast back);
  * nvls_ar        the same through NVLink multicast (multimem.ld_reduce /
                   multimem.st in the switch), when the GPUs support it;
  * gemm_nccl      our MXFP8 GEMM + NCCL all-reduce;
  * gemm_push      the GEMM whose split-K cluster epilogue stores its tiles
                   for the all-reduce (push protocol; M <= 128), + reduce;
  * gemm_nvls      the same epilogue into the NVLS input slot, + NVLS reduce;
  * lib_nccl       cuBLAS block-scaled GEMM (torch._scaled_mm) + NCCL.
  Roofline: max(GEMM FLOPs / fp8 peak (2 x measured bf16), weight bytes /
  measured HBM copy bandwidth, all-reduce bytes / 770 GB/s) with the
  all-reduce moving M x 7168 x 2 bytes per GPU each way (a partial leaves
  once, the sum arrives once).

EP dispatch / combine (fp8 rows of hidden 7168 + UE8M0 scales, 256 experts
top-8, uniform-random routing, seed 0):
  * ep_dispatch    our P2P push of each routed row to its expert owners +
                   the routing layout build (ep_dispatch + ep_align);
  * nccl_dispatch  the same rows through torch all_to_all_single (NCCL),
                   packed per destination beforehand;
  * ep_combine     our reduce-scatter of the expert partials into the owner
                   ranks + reduce (+residual +RMSNorm +MXFP8);
  * nccl_combine   NCCL all_to_all_single of the partial rows back + the
                   owner's index_add.
  Roofline: bytes this rank must send over NVLink (rows bound to other
  ranks) / 770 GB/s.
Prints one JSON object per (part, M) on rank 0.
"""
import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch
import torch.distributed as dist


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "measured"
    return 6.65e12, 1.59e15, "fallback"


HBM, BF16, PEAK_SRC = _peaks()
NVLINK = 770e9        # measured peer copy per direction, bytes/s

GRAPHS = []


def timed(fn, iters, warmup=3):
    """Device time per call (us) of `iters` graph-captured calls, max over ranks."""
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


def _out(ps, res):
    if ps.rank == 0:
        print(json.dumps({k: (round(v, 3) if isinstance(v, float) else v) for k, v in res.items()}), flush=True)


def ar_part(ps, Ms):
    from b200ds import _C
    from b200ds.ops import cuda as oc
    from b200ds.ops.quant import MXFP8Tensor
    from b200ds.parallel.symm import FusedAllReduce
    from b200ds.utils import levers
    W, H = ps.world_size, 7168
    K = 16384 // W
    dev = ps.device
    os.environ["B200_NVLS_MIN_WORLD"] = "2"
    levers.set_switch("nvls", False)
    far_push = FusedAllReduce(ps, H, max_tokens=max(Ms), push_ctas=296)
    levers.set_switch("nvls", True)
    far_nvls = FusedAllReduce(ps, H, max_tokens=max(Ms), push_ctas=296)
    if far_nvls.nvls is None:
        far_nvls = None
    wq = torch.empty(H, K, dtype=torch.uint8, device=dev)
    _C.fill_bytes(wq, 11 + ps.rank, 0xBF, 0)
    w = MXFP8Tensor(wq.view(torch.float8_e4m3fn), torch.full((H * K // 32,), 122, dtype=torch.uint8, device=dev))
    ln = torch.ones(H, device=dev)
    for M in Ms:
        iters = 20 if M <= 512 else 5
        x = oc.quant(torch.randn(M, K, device=dev, dtype=torch.bfloat16))
        part = torch.randn(M, H, device=dev, dtype=torch.bfloat16)
        resid = torch.zeros(M, H, device=dev)
        res = {"part": "gemm_ar", "M": M, "n_gpus": W, "N": H, "K": K}
        res["nccl_ar_us"] = timed(lambda: dist.all_reduce(part), iters)

        def nccl_norm():
            # the library chain the fused kernels replace: NCCL all-reduce,
            # residual add and RMSNorm in PyTorch ops
            r = part.clone()
            dist.all_reduce(r)
            resid.add_(r.float())
            return (resid * torch.rsqrt(resid.pow(2).mean(-1, keepdim=True) + 1e-6) * ln).to(torch.bfloat16)
        res["nccl_ar_norm_us"] = timed(nccl_norm, iters)
        res["push_ar_us"] = timed(lambda: far_push.allreduce_add_rmsnorm(part, resid, ln, 1e-6, True), iters)
        levers.set_switch("ar_one_kernel", False)
        res["push2_ar_us"] = timed(lambda: far_push.allreduce_add_rmsnorm(part, resid, ln, 1e-6, True), iters)
        levers.set_switch("ar_one_kernel", True)
        # one kernel whatever the row count, its stores spread over 1 / 4 CTAs per row owner
        os.environ["B200_AR_ONE_KERNEL_ROWS"] = str(1 << 30)
        for ch in (1, 4):
            os.environ["B200_AR_CHUNKS"] = str(ch)
            res[f"push1_c{ch}_ar_us"] = timed(lambda: far_push.allreduce_add_rmsnorm(part, resid, ln, 1e-6, True),
                                              iters)
        os.environ.pop("B200_AR_ONE_KERNEL_ROWS")
        os.environ["B200_AR_CHUNKS"] = "1"
        if far_nvls is not None:
            res["nvls_ar_us"] = timed(lambda: far_nvls.allreduce_add_rmsnorm(part, resid, ln, 1e-6, True), iters)
            levers.set_switch("nvls_one_kernel", True)
            res["nvls1_ar_us"] = timed(lambda: far_nvls.allreduce_add_rmsnorm(part, resid, ln, 1e-6, True), iters)
            levers.set_switch("nvls_one_kernel", False)
        res["gemm_nccl_us"] = timed(lambda: dist.all_reduce(oc.gemm(x, w)), iters)
        if M <= 128:
            res["gemm_push_us"] = timed(lambda: far_push.gemm_allreduce_add_rmsnorm(x, w, resid, ln, 1e-6, True),
                                        iters)
            if far_nvls is not None:
                res["gemm_nvls_us"] = timed(
                    lambda: far_nvls.gemm_allreduce_add_rmsnorm(x, w, resid, ln, 1e-6, True), iters)
        try:
            sa = x.sf.view(torch.float8_e8m0fnu)
            sb = w.sf.view(torch.float8_e8m0fnu)
            res["lib_nccl_us"] = timed(lambda: dist.all_reduce(
                torch._scaled_mm(x.q, w.data.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)), iters)
        except Exception as e:  # library path unavailable for this shape
            res["lib_nccl_us"] = None
            res["lib_error"] = str(e)[:120]
        flops = 2.0 * M * H * K
        ar_bytes = 1.0 * M * H * 2 if W > 1 else 0.0
        res["roofline_us"] = max(flops / (2 * BF16), (H * K + M * K) / HBM, ar_bytes / NVLINK) * 1e6
        res["ar_roofline_us"] = ar_bytes / NVLINK * 1e6
        fused = [res.get(k) for k in ("gemm_nvls_us", "gemm_push_us") if res.get(k)]
        best = min(fused) if fused else min(v for v in (res.get("gemm_nccl_us"),) if v)
        res["fused_gemm_ar_fraction_of_roofline"] = res["roofline_us"] / best
        ars = [res.get(k) for k in ("nvls_ar_us", "nvls1_ar_us", "push_ar_us") if res.get(k)]
        res["fused_ar_fraction_of_roofline"] = res["ar_roofline_us"] / min(ars) if ars else None
        res["peaks"] = PEAK_SRC
        for f in (far_push, far_nvls):
            if f is not None:
                f.check()
        _out(ps, res)


def ep_part(ps, Ms):
    from b200ds import _C
    from b200ds.ops import cuda as oc
    from b200ds.parallel.symm import EPDispatch, FusedAllReduce
    W, H, E, K = ps.world_size, 7168, 256, 8
    per = E // W
    dev = ps.device
    ep = EPDispatch(ps, H, K, max(Ms))
    far = FusedAllReduce(ps, H, max_tokens=max(Ms), push_ctas=296, group="ep")
    ln = torch.ones(H, device=dev)
    for M in Ms:
        iters = 10 if M <= 512 else 3
        g = torch.Generator().manual_seed(0)
        # uniform-random top-8 of 256 per token (seed 0), this rank's slice of the tokens
        ids_all = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(M * W)]).int()
        ids = ids_all[ps.rank * M:(ps.rank + 1) * M].contiguous().to(dev)
        wts = torch.rand(M, K, generator=g).to(dev)
        a = oc.quant(torch.randn(M, H, device=dev, dtype=torch.bfloat16))
        Tg = W * M
        seg_start = torch.empty(per, dtype=torch.int32, device=dev)
        seg_count = torch.empty(per, dtype=torch.int32, device=dev)
        tt1 = torch.empty(per + 1, dtype=torch.int32, device=dev)
        tt2 = torch.empty(per + 1, dtype=torch.int32, device=dev)
        max_rows = ((Tg * K + 127) // 128) * 128 + per * 128
        row_token = torch.empty(max_rows, dtype=torch.int32, device=dev)
        row_weight = torch.empty(max_rows, dtype=torch.float32, device=dev)
        pair_row = torch.empty(Tg, K, dtype=torch.int32, device=dev)
        total = torch.empty(1, dtype=torch.int32, device=dev)
        first = ps.rank * per

        def dispatch():
            _C.ep_dispatch(a.q, a.sf, None, H, ids, wts, M, per, ep.bases, ep.rank, ep.max_t, ep.epoch,
                           ep.push_ticket)
            _C.ep_align(ep.bases, ep.rank, ep.max_t, H, K, M, first, per, seg_start, seg_count, row_token,
                        row_weight, pair_row, total, 16, tt1, 16, tt2, ep.epoch, ep.err, release=True)
        res = {"part": "ep", "M": M, "n_gpus": W, "hidden": H, "experts": E, "topk": K}
        res["ep_dispatch_us"] = timed(dispatch, iters)
        # rows this rank must send to other ranks (a token goes once to each owner of its experts)
        owners = (ids.long() // per).cpu()
        remote_rows = sum(len(set(r.tolist()) - {ps.rank}) for r in owners)
        row_bytes = H + H // 32
        t = torch.tensor([remote_rows], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res["dispatch_roofline_us"] = float(t.item()) * row_bytes / NVLINK * 1e6
        # NCCL: rows packed per destination owner, all_to_all_single of bytes
        dest_rows = [[] for _ in range(W)]
        for tok, r in enumerate(owners):
            for d in sorted(set(r.tolist())):
                dest_rows[d].append(tok)
        send_idx = torch.tensor([t_ for d in range(W) for t_ in dest_rows[d]], dtype=torch.long, device=dev)
        send_counts = torch.tensor([len(dest_rows[d]) for d in range(W)], dtype=torch.long)
        sc_d = send_counts.to(dev)
        rc_d = torch.empty_like(sc_d)
        dist.all_to_all_single(rc_d, sc_d)
        recv_counts = rc_d.cpu()
        in_split = [int(c) * row_bytes for c in send_counts]
        out_split = [int(c) * row_bytes for c in recv_counts]
        sf_rows = torch.randint(0, 255, (M, H // 32), dtype=torch.uint8, device=dev)
        row_u8 = torch.cat([a.q.view(torch.uint8), sf_rows], 1)
        send = torch.empty(sum(in_split), dtype=torch.uint8, device=dev)
        recv = torch.empty(sum(out_split), dtype=torch.uint8, device=dev)

        def nccl_dispatch():
            send.view(-1, row_bytes).copy_(row_u8.index_select(0, send_idx))
            dist.all_to_all_single(recv, send, out_split, in_split)
        res["nccl_dispatch_us"] = timed(nccl_dispatch, iters)
        # combine: partial rows over this rank's experts for every received token -> owner
        dispatch()                       # a fresh layout (pair_row) for the combine arm
        torch.cuda.synchronize()
        rows = int(total.item())
        y = torch.randn(rows + 128, H, device=dev, dtype=torch.bfloat16) * 0.01
        resid = torch.zeros(M, H, device=dev)

        def combine():
            _C.ep_combine_rs(y, pair_row, M, M, None, far.bases, far.rank, far.max_tokens, far.epoch,
                             far.push_ticket, far.push_ctas)
            qa = oc.alloc_qact(M, H, dev)
            _C.ar_reduce_norm(M, H, far.bases, far.rank, far.max_tokens, far.epoch, far.ticket, 1, resid, ln, 1e-6,
                              None, qa.q, qa.sf, far.err)
        res["ep_combine_us"] = timed(combine, iters)
        n_recv = int(recv_counts.sum())
        yb = torch.randn(n_recv, H, device=dev, dtype=torch.bfloat16) * 0.01
        back = torch.empty(int(send_counts.sum()), H, device=dev, dtype=torch.bfloat16)
        out = torch.zeros(M, H, device=dev, dtype=torch.float32)

        def nccl_combine():
            dist.all_to_all_single(back, yb, [int(c) for c in send_counts], [int(c) for c in recv_counts])
            out.zero_()
            out.index_add_(0, send_idx, back.float())
        res["nccl_combine_us"] = timed(nccl_combine, iters)
        res["combine_roofline_us"] = float(t.item()) * H * 2 / NVLINK * 1e6
        res["ep_dispatch_fraction_of_roofline"] = res["dispatch_roofline_us"] / res["ep_dispatch_us"]
        res["ep_combine_fraction_of_roofline"] = res["combine_roofline_us"] / res["ep_combine_us"]
        ep.check()
        far.check()
        _out(ps, res)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--part", default="ar,ep")
    ap.add_argument("--ms", default=os.environ.get("MS", "1,8,64,512,4096,16384"))
    a = ap.parse_args()
    from b200ds import ops
    from b200ds.parallel.state import init_parallel
    ops.set_impl("native")
    ps = init_parallel(backend="nccl", timeout_s=120)
    Ms = [int(x) for x in a.ms.split(",")]
    parts = a.part.split(",")
    if "ar" in parts:
        ar_part(ps, Ms)
    if "ep" in parts:
        ep_part(ps, Ms)
    torch.cuda.synchronize()
    GRAPHS.clear()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
