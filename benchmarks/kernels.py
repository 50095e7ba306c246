#!/usr/bin/env python
"""Per-kernel roofline harness for the hot sm_100a kernels at the 671B decode
shapes (one GPU).

Every case builds its inputs once, runs 3 warm-up launches, then times each
of `--iters` launches with CUDA events on the launching stream, writing a
256 MiB buffer before every launch so L2 (126 MB) starts cold.  Each case
prints one JSON line: device time per launch, the algorithmic bytes / FLOPs
it must move / do, and the achieved fraction of the measured peaks in
MEASURED_PEAKS.json (copy bandwidth `hbm_gbs`, cuBLAS bf16 `bf16_tflops`; FP8
and FP4 tensor work is reported against 2x / 4x that figure).

    python benchmarks/kernels.py                 # all cases
    python benchmarks/kernels.py --only moe_fc1  # cases whose name contains the string
    python benchmarks/kernels.py --small         # reduced sizes (for ncu captures)
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"] * 1e9, d["bf16_tflops"] * 1e12, "measured"
    return 6.65e12, 1.59e15, "fallback"


HBM, BF16, PEAK_SRC = peaks()
FLUSH = None


def timed(fn, iters: int) -> float:
    """Median device time (s) of fn() over `iters` cold-L2 launches.  fn is
    captured once in a CUDA graph and the graph is replayed between the
    events, so the host work inside fn (allocations, argument marshalling)
    does not show up as device idle time; an fn that cannot be captured is
    timed by direct calls."""
    global FLUSH
    if FLUSH is None:
        FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    run = fn
    try:
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        GRAPHS.append(g)
        run = g.replay
    except Exception:
        torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        FLUSH.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b) / 1e3)
    ts.sort()
    return ts[len(ts) // 2]


GRAPHS = []


def report(name, shape, t, nbytes=0, flops=0, flop_peak=None, note=""):
    out = {"kernel": name, "shape": shape, "us": round(t * 1e6, 2)}
    if nbytes:
        out["bytes"] = int(nbytes)
        out["GBps"] = round(nbytes / t / 1e9, 1)
        out["frac_hbm_" + PEAK_SRC] = round(nbytes / t / HBM, 3)
    if flops:
        pk = flop_peak or BF16
        out["TFLOPs"] = round(flops / t / 1e12, 1)
        out["frac_tc_" + PEAK_SRC] = round(flops / t / pk, 3)
    if note:
        out["note"] = note
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
def _mx(shape_lead, N, K, dev):
    from b200ds.models.random_init import rand_mx, _Seeder
    return rand_mx(shape_lead, N, K, dev, _Seeder(1))


def _moe_layout(T, K, E_total, E_local, dev, bn1, bn2):
    from b200ds import _C
    from b200ds.ops.cuda import round_up
    g = torch.Generator(device=dev).manual_seed(0)
    ids = torch.stack([torch.randperm(E_total, device=dev, generator=g)[:K] for _ in range(T)]).int()
    w = torch.rand(T, K, device=dev)
    E = E_local
    max_rows = round_up(T * K, 128) + E * 128
    seg_start = torch.empty(E, dtype=torch.int32, device=dev)
    seg_count = torch.empty(E, dtype=torch.int32, device=dev)
    tt1 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    tt2 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    row_token = torch.empty(max_rows, dtype=torch.int32, device=dev)
    row_weight = torch.empty(max_rows, dtype=torch.float32, device=dev)
    pair_row = torch.empty(T, K, dtype=torch.int32, device=dev)
    total = torch.empty(1, dtype=torch.int32, device=dev)
    _C.moe_align(ids, w, 0, E, seg_start, seg_count, row_token, row_weight, pair_row, total, bn1, tt1, bn2, tt2)
    torch.cuda.synchronize()
    active = int((seg_count > 0).sum())
    return dict(ids=ids, w=w, max_rows=max_rows, seg_start=seg_start, seg_count=seg_count, tt1=tt1, tt2=tt2,
                row_weight=row_weight, pair_row=pair_row, row_token=row_token, active=active)


def run_moe(fmt: str, T: int, E_total: int, E_local: int, iters: int, h=7168, I=2048, tiled=False, fused=False,
            pull=False):
    from b200ds import _C
    from b200ds.ops import cuda
    from b200ds.models.random_init import _Seeder, rand_mx, rand_nvfp4
    dev = torch.device("cuda")
    K = 8
    exp_rows = T * K / E_total
    bn1, bn2 = cuda.moe_tiles(exp_rows)
    L = _moe_layout(T, K, E_total, E_local, dev, bn1, bn2)
    mr = L["max_rows"]
    sd = _Seeder(3)
    fp4 = fmt == "nvfp4"
    if fp4:
        w13, w2 = rand_nvfp4(E_local, 2 * I, h, dev, sd), rand_nvfp4(E_local, h, I, dev, sd)
        xs_q = torch.randint(0, 255, (mr, h // 2), dtype=torch.uint8, device=dev)
        xs_sf = torch.full((mr * h // 16,), 0x38, dtype=torch.uint8, device=dev)
        xs_g = torch.full((mr,), 1e-3, device=dev)
        hq = torch.empty(mr, I // 2, dtype=torch.uint8, device=dev)
        hsf = torch.empty(mr * I // 16, dtype=torch.uint8, device=dev)
        wbytes = (3 * I * h) * (0.5 + 1 / 16)
        fc1 = lambda: _C.gemm_grouped(w13.data, w13.sf, xs_q, xs_sf, 2 * I, h, E_local, I, bn1, L["seg_start"],
                                      L["seg_count"], L["tt1"], 2, None, 0, hq, hsf, I, None, 0, False,
                                      w_g=w13.global_scale, x_g=xs_g, out_g=1 / 32, a_tiled=tiled)
        y = torch.empty(mr, h, dtype=torch.bfloat16, device=dev)
        fc2 = lambda: _C.gemm_grouped(w2.data, w2.sf, hq, hsf, h, I, E_local, 0, bn2, L["seg_start"], L["seg_count"],
                                      L["tt2"], 3, y, h, None, None, 0, L["row_weight"], 0, False,
                                      w_g=w2.global_scale, x_g_const=1 / 32, a_tiled=tiled)
        peak = 4 * BF16
    else:
        w13, w2 = rand_mx((E_local,), 2 * I, h, dev, sd), rand_mx((E_local,), h, I, dev, sd)
        xs = cuda.alloc_qact(mr, h, dev)
        xs.q.view(torch.uint8).fill_(0x38)
        xs.sf.fill_(127)
        hqa = cuda.alloc_qact(mr, I, dev)
        wbytes = (3 * I * h) * (1 + 1 / 32)
        fc1 = lambda: _C.gemm_grouped(w13.data, w13.sf, xs.q, xs.sf, 2 * I, h, E_local, I, bn1, L["seg_start"],
                                      L["seg_count"], L["tt1"], 2, None, 0, hqa.q, hqa.sf, I, None, 0, False,
                                      a_tiled=tiled)
        y = torch.empty(mr, h, dtype=torch.bfloat16, device=dev)
        fc2 = lambda: _C.gemm_grouped(w2.data, w2.sf, hqa.q, hqa.sf, h, I, E_local, 0, bn2, L["seg_start"],
                                      L["seg_count"], L["tt2"], 3, y, h, None, None, 0, L["row_weight"], 0, False,
                                      a_tiled=tiled)
        peak = 2 * BF16
    pairs = int((L["pair_row"] >= 0).sum())
    if fused:
        from b200ds.ops import ExpertWeights
        ex = ExpertWeights(0, E_local, w13, w2, I, tiled=tiled, fc2_act_scale=1 / 32)
        src = None
        if pull:
            # FC1 rows read in place from the T token rows (no sorted copy)
            if fp4:
                src = dict(row_token=L["row_token"], src_q=[xs_q.data_ptr()], src_sf=[xs_sf.data_ptr()],
                           src_g=[xs_g.data_ptr()], src_rows=T)
            else:
                src = dict(row_token=L["row_token"], src_q=[xs.q.data_ptr()], src_sf=[xs.sf.data_ptr()], src_rows=T)
        if fp4:
            fn = lambda: cuda._expert_gemms(ex, xs_q, xs_sf, xs_g, hq, hsf, y, h, bn1, bn1, L["seg_start"],
                                            L["seg_count"], L["tt1"], L["tt2"], L["row_weight"], True, src)
        else:
            fn = lambda: cuda._expert_gemms(ex, xs.q, xs.sf, None, hqa.q, hqa.sf, y, h, bn1, bn1, L["seg_start"],
                                            L["seg_count"], L["tt1"], L["tt2"], L["row_weight"], False, src)
        t = timed(fn, iters)
        shape = f"{fmt} T={T} top8 E={E_local}/{E_total} active={L['active']} pairs={pairs}" + (" tiled" if tiled else "")
        report(f"moe_fc1fc2_fused_{fmt}" + ("_pull" if pull else ""), shape, t, nbytes=L["active"] * wbytes,
               flops=2 * pairs * 3 * I * h, flop_peak=peak,
               note=f"bn={bn1}, one launch" + (", rows read in place" if pull else ", pre-gathered rows"))
        return
    shape = f"{fmt} T={T} top8 E={E_local}/{E_total} active={L['active']} pairs={pairs}" + (" tiled" if tiled else "")
    t1 = timed(fc1, iters)
    report(f"moe_fc1_{fmt}", shape, t1, nbytes=L["active"] * wbytes * 2 / 3, flops=2 * pairs * 2 * I * h,
           flop_peak=peak, note=f"bn={bn1}")
    t2 = timed(fc2, iters)
    report(f"moe_fc2_{fmt}", shape, t2, nbytes=L["active"] * wbytes / 3, flops=2 * pairs * I * h, flop_peak=peak,
           note=f"bn={bn2}")


def run_mla(B: int, ctx: int, H: int, iters: int, topk: int = 0):
    from types import SimpleNamespace
    from b200ds.ops import cuda
    dev = torch.device("cuda")
    ps = 64
    pages = (ctx + ps - 1) // ps
    bt = (torch.arange(B * pages, dtype=torch.int32, device=dev).view(B, pages) + 1)
    rows = (B * pages + 1) * ps
    cache = torch.empty(rows, 576, dtype=torch.uint8, device=dev)
    from b200ds import _C
    _C.fill_bytes(cache, 7, 0xBF, 0)
    cache = cache.view(torch.float8_e4m3fn)
    q_abs = (torch.randn(B, H, 512, device=dev) * 0.3).to(torch.bfloat16)
    q_pe = (torch.randn(B, H, 64, device=dev) * 0.3).to(torch.bfloat16)
    fb = SimpleNamespace(block_table=bt, q_seq=torch.arange(B, dtype=torch.int32, device=dev),
                         positions=torch.full((B,), ctx - 1, dtype=torch.int32, device=dev), is_decode=True,
                         max_seq_len=ctx)
    tk = None
    keys = ctx
    if topk:
        tk = torch.stack([torch.randperm(ctx, device=dev)[:topk].sort().values for _ in range(B)]).int()
        keys = topk
    fn = lambda: cuda.mla_attention(q_abs, q_pe, cache, 1.0, fb, 0.06, ps, tk)
    t = timed(fn, iters)
    nbytes = B * keys * 576 + B * H * (512 + 64) * 2 + B * H * 512 * 2
    flops = 2 * B * H * keys * (576 + 512)
    report("mla_sparse" if topk else "mla_decode", f"B={B} ctx={ctx} H={H}" + (f" top{topk}" if topk else ""), t,
           nbytes=nbytes, flops=flops, flop_peak=2 * BF16,
           note=f"splits={cuda.mla_splits(B, H, keys)} hb={cuda.mla_hb(H)} incl. q quant + merge")
    return t


def mla_sweep(B: int, ctx: int, H: int, iters: int):
    """MLA decode time over KV splits x heads per CTA (diagnostic)."""
    from b200ds.ops import cuda
    for hb in (16, 32, 64):
        if H % hb:
            continue
        for ns in (1, 2, 3, 4, 6, 8):
            cuda.MLA_HB, cuda.MLA_SPLITS = hb, ns
            run_mla(B, ctx, H, iters)
    cuda.MLA_HB, cuda.MLA_SPLITS = 0, 0


def run_indexer(B: int, ctx: int, iters: int):
    from types import SimpleNamespace
    from b200ds import _C
    from b200ds.config import v32_sparse_config
    from b200ds.models.rope import cos_sin_table
    from b200ds.ops import cuda
    dev = torch.device("cuda")
    ps = 64
    pages = (ctx + ps - 1) // ps
    bt = (torch.arange(B * pages, dtype=torch.int32, device=dev).view(B, pages) + 1)
    rows = (B * pages + 1) * ps
    kc = torch.empty(rows, 128, dtype=torch.uint8, device=dev)
    _C.fill_bytes(kc, 9, 0xBF, 0)
    ks = torch.rand(rows, device=dev) + 0.5
    table = cos_sin_table(v32_sparse_config(), ctx + 1, device=dev)
    fb = SimpleNamespace(block_table=bt, q_seq=torch.arange(B, dtype=torch.int32, device=dev),
                         positions=torch.full((B,), ctx - 1, dtype=torch.int32, device=dev), is_decode=True,
                         max_seq_len=ctx)
    q = (torch.randn(B, 64 * 128, device=dev) * 0.3).to(torch.bfloat16)
    w = torch.randn(B, 64, device=dev).to(torch.bfloat16)
    fn = lambda: cuda.indexer_topk(q, w, 0.01, table, kc.view(torch.float8_e4m3fn), ks, fb, ps, 2048)
    t = timed(fn, iters)
    report("indexer_topk", f"B={B} ctx={ctx} 64 heads x 128, top2048", t, nbytes=B * ctx * (128 + 4 + 4 * 2),
           flops=2 * B * ctx * 64 * 128, flop_peak=2 * BF16, note="q quant + tcgen05 scores + radix top-k")
    # the two halves: tcgen05 scores alone, the top-k alone (one CTA per row / a cluster per row)
    q8 = torch.empty(B * 64, 128, dtype=torch.uint8, device=dev)
    wq = torch.empty(B, 64, dtype=torch.float32, device=dev)
    _C.ix_q_quant(q, w, 64, 0.01, fb.positions, table, q8, wq)
    scores = torch.empty(B, pages * ps, dtype=torch.float32, device=dev)
    t_s = timed(lambda: _C.ix_score(q8, wq, kc, ks, bt, fb.q_seq, fb.positions, ps, cuda.ix_splits(B, ctx), scores),
                iters)
    report("ix_score", f"B={B} ctx={ctx} 64 heads x 128", t_s, nbytes=B * ctx * (128 + 4 + 4),
           flops=2 * B * ctx * 64 * 128, flop_peak=2 * BF16)
    out = torch.empty(B, 2048, dtype=torch.int32, device=dev)
    for label, mx in (("one CTA per row", 0), ("cluster per row", ctx)):
        t_k = timed(lambda: _C.topk_select(scores, fb.positions, out, mx), iters)
        report("topk_select", f"B={B} n={ctx} top2048 {label}", t_k, nbytes=B * ctx * 4 + B * 2048 * 4)


def run_gemm(name: str, T: int, N: int, K: int, iters: int):
    from b200ds.ops import QAct, cuda
    dev = torch.device("cuda")
    w = _mx((), N, K, dev)
    x = cuda.quant(torch.randn(T, K, device=dev).to(torch.bfloat16))
    fn = lambda: cuda.gemm(QAct(x.q, x.sf), w)
    t = timed(fn, iters)
    report(f"gemm_{name}", f"T={T} N={N} K={K}", t, nbytes=N * K * (1 + 1 / 32) + T * K + T * N * 2,
           flops=2 * T * N * K, flop_peak=2 * BF16, note=f"splits={cuda.choose_splits(T, N, K)}")


def run_norm(T: int, iters: int, h=7168):
    from b200ds.ops import cuda
    dev = torch.device("cuda")
    x = torch.randn(T, h, device=dev)
    res = torch.randn(T, h, device=dev)
    w = torch.rand(h, device=dev)

    class _L:
        quantized = True
    fn = lambda: cuda.add_rmsnorm_act(x.to(torch.bfloat16), res, w, 1e-6, _L())
    t = timed(fn, iters)
    report("add_rmsnorm_quant", f"T={T} h={h}", t, nbytes=T * h * (2 + 4 + 4 + 1 + 2))


def run_v4(T: int, iters: int, D: int = 5120, H: int = 64, ctx: int = 1040):
    """DeepSeek-V4.1-Flash-shaped decode-step kernels: mHC post, stats GEMM +
    coefficient / combine / norm / quant, MQA with sinks (64 heads over the
    latent rows), Engram gather from mapped host memory, E5 prune."""
    from types import SimpleNamespace
    from b200ds import _C, ops
    from b200ds.config import v41_flash_config
    from b200ds.models.deepseek_v4 import host_mapped_copy
    from b200ds.models.rope import cos_sin_table
    from b200ds.ops import HcWeights, cuda
    cfg = v41_flash_config()
    dev = torch.device("cuda")
    X = torch.randn(T, 4, D, device=dev).to(torch.bfloat16)
    y = torch.randn(T, D, device=dev).to(torch.bfloat16)
    post = torch.rand(T, 4, device=dev)
    comb = torch.rand(T, 16, device=dev) * 0.5
    t = timed(lambda: cuda.hc_post(X, y, post, comb), iters)
    report("v4_hc_post", f"T={T} hc=4 D={D}", t, nbytes=T * D * 2 * (4 + 4 + 1))
    hw = HcWeights(torch.randn(24, 4 * D, device=dev) * 0.02, torch.ones(3, device=dev), torch.zeros(24, device=dev))
    hw.fn_parts = cuda.hc_fn_parts(hw.fn)
    ss = X.float().pow(2).sum((1, 2))
    w = torch.ones(D, device=dev)

    class _Q:
        quantized = True
    t = timed(lambda: cuda.hc_pre(X, ss, hw, w, 1e-6, cfg, _Q(), False, False), iters)
    report("v4_hc_pre", f"T={T} hc=4 D={D} (stats GEMM + coeff/Sinkhorn/combine/norm/MXFP8)", t,
           nbytes=T * 4 * D * 2 * 2 + 128 * 4 * D * 2 + T * D, note="3 launches incl. the zeroed raw buffer")
    # the same boundary as one kernel (post + fp32 mixes + coefficients + normed input)
    t = timed(lambda: cuda.hc_boundary(X, (y, post, comb), hw, w, 1e-6, cfg, _Q(), False, False), iters)
    report("v4_hc_boundary", f"T={T} hc=4 D={D} (hc_post + mixes + coeff/Sinkhorn/combine/norm/MXFP8, one kernel)",
           t, nbytes=T * 4 * D * 2 * 2 + T * D * 2 + 24 * 4 * D * 4 + T * D,
           note="fn read from L2 by every row's cluster; compare with v4_hc_post + v4_hc_pre")
    ps = 64
    pages = (ctx + ps - 1) // ps
    table = cos_sin_table(cfg, 4096, device=dev)
    bt = (torch.arange(T * pages, dtype=torch.int32, device=dev).view(T, pages) + 1)
    cache = torch.empty((T * pages + 1) * ps, 576, dtype=torch.uint8, device=dev)
    _C.fill_bytes(cache, 7, 0xBF, 0)
    cache = cache.view(torch.float8_e4m3fn)
    q = (torch.randn(T, H, 512, device=dev) * 0.3).to(torch.bfloat16)
    fb = SimpleNamespace(block_table=bt, q_seq=torch.arange(T, dtype=torch.int32, device=dev),
                         positions=torch.full((T,), ctx - 1, dtype=torch.int32, device=dev), is_decode=True,
                         max_seq_len=ctx)
    sink = torch.randn(H, device=dev)
    t = timed(lambda: ops.mqa_attention(q, cache, 1.0, fb, cfg.softmax_scale, ps, sink, table, 64), iters)
    report("v4_mqa_sink", f"B={T} ctx={ctx} H={H} (q prep + latent attention + sink/inverse-rope fix-up)", t,
           nbytes=T * ctx * 576 + T * H * 512 * 2 * 2, flops=2 * T * H * ctx * (512 + 512))
    rows = 1 << 20
    tab = host_mapped_copy(torch.randint(0, 256, (rows, 256), dtype=torch.uint8) & 0xBF)
    sc = host_mapped_copy(torch.full((rows, 8), 122, dtype=torch.uint8))
    ids = torch.randint(0, rows, (T, 100), dtype=torch.int32, device=dev)
    out = torch.empty(T * 100, 256, dtype=torch.bfloat16, device=dev)
    t = timed(lambda: _C.engram_gather(tab, sc, ids, 0, out), iters)
    report("v4_engram_gather", f"T={T} x 100 heads from mapped host memory", t, nbytes=T * 100 * (256 + 8),
           note="host-link bound")
    wts = torch.rand(T, 6, device=dev)
    eids = torch.randint(0, 384, (T, 6), dtype=torch.int32, device=dev)
    t = timed(lambda: cuda.e5_prune(wts.clone(), eids.clone(), cfg, 384), iters)
    report("v4_e5_prune", f"T={T} top6 of 384", t, note="includes two input copies")


# ---------------------------------------------------------------------------
# tactic tuning: measure every legal choice per decode shape, write a table
# (b200ds/ops/tactics.py) that B200_TACTICS=<file> loads
TUNE_GEMMS = [  # DeepSeek-V3 671B decode GEMMs (N, K) at TP1 and TP8 widths
    ("qkv_a", 2176, 7168), ("q_b", 24576, 1536), ("q_b_tp8", 3072, 1536), ("o_proj", 7168, 16384),
    ("o_proj_tp8", 7168, 2048), ("shared_gate_up", 4096, 7168), ("shared_down", 7168, 2048),
    ("dense_down_tp8", 7168, 2304)]
TUNE_ROWS = (1, 8, 16, 32, 64, 128)


def tune(path: str, iters: int, quick: bool = False) -> None:
    """quick: one GEMM shape at two row counts and one MLA shape (a smoke run
    of the whole procedure)."""
    from b200ds.ops import QAct, cuda, tactics
    dev = torch.device("cuda")
    table = {"gemm_splits": [], "mla_splits": []}
    gemms = TUNE_GEMMS[:1] if quick else TUNE_GEMMS
    rows = (8, 64) if quick else TUNE_ROWS
    for name, N, K in gemms:
        w = _mx((), N, K, dev)
        for T in rows:
            x = cuda.quant(torch.randn(T, K, device=dev).to(torch.bfloat16))
            tactics.set_table({})
            default = cuda.choose_splits(T, N, K)
            times = {}
            for s in (1, 2, 4, 8):
                if not tactics._LEGAL["gemm_splits"](s, dict(N=N, K=K, rows=T, max_ctas=2 * 148)):
                    continue
                tactics.set_table({"gemm_splits": [{"N": N, "K": K, "rows": T, "value": s}]})
                times[s] = timed(lambda: cuda.gemm(QAct(x.q, x.sf), w), iters)
            best = min(times, key=times.get)
            table["gemm_splits"].append({"N": N, "K": K, "rows": T, "value": best})
            print(json.dumps({"tune": f"gemm_{name}", "T": T, "default": default, "best": best,
                              "us": {str(k): round(v * 1e6, 2) for k, v in times.items()}}), flush=True)
    for H in ((16,) if quick else (16, 128)):
        for B in ((8,) if quick else (8, 64)):
            times = {}
            for s in (1, 2, 3, 4, 6, 8):
                tactics.set_table({"mla_splits": [{"H": H, "rows": B, "keys": [0, 2048], "value": s}]})
                times[s] = run_mla(B, 1040, H, iters)
            best = min(times, key=times.get)
            table["mla_splits"].append({"H": H, "rows": B, "keys": [0, 2048], "value": best})
            print(json.dumps({"tune": "mla_decode", "H": H, "B": B, "best": best,
                              "us": {str(k): round(v * 1e6, 2) for k, v in times.items()}}), flush=True)
    tactics.set_table(None)
    tactics.write(table, path)
    print(json.dumps({"tactics_table": path, "entries": sum(len(v) for v in table.values())}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--small", action="store_true", help="reduced sizes (ncu captures)")
    ap.add_argument("--tune", default="", help="measure the legal tactics and write this tactics table (JSON)")
    ap.add_argument("--tune-quick", action="store_true", help="with --tune: a reduced set of shapes")
    a = ap.parse_args()
    import b200ds._C  # noqa: F401
    from b200ds import ops
    ops.set_impl("native")
    torch.cuda.set_device(0)
    if a.tune:
        tune(a.tune, a.iters, quick=a.tune_quick)
        return
    small = a.small
    cases = [
        # grouped MoE at the headline decode step: 64 tokens x top-8 over 256 experts
        ("moe_mxfp8_T64_ep1", lambda: run_moe("mxfp8", 64, 256, 64 if small else 256, a.iters)),
        ("moe_mxfp8_T64_ep8", lambda: run_moe("mxfp8", 64, 256, 32, a.iters)),
        ("moe_nvfp4_T256_ep8", lambda: run_moe("nvfp4", 256, 256, 32, a.iters)),
        ("moe_nvfp4_T64_ep1", lambda: run_moe("nvfp4", 64, 256, 64 if small else 256, a.iters)),
        # FC1 + FC2 in one persistent launch (dynamic work grabbing, FC2 fills FC1's tail)
        ("moe_mxfp8_T64_ep1_fused", lambda: run_moe("mxfp8", 64, 256, 64 if small else 256, a.iters, fused=True)),
        ("moe_mxfp8_T64_ep8_fused", lambda: run_moe("mxfp8", 64, 256, 32, a.iters, tiled=True, fused=True)),
        ("moe_nvfp4_T256_ep8_fused", lambda: run_moe("nvfp4", 256, 256, 32, a.iters, tiled=True, fused=True)),
        ("moe_nvfp4_T64_ep1_fused", lambda: run_moe("nvfp4", 64, 256, 64 if small else 256, a.iters, fused=True)),
        ("moe_mxfp8_T64_ep1_pull", lambda: run_moe("mxfp8", 64, 256, 64 if small else 256, a.iters, fused=True,
                                                    pull=True)),
        ("moe_mxfp8_T64_ep8_pull", lambda: run_moe("mxfp8", 64, 256, 32, a.iters, tiled=True, fused=True, pull=True)),
        ("moe_nvfp4_T256_ep8_pull", lambda: run_moe("nvfp4", 256, 256, 32, a.iters, tiled=True, fused=True,
                                                     pull=True)),
        ("moe_nvfp4_T64_ep1_pull", lambda: run_moe("nvfp4", 64, 256, 64 if small else 256, a.iters, fused=True,
                                                    pull=True)),
        # the same with weights stored as contiguous 128 x 128-byte tiles
        ("moe_mxfp8_T64_ep1_tiled", lambda: run_moe("mxfp8", 64, 256, 64 if small else 256, a.iters, tiled=True)),
        ("moe_mxfp8_T64_ep8_tiled", lambda: run_moe("mxfp8", 64, 256, 32, a.iters, tiled=True)),
        ("moe_nvfp4_T256_ep8_tiled", lambda: run_moe("nvfp4", 256, 256, 32, a.iters, tiled=True)),
        ("moe_nvfp4_T64_ep1_tiled", lambda: run_moe("nvfp4", 64, 256, 64 if small else 256, a.iters, tiled=True)),
        ("mla_decode_B64_1k_H128", lambda: run_mla(64, 1040, 128, a.iters)),
        ("mla_decode_B64_1k_H16", lambda: run_mla(64, 1040, 16, a.iters)),
        ("mla_sweep_B64_1k_H128", lambda: mla_sweep(64, 1040, 128, a.iters)),
        ("mla_sweep_B64_1k_H16", lambda: mla_sweep(64, 1040, 16, a.iters)),
        ("mla_sparse_B8_32k_H128", lambda: run_mla(8, 8192 if small else 32768, 128, a.iters, topk=2048)),
        ("indexer_B8_32k", lambda: run_indexer(8, 8192 if small else 32768, a.iters)),
        ("gemm_qkv_a_T64", lambda: run_gemm("qkv_a", 64, 2176, 7168, a.iters)),
        ("gemm_o_proj_T64", lambda: run_gemm("o_proj", 64, 7168, 16384, a.iters)),
        ("gemm_o_proj_tp8_T64", lambda: run_gemm("o_proj_tp8", 64, 7168, 2048, a.iters)),
        ("add_rmsnorm_quant_T64", lambda: run_norm(64, a.iters)),
        # prefill shapes (compute-bound)
        ("gemm_dense_T4096", lambda: run_gemm("dense_T4096", 1024 if small else 4096, 7168, 7168, a.iters)),
        ("gemm_o_proj_T512", lambda: run_gemm("o_proj_T512", 512, 7168, 2048, a.iters)),
        ("moe_mxfp8_T2048_ep1", lambda: run_moe("mxfp8", 512 if small else 2048, 256, 64 if small else 256,
                                                 a.iters)),
        # a 16K-token prefill chunk: ~512 rows per expert, 128 / 256-token tiles
        ("moe_mxfp8_T16384_ep1", lambda: run_moe("mxfp8", 2048 if small else 16384, 256, 32 if small else 256,
                                                  a.iters)),
        ("moe_nvfp4_T16384_ep1", lambda: run_moe("nvfp4", 2048 if small else 16384, 256, 32 if small else 256,
                                                  a.iters)),
        ("v4_T64", lambda: run_v4(64, a.iters)),
    ]
    for name, fn in cases:
        if a.only and a.only not in name:
            continue
        fn()


if __name__ == "__main__":
    main()
