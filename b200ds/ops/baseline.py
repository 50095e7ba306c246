"""Library baseline for the GPU path: cuBLAS block-scaled GEMM through
torch._scaled_mm (MXFP8, the same sf128x4 scale layout), PyTorch elementwise
ops and NCCL collectives.  This is the comparison arm of the benchmarks, not
a fallback: it runs only under ``ops.set_impl("torch")``."""
from __future__ import annotations

import torch

from .quant import MXFP8Tensor, dequant_mxfp8, quant_mxfp8_ref

_SCALED_MM_OK = None


def _qact(q, sf, hf=None):
    from . import QAct
    return QAct(q, sf, hf)


def quant(x: torch.Tensor):
    q, sf = quant_mxfp8_ref(x.float())
    return _qact(q, sf)


def rmsnorm_quant(x, w, eps, keep_hf=True):
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    a = quant(y)
    a.hf = y.to(torch.bfloat16) if keep_hf else None
    return a


def gemm(a, w: MXFP8Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    global _SCALED_MM_OK
    T, K = a.q.shape
    N = w.data.shape[0]
    if _SCALED_MM_OK is not False:
        try:
            sa = a.sf.view(torch.float8_e8m0fnu)
            sb = w.sf.view(torch.float8_e8m0fnu)
            out = torch._scaled_mm(a.q, w.data.t(), scale_a=sa, scale_b=sb, out_dtype=torch.bfloat16)
            _SCALED_MM_OK = True
            return out.to(out_dtype)
        except Exception:
            _SCALED_MM_OK = False
    return (dequant_mxfp8(a.q, a.sf).to(torch.bfloat16) @ dequant_mxfp8(w.data, w.sf).to(torch.bfloat16).t()).to(out_dtype)


def _rows(ex, name: str, e: int) -> torch.Tensor:
    """Expert e's weight as a plain row-major matrix (undoing the tiled
    serving layout when the experts use it)."""
    d = getattr(ex, name).data[e]
    if getattr(ex, "tiled", False):
        from .quant import untile_rows128
        d = untile_rows128(d.view(torch.uint8)).view(d.dtype)
    return d


def moe_experts(a, w, ids, ex, out_dtype=torch.bfloat16):
    """Per-expert loop over library GEMMs (host-synchronising)."""
    T = a.q.shape[0]
    out = torch.zeros(T, a.q.shape[1], dtype=torch.float32, device=a.q.device)
    ids_c = ids.cpu()
    for e in range(ex.count):
        gid = ex.first + e
        hit = (ids_c == gid)
        tok = hit.any(-1).nonzero().flatten()
        if tok.numel() == 0:
            continue
        tok_d = tok.to(a.q.device)
        we = (w * hit.to(w.device)).sum(-1)[tok_d].unsqueeze(-1)
        xe = _qact(a.q[tok_d], None)
        xf = dequant_mxfp8(a.q, a.sf)[tok_d]
        xe = quant(xf)
        w13, w2 = _rows(ex, "w13", e), _rows(ex, "w2", e)
        y = gemm(xe, MXFP8Tensor(w13, ex.w13.sf[e]), torch.float32)
        I = y.shape[1] // 2
        h = torch.nn.functional.silu(y[:, :I]) * y[:, I:]
        o = gemm(quant(h), MXFP8Tensor(w2, ex.w2.sf[e]), torch.float32)
        out.index_add_(0, tok_d, we * o)
    return out.to(out_dtype)


# ---------------------------------------------------------------------------
# Stock-library kernels of the comparison arm: FlashInfer's trtllm-gen fused
# MoE (DeepSeek FP8: e4m3 weights with 128 x 128 block scales, activations
# with 1 x 128 scales) and trtllm-gen MLA decode over the fp8 latent cache -
# the kernel families the reference's served stack calls (mo.py:19-40,
# bsa.py:50-57) - plus cuBLAS (torch matmul / _scaled_mm) for the rest.
# ---------------------------------------------------------------------------
_FI_WS = {}


def flashinfer_ok() -> bool:
    """FlashInfer's trtllm-gen launchers are JIT-compiled on first use (many
    minutes offline); the arm uses them only when B200_BASELINE_FLASHINFER=1
    and the modules import."""
    import os
    if os.environ.get("B200_BASELINE_FLASHINFER", "0") != "1":
        return False
    try:
        import flashinfer.fused_moe  # noqa: F401
        import flashinfer.decode  # noqa: F401
        return True
    except Exception:
        return False


# ---------------------------------------------------------------------------
# Library MoE and decode attention (no FlashInfer): PyTorch ops with static
# shapes (no host synchronisation, CUDA-graph capturable) around the MXFP8
# grouped GEMM of the PyTorch build (F.scaled_grouped_mm: e4m3 operands with
# UE8M0 per-32 scales in the 32_4_4 swizzled layout, which is the layout our
# MXFP8 tensors already use).
# ---------------------------------------------------------------------------
_GROUPED_MX_OK = None


def _scaled_grouped(aq, asf, w, offs):
    """[R, K] MXFP8 rows (groups at offs, 128-row aligned) x expert weights
    w [E, N, K] (MXFP8) -> [R, N] bf16.  The rows' scales go in as [R, K/32],
    each expert's as one row of its blocked (32_4_4) scale bytes [E, N*K/32]:
    the shapes PyTorch's 2d x 3d block-scaled grouped GEMM accepts (checked
    on a B200: 1.7e-3 relative to the dequantized product)."""
    import torch.nn.functional as F
    R, K = aq.shape
    E, N = w.data.shape[0], w.data.shape[1]
    sw = F.SwizzleType.SWIZZLE_32_4_4
    return F.scaled_grouped_mm(aq.view(torch.float8_e4m3fn), w.data.view(torch.float8_e4m3fn).transpose(-2, -1),
                               asf.view(torch.float8_e8m0fnu).view(R, K // 32), F.ScalingType.BlockWise1x32,
                               w.sf.view(torch.float8_e8m0fnu).view(E, -1), F.ScalingType.BlockWise1x32,
                               swizzle_a=sw, swizzle_b=sw, offs=offs, output_dtype=torch.bfloat16)


def moe_experts_grouped(x: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, ex, out_dtype=torch.bfloat16):
    """Routed experts of this rank through two library grouped MXFP8 GEMMs:
    the (token, choice) pairs of local experts are sorted by expert into
    128-row-aligned groups (PyTorch scatter / sort / cumsum on the device),
    quantized per 32, FC1 -> SwiGLU -> requantize -> FC2, and the weighted
    rows are summed per token.  Experts in the tiled serving layout are
    untiled once (random-init bytes are read row-major as they are: the
    native kernels' tiled reading of the same bytes is another random matrix
    of the same distribution)."""
    if getattr(ex, "tiled", False) and not getattr(ex, "random_init", False):
        ex = _untiled(ex)
    T, H = x.shape
    K = ids.shape[1]
    E = ex.count
    dev = x.device
    e = ids.reshape(-1).long() - ex.first
    valid = (e >= 0) & (e < E)
    ek = torch.where(valid, e, torch.full_like(e, E))
    counts = torch.zeros(E + 1, dtype=torch.long, device=dev).scatter_add_(0, ek, torch.ones_like(ek))[:E]
    padded = (counts + 127) // 128 * 128
    pstart = torch.cumsum(padded, 0) - padded
    ustart = torch.cumsum(counts, 0) - counts
    order = torch.argsort(ek, stable=True)
    es = ek.index_select(0, order)
    ec = es.clamp(max=E - 1)
    rank = torch.arange(order.numel(), device=dev) - ustart.index_select(0, ec)
    R = (T * K + 127) // 128 * 128 + E * 128 + 128          # static bound; the last row takes unrouted pairs
    dest = torch.where(es < E, pstart.index_select(0, ec) + rank, torch.full_like(rank, R - 1))
    tok = order // K
    rows = torch.zeros(R, H, dtype=torch.bfloat16, device=dev)
    rows.index_copy_(0, dest, x.to(torch.bfloat16).index_select(0, tok))
    rows[R - 1].zero_()
    offs = torch.cumsum(padded, 0).to(torch.int32)
    aq, asf = quant_mxfp8_ref(rows)
    y1 = _scaled_grouped(aq, asf, ex.w13, offs)
    I = ex.inter
    h = torch.nn.functional.silu(y1[:, :I].float()) * y1[:, I:2 * I].float()
    hq, hsf = quant_mxfp8_ref(h)
    y2 = _scaled_grouped(hq, hsf, ex.w2, offs)
    wp = (w.reshape(-1).float().index_select(0, order) * (es < E)).unsqueeze(1)
    contrib = y2.index_select(0, dest).float() * wp
    out = torch.zeros(T, H, dtype=torch.float32, device=dev).index_add_(0, tok, contrib)
    return out.to(out_dtype)


def _untiled(ex):
    """Row-major copy of tiled expert weights, kept on the ExpertWeights
    object (it lives and dies with the weights)."""
    from .quant import untile_rows128
    import dataclasses
    u = getattr(ex, "_untiled", None)
    if u is None:
        f = lambda t: MXFP8Tensor(untile_rows128(t.data.view(torch.uint8)).view(t.data.dtype), t.sf, t.rows)
        u = dataclasses.replace(ex, w13=f(ex.w13), w2=f(ex.w2), tiled=False)
        object.__setattr__(ex, "_untiled", u)
    return u


def grouped_mx_ok(dev) -> bool:
    """Whether this PyTorch build runs the MXFP8 grouped GEMM here (checked
    once on a tiny case against the per-expert library GEMM)."""
    global _GROUPED_MX_OK
    if _GROUPED_MX_OK is None:
        try:
            import torch.nn.functional as F  # noqa: F401
            from . import ExpertWeights
            g = torch.Generator(device=dev).manual_seed(0)
            E, H, I, T, K = 2, 256, 128, 8, 2
            mk = lambda n, k: MXFP8Tensor(*quant_mxfp8_ref(torch.randn(E * n, k, device=dev, generator=g) * 0.1))
            w13, w2 = mk(2 * I, H), mk(H, I)
            ex = ExpertWeights(0, E, MXFP8Tensor(w13.data.view(E, 2 * I, H), w13.sf.view(E, -1)),
                               MXFP8Tensor(w2.data.view(E, H, I), w2.sf.view(E, -1)), I)
            x = torch.randn(T, H, device=dev, generator=g)
            ids = torch.stack([torch.randperm(E, device=dev)[:K] for _ in range(T)]).int()
            wt = torch.rand(T, K, device=dev)
            got = moe_experts_grouped(x, wt, ids, ex, torch.float32)
            want = moe_experts(quant(x), wt, ids, ex, torch.float32)
            _GROUPED_MX_OK = bool(((got - want).norm() / want.norm()).item() < 0.1)
        except Exception:
            _GROUPED_MX_OK = False
    return _GROUPED_MX_OK


def mla_decode_torch(q_abs: torch.Tensor, q_pe: torch.Tensor, cache: torch.Tensor, kv_scale: float, fb,
                     softmax_scale: float, page_size: int) -> torch.Tensor:
    """Absorbed MLA decode (one query row per sequence) in PyTorch ops with
    static shapes: every sequence's block-table rows are gathered and
    dequantized to bf16 [B, pages * page_size, 576], S = q . K^T by cuBLAS
    batched GEMM, positions past the query masked, fp32 softmax, O = P . V.
    Returns the latent output [B, H, 512] bf16."""
    B, H, L = q_abs.shape
    bt = fb.block_table.long()
    S = bt.shape[1] * page_size
    slots = (bt.unsqueeze(-1) * page_size + torch.arange(page_size, device=bt.device)).view(B, S)
    kv = (cache.index_select(0, slots.view(-1)).float() * kv_scale).to(torch.bfloat16).view(B, S, -1)
    q = torch.cat([q_abs.to(torch.bfloat16), q_pe.to(torch.bfloat16)], -1)
    s = torch.matmul(q, kv.transpose(1, 2)).float() * softmax_scale                 # [B, H, S]
    mask = torch.arange(S, device=q.device).unsqueeze(0) > fb.positions.long().unsqueeze(1)
    s.masked_fill_(mask.unsqueeze(1), float("-inf"))
    p = torch.softmax(s, -1).to(torch.bfloat16)
    return torch.matmul(p, kv[..., :L])


def _block128_scales(t: MXFP8Tensor, E: int, N: int, K: int) -> torch.Tensor:
    """fp32 [E, N/128, K/128] block scales of the same e4m3 bytes.  Exact when
    every per-32 scale of a 128 x 128 block is equal (random-init weights);
    otherwise the block takes its largest per-32 scale and the data are
    re-quantized (one expert at a time) so the values are kept to e4m3
    precision."""
    sf = t.sf.view(E, -1)
    lo, hi = int(sf.min()), int(sf.max())
    if lo == hi:
        return torch.full((E, N // 128, K // 128), 2.0 ** (lo - 127), dtype=torch.float32, device=sf.device)
    out = torch.empty(E, N // 128, K // 128, dtype=torch.float32, device=sf.device)
    for e in range(E):
        w = dequant_mxfp8(t.data[e][:N], t.sf[e]).float()
        blk = w.view(N // 128, 128, K // 128, 128).abs().amax(dim=(1, 3)).clamp(min=1e-30)
        s = torch.exp2(torch.ceil(torch.log2(blk / 448.0)))
        out[e] = s
        q = (w.view(N // 128, 128, K // 128, 128) / s[:, None, :, None]).view(N, K)
        t.data[e][:N].copy_(q.to(torch.float8_e4m3fn))
    return out


def _expert_block_weights(ex):
    """(w13 e4m3 [E, 2I, h], s13, w2 [E, h, I], s2) in the DeepSeek FP8 block
    format, cached on the ExpertWeights (the bytes are shared with the MXFP8
    tensors; experts stored in the tiled layout are read as plain rows, which
    for random-init weights is the same distribution)."""
    c = getattr(ex, "_fi_block", None)
    if c is not None:
        return c
    E, I = ex.count, ex.inter
    h = ex.w2.data.shape[1]
    w13 = ex.w13.data.view(torch.float8_e4m3fn)[:, : 2 * I]
    w2 = ex.w2.data.view(torch.float8_e4m3fn)[:, :h]
    s13 = _block128_scales(ex.w13, E, 2 * I, h)
    s2 = _block128_scales(ex.w2, E, h, I)
    ex._fi_block = (w13.contiguous(), s13, w2.contiguous(), s2)
    return ex._fi_block


def quant_block128(x: torch.Tensor):
    """bf16 [T, K] -> (e4m3 [T, K], fp32 scales [K/128, T]) with one power-of-two
    scale per 128 elements of a row."""
    T, K = x.shape
    xf = x.float().view(T, K // 128, 128)
    s = torch.exp2(torch.ceil(torch.log2(xf.abs().amax(-1).clamp(min=1e-30) / 448.0)))
    q = (xf / s.unsqueeze(-1)).to(torch.float8_e4m3fn).view(T, K)
    return q, s.t().contiguous()


def moe_experts_flashinfer(x_bf16: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, ex,
                           n_experts_total: int) -> torch.Tensor:
    """Local-expert partial of the MoE through FlashInfer's trtllm-gen
    FP8 block-scale fused MoE with precomputed routing (ids / weights packed
    as (id << 16) | bf16 weight bits): gather, FC1 + SwiGLU, FC2 and the
    weighted finalize in the library's kernels.  Returns bf16 [T, h]."""
    from flashinfer.fused_moe import RoutingMethodType, trtllm_fp8_block_scale_routed_moe
    w13, s13, w2, s2 = _expert_block_weights(ex)
    hq, hs = quant_block128(x_bf16)
    packed = (ids.to(torch.int32) << 16) | (w.to(torch.bfloat16).view(torch.int16).to(torch.int32) & 0xFFFF)
    out = trtllm_fp8_block_scale_routed_moe(
        packed, None, hq, hs, w13, s13, w2, s2, n_experts_total, ids.shape[1], None, None, ex.inter,
        ex.first, ex.count, None, routing_method_type=int(RoutingMethodType.DeepSeekV3),
        use_shuffled_weight=False, weight_layout=0, do_finalize=True)
    return out


def _workspace(dev) -> torch.Tensor:
    ws = _FI_WS.get(dev)
    if ws is None:
        ws = _FI_WS[dev] = torch.zeros(128 << 20, dtype=torch.uint8, device=dev)
    return ws


def mla_decode_flashinfer(q_abs: torch.Tensor, q_pe: torch.Tensor, cache: torch.Tensor, kv_scale: float, fb,
                          softmax_scale: float, page_size: int) -> torch.Tensor:
    """Absorbed MLA decode (one query row per sequence) through FlashInfer's
    trtllm-gen MLA kernel over the paged e4m3 latent cache; the query is cast
    to e4m3 (unit scale).  Returns the latent output [T, H, 512] bf16."""
    from flashinfer.decode import trtllm_batch_decode_with_kv_cache_mla
    T, H, L = q_abs.shape
    q = torch.cat([q_abs.to(torch.bfloat16), q_pe.to(torch.bfloat16)], -1).to(torch.float8_e4m3fn)
    kv = cache.view(-1, page_size, cache.shape[-1])
    out = trtllm_batch_decode_with_kv_cache_mla(
        q.view(T, 1, H, -1), kv, _workspace(q.device), 128, L, q_pe.shape[-1], fb.block_table,
        fb.seq_lens, int(fb.max_seq_len), bmm1_scale=float(softmax_scale * kv_scale), bmm2_scale=float(kv_scale))
    return out.view(T, H, L)


def mla_prefill_torch(q_abs: torch.Tensor, q_pe: torch.Tensor, cache: torch.Tensor, kv_scale: float, fb,
                      softmax_scale: float, page_size: int, head_chunk: int = 32) -> torch.Tensor:
    """Absorbed MLA for prefill chunks with cuBLAS batched GEMMs: per
    sequence, S = [q_abs | q_pe] . K^T over its cached latent rows (dequantized
    to bf16), causal mask, softmax in fp32, O = P . V_latent.  Returns the
    latent output [T, H, 512] bf16."""
    T, H, L = q_abs.shape
    out = torch.empty(T, H, L, dtype=torch.bfloat16, device=q_abs.device)
    qs = fb.q_seq.long().cpu()
    pos = fb.positions.long().cpu()
    lens = fb.seq_lens.long().cpu()
    bt = fb.block_table.long()
    q = torch.cat([q_abs.to(torch.bfloat16), q_pe.to(torch.bfloat16)], -1)
    starts = torch.nonzero(torch.diff(qs, prepend=torch.tensor([-1]))).flatten().tolist() + [T]
    for i in range(len(starts) - 1):
        r0, r1 = starts[i], starts[i + 1]
        b = int(qs[r0])
        n_k = int(lens[b])
        npg = (n_k + page_size - 1) // page_size
        slots = (bt[b, :npg].unsqueeze(1) * page_size + torch.arange(page_size, device=bt.device)).flatten()[:n_k]
        kv = (cache[slots].float() * kv_scale).to(torch.bfloat16)              # [n_k, 576]
        qpos = pos[r0:r1].to(q.device)
        mask = torch.arange(n_k, device=q.device).unsqueeze(0) > qpos.unsqueeze(1)   # [n_q, n_k]
        for h0 in range(0, H, head_chunk):
            qh = q[r0:r1, h0:h0 + head_chunk].transpose(0, 1)                   # [hc, n_q, 576]
            s = torch.matmul(qh, kv.t()).float() * softmax_scale                 # [hc, n_q, n_k]
            s.masked_fill_(mask.unsqueeze(0), float("-inf"))
            p = torch.softmax(s, -1).to(torch.bfloat16)
            out[r0:r1, h0:h0 + head_chunk] = torch.matmul(p, kv[:, :L]).transpose(0, 1)
    return out


def prebuild_flashinfer(workspace: str) -> None:
    """Compile the FlashInfer JIT modules the comparison arm uses (trtllm-gen
    fused MoE and MLA decode launchers) for sm_100a into `workspace` (the
    FLASHINFER_WORKSPACE_BASE the bench's baseline arm points at).  Runs on a
    machine without a GPU; the kernels themselves come from FlashInfer's
    packaged cubins."""
    import os
    os.environ["FLASHINFER_WORKSPACE_BASE"] = workspace
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0a")
    from flashinfer.jit.attention.modules import gen_trtllm_gen_fmha_module
    from flashinfer.fused_moe.core import gen_trtllm_gen_fused_moe_sm100_module
    for spec in (gen_trtllm_gen_fused_moe_sm100_module(), gen_trtllm_gen_fmha_module()):
        spec.build(verbose=False)        # compile only (loading needs the driver)


if __name__ == "__main__":
    # python -m b200ds.ops.baseline prebuild [workspace]
    import os
    import sys
    if len(sys.argv) > 1 and sys.argv[1] == "prebuild":
        root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
        prebuild_flashinfer(sys.argv[2] if len(sys.argv) > 2 else os.path.join(root, "baseline", "_fi"))


def sample_torch(logits: torch.Tensor, temperature, top_p, top_k, uniform) -> torch.Tensor:
    """Batched sampling in PyTorch ops (no host synchronisation): greedy rows
    (temperature <= 0) take the argmax; the others draw from softmax(logits /
    temperature) restricted to top-k (<= 0: off) and top-p, by inverse CDF at
    the row's given uniform - the semantics of ref.sample."""
    T, V = logits.shape
    x = logits.float()
    t = temperature.float().clamp(min=1e-6).unsqueeze(1)
    p = (x / t).softmax(-1)
    sp, si = p.sort(-1, descending=True)
    ar = torch.arange(V, device=x.device).unsqueeze(0)
    k = top_k.long().unsqueeze(1)
    keep = (k <= 0) | (ar < k)
    c = sp.cumsum(-1)
    keep &= (c - sp) < top_p.float().unsqueeze(1)
    sp = sp * keep
    c = sp.cumsum(-1)
    u = uniform.float().unsqueeze(1) * c[:, -1:]
    j = torch.searchsorted(c, u).clamp(max=V - 1)
    tok = si.gather(1, j).squeeze(1)
    return torch.where(temperature.reshape(-1) <= 0, x.argmax(-1), tok)

