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
    try:
        import flashinfer.fused_moe  # noqa: F401
        import flashinfer.decode  # noqa: F401
        return True
    except Exception:
        return False


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
