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
