"""Plain-PyTorch fp32 reference implementations of every hot op.

Each CUDA kernel in csrc/ is tested against the function of the same name
here; the CPU execution path of the engine also runs these.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn.functional as F

from .quant import E4M3_MAX, dequant_mxfp8, quant_mxfp8_ref, ue8m0_ceil_exponent


# -- norms -----------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float):
    """residual += x; returns (rmsnorm(residual), residual)."""
    r = residual.float() + x.float()
    return rmsnorm(r, w, eps), r


def rmsnorm_quant(x, w, eps):
    return quant_mxfp8_ref(rmsnorm(x, w, eps))


# -- gemm --------------------------------------------------------------------------

def gemm_mxfp8(a_q, a_sf, w_q, w_sf) -> torch.Tensor:
    """D[T, N] = dequant(A)[T, K] @ dequant(W)[N, K]^T in fp32."""
    return dequant_mxfp8(a_q, a_sf) @ dequant_mxfp8(w_q, w_sf).T


def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    """gate_up [T, 2I] (gate first) -> silu(gate) * up [T, I]."""
    I = gate_up.shape[-1] // 2
    g, u = gate_up[..., :I].float(), gate_up[..., I:].float()
    return F.silu(g) * u


# -- rope ---------------------------------------------------------------------------

def rope(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """Interleaved-pair rotation. x [T, ..., d], pos [T], table [P, d] (cos|sin)."""
    d = x.shape[-1]
    cs = table[pos.long()].float()
    cos, sin = cs[:, : d // 2], cs[:, d // 2:]
    while cos.dim() < x.dim():
        cos, sin = cos.unsqueeze(-2), sin.unsqueeze(-2)
    xf = x.float()
    x0, x1 = xf[..., 0::2], xf[..., 1::2]
    return torch.stack([x0 * cos - x1 * sin, x0 * sin + x1 * cos], -1).flatten(-2)


# -- routing -------------------------------------------------------------------------

def router_topk(logits: torch.Tensor, bias: torch.Tensor, topk: int, n_group: int,
                topk_group: int, scaling: float, renorm: bool = True):
    """Sigmoid scores, group-limited top-k (sum of top-2 per group), weights
    renormalised and scaled.  Returns (weights fp32 [T,k], ids int32 [T,k])."""
    scores = logits.float().sigmoid()
    choice = scores + bias.float()
    T, E = scores.shape
    if n_group > 1:
        g = choice.view(T, n_group, E // n_group)
        gscore = g.topk(2, dim=-1).values.sum(-1)
        gidx = gscore.topk(topk_group, dim=-1).indices
        gmask = torch.zeros_like(gscore).scatter_(1, gidx, 1.0)
        emask = gmask.unsqueeze(-1).expand(T, n_group, E // n_group).reshape(T, E)
        choice = choice.masked_fill(emask == 0, float("-inf"))
    ids = choice.topk(topk, dim=-1).indices
    w = scores.gather(1, ids)
    if renorm and topk > 1:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return w * scaling, ids.to(torch.int32)


# -- attention ------------------------------------------------------------------------

def kv_quant(ckv: torch.Tensor, kpe: torch.Tensor, kv_scale: float) -> torch.Tensor:
    """Latent cache entry: e4m3([ckv | kpe] / kv_scale) -> [T, 576] e4m3."""
    x = torch.cat([ckv.float(), kpe.float()], -1) / kv_scale
    return x.clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)


def mla_attention(q_abs: torch.Tensor, q_pe: torch.Tensor, kv_cache: torch.Tensor,
                  kv_scale: float, block_table: torch.Tensor, seq_lens: torch.Tensor,
                  q_seq: torch.Tensor, q_pos: torch.Tensor, softmax_scale: float,
                  page_size: int, topk_idx: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Absorbed MLA over a paged fp8 latent cache (fp32 math).

    q_abs [T, H, L] (L = kv_lora_rank), q_pe [T, H, R]; kv_cache
    [pages*page_size, L+R] e4m3; block_table [B, max_pages]; seq_lens [B];
    q_seq [T] sequence index per query; q_pos [T] absolute position (query
    attends to cache positions <= q_pos).  topk_idx [T, k] (optional, -1 =
    unused) restricts each query to those cache positions (sparse MLA).
    Returns latent output [T, H, L] fp32."""
    T, H, L = q_abs.shape
    out = torch.zeros(T, H, L, dtype=torch.float32, device=q_abs.device)
    kvf = kv_cache.float() * kv_scale
    for t in range(T):
        b = int(q_seq[t])
        n = int(q_pos[t]) + 1
        pos = torch.arange(n, device=q_abs.device)
        if topk_idx is not None:
            sel = topk_idx[t]
            sel = sel[(sel >= 0) & (sel < n)].long()
            pos = sel
        pages = block_table[b, (pos // page_size).long()].long()
        slots = pages * page_size + pos % page_size
        kv = kvf[slots]                                   # [n, L+R]
        s = q_abs[t].float() @ kv[:, :L].T + q_pe[t].float() @ kv[:, L:].T   # [H, n]
        p = (s * softmax_scale).softmax(-1)
        out[t] = p @ kv[:, :L]
    return out


def indexer_scores(q: torch.Tensor, w: torch.Tensor, k_cache: torch.Tensor, k_scale: torch.Tensor,
                   block_table: torch.Tensor, q_seq: torch.Tensor, q_pos: torch.Tensor,
                   page_size: int, topk: int) -> torch.Tensor:
    """Lightning indexer top-k: score[s] = sum_h w[t,h] * relu(q[t,h] . k[s]).

    q [T, Hi, D] (float), w [T, Hi], k_cache [slots, D] e4m3 with per-token
    fp32 k_scale [slots].  Returns top-k cache positions [T, topk] int32
    (-1 padded), causal (positions <= q_pos)."""
    T = q.shape[0]
    out = torch.full((T, topk), -1, dtype=torch.int32, device=q.device)
    for t in range(T):
        b = int(q_seq[t])
        n = int(q_pos[t]) + 1
        pos = torch.arange(n, device=q.device)
        pages = block_table[b, (pos // page_size).long()].long()
        slots = pages * page_size + pos % page_size
        k = k_cache[slots].float() * k_scale[slots].float().unsqueeze(-1)
        sc = ((q[t].float() @ k.T).relu() * w[t].float().unsqueeze(-1)).sum(0)
        kk = min(topk, n)
        idx = sc.topk(kk).indices
        out[t, :kk] = idx.sort().values.to(torch.int32)
    return out


# -- sampling ----------------------------------------------------------------------------

def sample(logits: torch.Tensor, temperature: torch.Tensor, top_p: torch.Tensor,
           top_k: torch.Tensor, uniform: torch.Tensor) -> torch.Tensor:
    """Per-row sampling with temperature (<=0 -> greedy), top-k (<=0 -> off)
    and top-p, driven by a given uniform draw per row (reproducible)."""
    T, V = logits.shape
    out = torch.empty(T, dtype=torch.int64, device=logits.device)
    for i in range(T):
        row = logits[i].float()
        if float(temperature[i]) <= 0:
            out[i] = row.argmax()
            continue
        p = (row / float(temperature[i])).softmax(-1)
        sp, si = p.sort(descending=True)
        keep = torch.ones_like(sp, dtype=torch.bool)
        k = int(top_k[i])
        if k > 0:
            keep[k:] = False
        c = sp.cumsum(0)
        keep &= (c - sp) < float(top_p[i])
        sp = torch.where(keep, sp, torch.zeros_like(sp))
        c = sp.cumsum(0)
        u = float(uniform[i]) * float(c[-1])
        j = int(torch.searchsorted(c, torch.tensor([u], device=c.device)).clamp(max=V - 1))
        out[i] = si[j]
    return out
