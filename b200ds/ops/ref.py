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
                   page_size: int, topk: int, swa: int = 0) -> torch.Tensor:
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
        if swa > 0:
            sc[max(0, n - swa):] = float("inf")       # the window is always kept
        kk = min(topk, n)
        idx = sc.topk(kk).indices
        out[t, :kk] = idx.sort().values.to(torch.int32)
    return out


# -- sampling ----------------------------------------------------------------------------

def sampling_probs(logits: torch.Tensor, temperature: float, top_p: float, top_k: int) -> torch.Tensor:
    """The distribution `sample` draws from for one row: softmax(logits / T)
    restricted to the top-k, then to the smallest prefix (by probability) whose
    mass reaches top_p; unnormalised kept probabilities, zeros elsewhere."""
    p = (logits.float() / temperature).softmax(-1)
    sp, si = p.sort(descending=True)
    keep = torch.ones_like(sp, dtype=torch.bool)
    if top_k > 0:
        keep[top_k:] = False
    c = sp.cumsum(0)
    keep &= (c - sp) < top_p
    out = torch.zeros_like(p)
    out[si[keep]] = sp[keep]
    return out


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


# -- DeepSeek-V4 family ------------------------------------------------------------------
# mHC (hyper-connections over hc residual streams), sqrt-softplus routing with
# the E5 prune, MQA attention with sinks, Engram lookups.  Reference parity:
# sk_unit.cu:1-15 (coefficient epilogue: sigmoid pre / 2*sigmoid post,
# row-softmax + Sinkhorn comb), fin.py:218-246 (post: out_c = post_c * y +
# sum_r comb[r][c] * x_r), route_e5.cu:4-12 (sqrt-softplus top-k, E5 prune),
# eg_gather.cu:1-5 (e4m3 rows x 2^(e-127)).

def hc_stats(X: torch.Tensor, fn: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """X [T, hc, D] -> (raw mixes [T, M] = X_flat . fn^T, sum of squares [T])."""
    xf = X.float().flatten(1)
    return xf @ fn.float().T, xf.pow(2).sum(-1)


def sinkhorn(c: torch.Tensor, iters: int, eps: float) -> torch.Tensor:
    """[.., n, n] logits -> row softmax (+eps), then column / row
    normalisations (each sum + eps) ending on columns: iters column passes."""
    m = c.float().softmax(-1) + eps
    m = m / (m.sum(-2, keepdim=True) + eps)
    for _ in range(iters - 1):
        m = m / (m.sum(-1, keepdim=True) + eps)
        m = m / (m.sum(-2, keepdim=True) + eps)
    return m


def hc_coeffs(raw: torch.Tensor, sumsq: torch.Tensor, scale: torch.Tensor, base: torch.Tensor, hc: int,
              width: int, iters: int, eps: float):
    """Sublayer coefficients from the raw mixes: (pre [T,hc], post [T,hc],
    comb [T,hc,hc]); width = hc * hidden (the RMS divisor)."""
    r = torch.rsqrt(sumsq.float() / width + eps).unsqueeze(-1)
    s = scale.float()
    b = base.float()
    pre = torch.sigmoid(s[0] * r * raw[:, :hc] + b[:hc]) + eps
    post = 2.0 * torch.sigmoid(s[1] * r * raw[:, hc:2 * hc] + b[hc:2 * hc])
    c = (s[2] * r * raw[:, 2 * hc:2 * hc + hc * hc] + b[2 * hc:]).view(-1, hc, hc)
    return pre, post, sinkhorn(c, iters, eps)


def hc_head_coeffs(raw: torch.Tensor, sumsq: torch.Tensor, scale: torch.Tensor, base: torch.Tensor, hc: int,
                   width: int, eps: float) -> torch.Tensor:
    r = torch.rsqrt(sumsq.float() / width + eps).unsqueeze(-1)
    return torch.sigmoid(scale.float()[0] * r * raw[:, :hc] + base.float()[:hc]) + eps


def hc_combine(X: torch.Tensor, pre: torch.Tensor) -> torch.Tensor:
    return (pre.float().unsqueeze(-1) * X.float()).sum(1)


def hc_post(X: torch.Tensor, y: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
    """out[:, c] = post[:, c] * y + sum_r comb[:, r, c] * X[:, r]."""
    return post.float().unsqueeze(-1) * y.float().unsqueeze(1) + torch.einsum("trc,trd->tcd", comb.float(),
                                                                                X.float())


def router_sqrtsoftplus(logits: torch.Tensor, bias: torch.Tensor, topk: int, scaling: float):
    """score = sqrt(softplus(logit)); top-k by score + bias; weights = the
    chosen scores / (sum + 1e-20) x scaling."""
    s = F.softplus(logits.float()).sqrt()
    ids = (s + bias.float()).topk(topk, dim=-1).indices
    w = s.gather(1, ids)
    w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return w * scaling, ids.to(torch.int32)


def e5_prune(ids: torch.Tensor, w: torch.Tensor, budget: float, max_count: int):
    """E5 routed-expert prune of one batch (in place semantics, returns new
    tensors): an expert picked by <= max_count rows is eligible; in each row
    a pick's run is the sum of the eligible weights before it in (weight,
    slot) order plus its own; it is a candidate when eligible and run <=
    budget * the row's mass; an expert whose every pick is a candidate is
    dropped (id -1, weight 0; kept weights are not renormalised)."""
    ids = ids.clone()
    w = w.clone().float()
    T, K = ids.shape
    valid = ids >= 0
    count = {}
    for e in ids[valid].tolist():
        count[e] = count.get(e, 0) + 1
    elig = torch.tensor([[bool(valid[t, k]) and count.get(int(ids[t, k]), 0) <= max_count for k in range(K)]
                         for t in range(T)], dtype=torch.bool).reshape(T, K)
    cand = torch.zeros(T, K, dtype=torch.bool)
    for t in range(T):
        mass = float(w[t][valid[t]].sum())
        order = sorted(range(K), key=lambda k: (float(w[t, k]), k))
        run = 0.0
        for k in order:
            if not elig[t, k]:
                continue
            run += float(w[t, k])
            cand[t, k] = run <= budget * mass
    drop = set()
    for e in set(ids[valid].tolist()):
        picks = (ids == e)
        if bool(cand[picks].all()):
            drop.add(e)
    for t in range(T):
        for k in range(K):
            if int(ids[t, k]) in drop:
                ids[t, k] = -1
                w[t, k] = 0.0
    return w, ids


# A selection entry with this bit set names compressed block j = entry - COMP_FLAG
# of a compressed-attention layer (its row in the compressed cache), not a
# full-resolution position.
COMP_FLAG = 1 << 30


def comp_rows(block_table: torch.Tensor, b: int, j: torch.Tensor, r: int, page_size: int) -> torch.Tensor:
    """Rows of compressed blocks j of sequence b: block j covers positions
    j*r .. j*r + r - 1 (one page), stored at page * (page_size / r) +
    (j*r mod page_size) / r of the compressed tensors."""
    p0 = j.long() * r
    return block_table[b, (p0 // page_size).long()].long() * (page_size // r) + (p0 % page_size) // r


def mqa_sink_attention(q: torch.Tensor, kv_cache: torch.Tensor, kv_scale: float, block_table: torch.Tensor,
                       q_seq: torch.Tensor, q_pos: torch.Tensor, softmax_scale: float, page_size: int,
                       sink: Optional[torch.Tensor], L: int,
                       topk_idx: Optional[torch.Tensor] = None, comp=None) -> torch.Tensor:
    """MQA over the paged latent rows: K = V = cache[:, :L]; q [T, H, L];
    sink [H] (natural-log logits joining each head's softmax denominator).
    comp = (compressed rows, ratio): selection entries >= COMP_FLAG name
    compressed blocks (compressed attention)."""
    T, H, _ = q.shape
    out = torch.zeros(T, H, L, dtype=torch.float32, device=q.device)
    kvf = kv_cache.float() * kv_scale
    ckf = comp[0].float() * kv_scale if comp is not None else None
    for t in range(T):
        b = int(q_seq[t])
        n = int(q_pos[t]) + 1
        pos = torch.arange(n, device=q.device)
        kc = None
        if topk_idx is not None:
            sel = topk_idx[t].long()
            if comp is not None:
                cj = sel[sel >= COMP_FLAG] - COMP_FLAG
                kc = ckf[comp_rows(block_table, b, cj, comp[1], page_size)][:, :L]
            pos = sel[(sel >= 0) & (sel < n)].long()
        pages = block_table[b, (pos // page_size).long()].long()
        k = kvf[pages * page_size + pos % page_size][:, :L]
        if kc is not None:
            k = torch.cat([k, kc], 0)
        s = (q[t].float() @ k.T) * softmax_scale                       # [H, n]
        if sink is not None:
            s = torch.cat([s, sink.float().unsqueeze(-1)], -1)
            p = s.softmax(-1)[:, :-1]
        else:
            p = s.softmax(-1)
        out[t] = p @ k
    return out


ENGRAM_SALT = 0x9E3779B97F4A7C15


def _splitmix64(x: int) -> int:
    m = (1 << 64) - 1
    x = (x + ENGRAM_SALT) & m
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & m
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & m
    return x ^ (x >> 31)


def engram_multipliers(heads: int):
    """Odd 64-bit hash multipliers, one per head (shared by the CUDA kernel)."""
    return [_splitmix64(j + 1) | 1 for j in range(heads)]


def engram_hash(ctx: torch.Tensor, heads: int, rows: int, max_ngram: int) -> torch.Tensor:
    """ctx [T, max_ngram] int64: token at position p - i in column i (-1
    where p - i < 0).  Head j hashes an n-gram of order 2 + j % (max_ngram - 1)
    into its own range of rows // heads rows: h = ((h ^ (tok + 1)) * M_j)
    over the n-gram (64-bit wrap), row = j * per + (h >> 32) % per."""
    per = rows // heads
    mults = engram_multipliers(heads)
    T = ctx.shape[0]
    out = torch.empty(T, heads, dtype=torch.int32)
    span = max(1, max_ngram - 1)
    for j in range(heads):
        n = 2 + j % span if max_ngram >= 2 else 1
        h = torch.zeros(T, dtype=torch.int64)
        m = mults[j]
        m_signed = m - (1 << 64) if m >= (1 << 63) else m
        for i in range(n):
            v = (ctx[:, i] + 1).clamp(min=0)
            h = (h ^ v) * m_signed                                      # wrapping int64 == uint64 bits
        hi = (h >> 32) & 0xFFFFFFFF
        out[:, j] = (j * per + hi % per).to(torch.int32)
    return out


def e8m0_to_float(e: torch.Tensor) -> torch.Tensor:
    e = e.to(torch.int32)
    return torch.where(e == 0, torch.full_like(e, 0, dtype=torch.float32) + 2.0 ** -127,
                       torch.pow(2.0, (e - 127).float()))


def engram_gather(table: torch.Tensor, scale: torch.Tensor, ids: torch.Tensor, row_lo: int = 0,
                  row_hi: Optional[int] = None) -> torch.Tensor:
    """table [rows, dim] e4m3 bytes (uint8), scale [rows, dim/32] UE8M0 bytes,
    ids [T, heads] global row ids -> [T, heads, dim] fp32; rows outside
    [row_lo, row_hi) of this shard give zeros."""
    row_hi = row_lo + table.shape[0] if row_hi is None else row_hi
    T, nh = ids.shape
    dim = table.shape[1]
    flat = ids.reshape(-1).long()
    own = (flat >= row_lo) & (flat < row_hi)
    loc = (flat - row_lo).clamp(0, table.shape[0] - 1)
    v = table[loc].view(torch.float8_e4m3fn).float()
    s = e8m0_to_float(scale[loc]).repeat_interleave(32, -1)
    out = (v * s) * own.unsqueeze(-1).float()
    return out.view(T, nh, dim)


def engram_gate(X: torch.Tensor, kv: torch.Tensor, q_w: torch.Tensor, k_w: torch.Tensor, eps: float,
                clamp: float) -> torch.Tensor:
    """X [T, hc, D]; kv [T, 2D] = [k | v].  Each stream c: a = sigmoid(clamp(
    <rmsnorm(X_c) * q_w, rmsnorm(k) * k_w> / sqrt(D))), X_c + a * v."""
    D = X.shape[-1]
    k, v = kv[:, :D].float(), kv[:, D:].float()
    kn = rmsnorm(k, k_w, eps)
    qn = rmsnorm(X.float(), q_w, eps)
    a = torch.sigmoid(((qn * kn.unsqueeze(1)).sum(-1) / (D ** 0.5)).clamp(-clamp, clamp))
    return X.float() + a.unsqueeze(-1) * v.unsqueeze(1)


def inv_rope_tail(o: torch.Tensor, pos: torch.Tensor, table: torch.Tensor, rd: int) -> torch.Tensor:
    """Rotate the last rd dims of o [T, H, L] back by each token's position."""
    cs = table[pos.long()].float()
    neg = torch.cat([cs[:, : rd // 2], -cs[:, rd // 2:]], -1)
    tail = rope(o[..., -rd:], torch.arange(o.shape[0]), neg)
    return torch.cat([o[..., :-rd].float(), tail], -1)


def compress_store(g: torch.Tensor, bias: torch.Tensor, positions: torch.Tensor, out_slots: torch.Tensor,
                   q_seq: torch.Tensor, block_table: torch.Tensor, r: int, kv_cache: torch.Tensor, kv_scale: float,
                   ix_cache: torch.Tensor, ix_scale: torch.Tensor, gate: torch.Tensor, ckv: torch.Tensor,
                   cik: torch.Tensor, cis: torch.Tensor, page_size: int) -> None:
    """Compressor: store each row's gate logit g[t] at its slot; for every row
    that completes a block (position p with (p + 1) % r == 0), write block
    j = p // r's compressed latent row (softmax over the block of gate +
    bias[i mod r] weighting its r cached rows; same scale as the cache) and
    compressed indexer key (own per-row scale amax / 448 for e4m3)."""
    gate[out_slots.long()] = g.float()
    fp8 = kv_cache.dtype == torch.float8_e4m3fn
    for t in range(positions.shape[0]):
        p = int(positions[t])
        if (p + 1) % r:
            continue
        b = int(q_seq[t])
        pos = torch.arange(p + 1 - r, p + 1, device=positions.device)
        slots = block_table[b, (pos // page_size).long()].long() * page_size + pos % page_size
        w = torch.softmax(gate[slots].float() + bias.float(), 0).unsqueeze(-1)
        kv = (w * (kv_cache[slots].float() * kv_scale)).sum(0)
        ik = (w * (ix_cache[slots].float() * ix_scale[slots].float().unsqueeze(-1))).sum(0)
        row = int(comp_rows(block_table, b, torch.tensor([p // r], device=positions.device), r, page_size)[0])
        ckv[row] = (kv / kv_scale).to(ckv.dtype)
        if fp8:
            s = ik.abs().amax().clamp(min=1e-12) / 448.0
            cik[row] = (ik / s).to(cik.dtype)
            cis[row] = s
        else:
            cik[row] = ik.to(cik.dtype)
            cis[row] = 1.0


def indexer_select_compressed(q: torch.Tensor, w: torch.Tensor, cik: torch.Tensor, cis: torch.Tensor,
                              block_table: torch.Tensor, q_seq: torch.Tensor, q_pos: torch.Tensor, page_size: int,
                              r: int, topk: int, swa: int) -> torch.Tensor:
    """Selection of a compressed-attention layer: per query at position p,
    its window positions p - swa + 1 .. p (-1 before position 0) followed by
    the top-`topk` compressed blocks j < (p + 1 - swa) // r by indexer score
    sum_h w[t,h] relu(q[t,h] . key_j) (entries COMP_FLAG + j, -1 padded).
    Returns int32 [T, swa + topk]."""
    T = q.shape[0]
    out = torch.full((T, swa + topk), -1, dtype=torch.int32, device=q.device)
    for t in range(T):
        b = int(q_seq[t])
        p = int(q_pos[t])
        win = torch.arange(p - swa + 1, p + 1, device=q.device)
        out[t, :swa] = torch.where(win >= 0, win, torch.full_like(win, -1)).to(torch.int32)
        nc = max(0, (p + 1 - swa) // r)
        if nc == 0:
            continue
        j = torch.arange(nc, device=q.device)
        rows = comp_rows(block_table, b, j, r, page_size)
        k = cik[rows].float() * cis[rows].float().unsqueeze(-1)
        sc = ((q[t].float() @ k.T).relu() * w[t].float().unsqueeze(-1)).sum(0)
        kk = min(topk, nc)
        idx = sc.topk(kk).indices.sort().values
        out[t, swa: swa + kk] = (idx + COMP_FLAG).to(torch.int32)
    return out
