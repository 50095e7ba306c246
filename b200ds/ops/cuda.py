"""CUDA implementations of the op surface: thin wrappers over b200ds._C.

Importing this module on a machine with a GPU but without the built
extension raises: there is no silent fallback.
"""
from __future__ import annotations

import os
import weakref
from typing import List, Optional

import torch
import torch.distributed as dist

from ..utils import levers
from . import tactics
from .quant import MXFP8Tensor, round_up

try:
    from .. import _C  # noqa: F401
except ImportError as e:  # pragma: no cover - only on a box without the build
    raise ImportError("b200ds native extension is not built: run `python setup.py build_ext --inplace` "
                      "(or __graft_entry__.build())") from e

from .. import _C

levers.register("srcpin", "B200_SRCPIN", True,
                "refuse a native library built from other csrc/ sources than the tree's (source-hash pin)")
if levers.on("srcpin"):
    from ..utils.srcpin import check_pin
    _stale = check_pin()
    if _stale is not None:
        raise ImportError(f"b200ds native extension: {_stale}")


def _qact():
    from . import QAct
    return QAct


def sf_bytes(rows: int, k: int) -> int:
    return round_up(rows, 128) * (k // 32)


def alloc_qact(rows: int, k: int, device) -> "QAct":
    QAct = _qact()
    q = torch.empty(rows, k, dtype=torch.float8_e4m3fn, device=device)
    sf = torch.empty(sf_bytes(rows, k), dtype=torch.uint8, device=device)
    return QAct(q, sf, None)


# ---------------------------------------------------------------------------
def quant(x: torch.Tensor):
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    if x2.dtype not in (torch.bfloat16, torch.float32):
        x2 = x2.to(torch.bfloat16)
    a = alloc_qact(x2.shape[0], x2.shape[1], x2.device)
    _C.quant(x2, a.q, a.sf)
    return a


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    xx = x if x.dtype in (torch.bfloat16, torch.float32) else x.to(torch.bfloat16)
    _C.rmsnorm(xx, None, w, eps, y, None, None)
    return y


def rmsnorm_quant(x: torch.Tensor, w: torch.Tensor, eps: float, keep_hf: bool = True):
    a = alloc_qact(x.shape[0], x.shape[1], x.device)
    y = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device) if keep_hf else None
    _C.rmsnorm(x, None, w, eps, y, a.q, a.sf)
    a.hf = y
    return a


def add_rmsnorm_act(a: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float, next_linear=None):
    """residual (fp32, in place) += a; returns (normalized act, residual)."""
    if residual.dtype != torch.float32:
        residual = residual.float()
    a2 = a if a.dtype == torch.bfloat16 else a.to(torch.bfloat16)
    rows, K = residual.shape
    quantized = next_linear is not None and getattr(next_linear, "quantized", False)
    y = torch.empty(rows, K, dtype=torch.bfloat16, device=a.device)
    if quantized:
        q = alloc_qact(rows, K, a.device)
        _C.rmsnorm(a2, residual, w, eps, y, q.q, q.sf)
        q.hf = y
        return q, residual
    _C.rmsnorm(a2, residual, w, eps, y, None, None)
    return y, residual


def allreduce_add_rmsnorm(a, residual, w, eps, ps, next_linear=None):
    """TP all-reduce + residual add + RMSNorm (+ MXFP8 quant): one fused
    NVLink kernel pair when the symmetric workspace is set up and the step
    fits it, else NCCL followed by the fused add+norm kernel."""
    from . import EPPartial, MoEPartial, PendingLinear, materialize
    far = getattr(ps, "fused_ar", None)
    T = residual.shape[0]
    if isinstance(a, EPPartial):
        quantized = next_linear is not None and getattr(next_linear, "quantized", False)
        if residual.dtype != torch.float32:
            residual = residual.float()
        if a.pushed:
            return far.ep_comb_add_rmsnorm(a, residual, w, eps, quantized)
        return far.ep_rs_add_rmsnorm(a, residual, w, eps, quantized)
    if far is not None and far.supports(T):
        quantized = next_linear is not None and getattr(next_linear, "quantized", False)
        if residual.dtype != torch.float32:
            residual = residual.float()
        if isinstance(a, PendingLinear) and isinstance(a.w, MXFP8Tensor) and a.n_out == a.w.data.shape[0]:
            return far.gemm_allreduce_add_rmsnorm(a.x, a.w, residual, w, eps, quantized)
        if isinstance(a, MoEPartial):
            return far.moe_allreduce_add_rmsnorm(a, residual, w, eps, quantized)
        return far.allreduce_add_rmsnorm(materialize(a), residual, w, eps, quantized)
    from . import comm
    a = comm.all_reduce(materialize(a), ps)
    return add_rmsnorm_act(a, residual, w, eps, next_linear)


# ---------------------------------------------------------------------------
def _gemm_raw(a, w: MXFP8Tensor, out: torch.Tensor, epi: int, splits: int = 1, pdl: bool = False):
    T, K = a.q.shape
    N = w.data.shape[0]
    _C.gemm(w.data, w.sf, 0, a.q, a.sf, N, T, K, epi, splits, out, out.stride(0), None, None, 0, 0, 0,
            None, None, 0, None, None, pdl)


def choose_splits(T: int, N: int, K: int, max_ctas: int = 2 * 148) -> int:
    """Cluster split-K factor (1, 2, 4 or 8) so small-token GEMMs cover the
    148 SMs: the largest factor whose CTAs all stay resident at once (the
    split-K kernels fit two CTAs per SM); every split keeps at least two
    k-tiles.  (o_proj at N = 7168: 4 splits, 224 CTAs; at 2 splits only 112
    SMs streamed weights, 0.47 of copy bandwidth under ncu.)  max_ctas caps
    the grid (the push epilogue's GEMM keeps its 1.5-wave cap)."""
    s = 1
    if T <= 128:
        tiles = N // 128
        ktiles = K // 128
        while s < 8 and tiles * s * 2 <= max_ctas and ktiles // (s * 2) >= 2:
            s *= 2
    return tactics.pick("gemm_splits", s, N=N, K=K, rows=T, max_ctas=max_ctas)


def gemm(a, w: MXFP8Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
    T, K = a.q.shape
    N = w.data.shape[0]
    assert w.data.shape[1] == K, (w.data.shape, a.q.shape)
    if out_dtype == torch.float32:
        out = torch.zeros(T, N, dtype=torch.float32, device=a.q.device)
        _gemm_raw(a, w, out, 1, choose_splits(T, N, K))
        return out
    out = torch.empty(T, N, dtype=torch.bfloat16, device=a.q.device)
    splits = choose_splits(T, N, K)
    _gemm_raw(a, w, out, 4 if splits > 1 else 0, splits, pdl=True)
    return out


def swiglu_splits(T: int, I: int, K: int) -> int:
    """Cluster split-K for thin gate_up GEMMs (few 128-channel tiles)."""
    if T > 128:
        return 1
    tiles = I // 128
    ktiles = K // 128
    for s in (8, 4, 2):
        if tiles * s <= 148 and ktiles // s >= 4:
            return s
    return 1


def gemm_swiglu_quant(a, w: MXFP8Tensor, splits: Optional[int] = None):
    """MXFP8 act [T, K] x gate_up [2I, K] -> MXFP8(silu(g) * u) [T, I]."""
    T, K = a.q.shape
    I = w.data.shape[0] // 2
    o = alloc_qact(T, I, a.q.device)
    s = swiglu_splits(T, I, K) if splits is None else splits
    _C.gemm(w.data, w.sf, 0, a.q, a.sf, 2 * I, T, K, 6 if s > 1 else 2, s, None, 0, o.q, o.sf, I, I, 0, None, None,
            0, None, None, s > 1)
    return o


# ---------------------------------------------------------------------------
def rope(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """In-place rotation of x [T, H, d] (any row strides, unit inner stride)."""
    if x.dim() == 2:
        x3 = x.unsqueeze(1)
    else:
        x3 = x
    _C.rope(x3, pos, table)
    return x


def kv_store(kv_a, ln_w, eps, table, pos, cache, slots, kv_scale, kv_lora):
    _C.kv_store(kv_a, ln_w, eps, pos, table, slots, cache.view(torch.uint8), kv_scale, kv_lora)


MLA_SPLITS = int(os.environ.get("B200_MLA_SPLITS", "0"))     # diagnostics: fixed KV splits
MLA_HB = int(os.environ.get("B200_MLA_HB", "0"))             # diagnostics: fixed heads per CTA


def mla_hb(H: int) -> int:
    if MLA_HB and H % MLA_HB == 0:
        return MLA_HB
    return 64 if H % 64 == 0 else (32 if H % 32 == 0 else 16)


def mla_splits(T: int, H: int, max_len: int) -> int:
    """KV splits so that decode grids cover the SMs (at least ~2 tiles each)."""
    if MLA_SPLITS:
        return MLA_SPLITS
    # Split only up to one wave of CTAs: the split partials and their merge
    # cost more than a longer per-CTA tile loop (measured: 64 x 1K, 128 heads
    # 91 us unsplit vs 163 us in 3 splits; 16 heads best at 2 splits).
    groups = H // mla_hb(H)
    ctas = T * max(1, groups)
    tiles = max(1, -(-max_len // 128))
    s = max(1, min(16, 148 // max(ctas, 1), tiles // 2))
    return tactics.pick("mla_splits", s, H=H, rows=T, keys=max_len)


def quant_heads(y: torch.Tensor):
    """[H, T, v] bf16 (head-major batched-GEMM output) -> MXFP8 QAct [T, H*v]."""
    H, T, v = y.shape
    a = alloc_qact(T, H * v, y.device)
    _C.quant_heads(y.contiguous(), a.q, a.sf)
    return a


def absorb_q_prep(q_nope, q_pe, w_uk_t, pos, table):
    """tcgen05 absorption of the query into the latent space fused with RoPE
    and e4m3 quantization: q_nope / q_pe strided [T, H, 128 / 64] bf16 views,
    w_uk_t [H, 512, 128] -> (q8 [T, H, 576] e4m3, qs [T, H])."""
    T, H, _ = q_nope.shape
    q8 = torch.empty(T, H, 576, dtype=torch.uint8, device=q_nope.device)
    qs = torch.empty(T, H, dtype=torch.float32, device=q_nope.device)
    _C.bf16_absorb(w_uk_t, q_nope, 1, None, q_pe, pos, table, q8, qs, None, None)
    return q8, qs


def absorb_o_mx(o_lat, w_uv):
    """tcgen05 value absorption [T, H, 512] x [H, 128, 512] fused with the
    MXFP8 quantization of the output projection's operand [T, H * 128]."""
    T, H, _ = o_lat.shape
    a = alloc_qact(T, H * w_uv.shape[1], o_lat.device)
    _C.bf16_absorb(w_uv, o_lat, 2, None, None, None, None, None, None, a.q, a.sf)
    return a


def mla_decode_from_q(q_nope, q_pe, w_uk_t, cache, kv_scale, fb, softmax_scale, page_size, topk, rope_table):
    """Absorbed MLA from the un-absorbed query: absorption + RoPE + quant in one
    tcgen05 kernel, then the attention kernel (+ split merge)."""
    q8, qs = absorb_q_prep(q_nope, q_pe, w_uk_t, fb.positions, rope_table)
    return _mla_core(q8, qs, cache, kv_scale, fb, softmax_scale, page_size, topk)


def mla_attention(q_abs, q_pe, cache, kv_scale, fb, softmax_scale, page_size, topk=None, impl=None,
                  rope_table=None):
    T, H, L = q_abs.shape
    dev = q_abs.device
    use_tc = (impl or "tc") == "tc" and page_size == 64 and L == 512 and H % 16 == 0 \
        and q_pe.shape[-1] == 64
    if not use_tc:
        out = torch.empty(T, H, L, dtype=torch.bfloat16, device=dev)
        qp = q_pe.to(torch.bfloat16).contiguous()
        if rope_table is not None:
            rope(qp, fb.positions, rope_table)
        _C.mla_simt(q_abs.to(torch.bfloat16).contiguous(), qp, cache.view(torch.uint8), kv_scale, fb.block_table,
                    fb.q_seq, fb.positions, topk, page_size, softmax_scale, out)
        return out
    q8 = torch.empty(T, H, 576, dtype=torch.uint8, device=dev)
    qs = torch.empty(T, H, dtype=torch.float32, device=dev)
    if rope_table is not None and q_abs.dtype == torch.bfloat16 and q_pe.dtype == torch.bfloat16 \
            and q_abs.stride(-1) == 1 and q_pe.stride(-1) == 1:
        # RoPE + e4m3 straight from the strided projections (no copies)
        _C.mla_q_prep(q_abs, q_pe, fb.positions, rope_table, q8, qs)
    else:
        qa = q_abs.to(torch.bfloat16).contiguous()
        qp = q_pe.to(torch.bfloat16).contiguous()
        if rope_table is not None:
            rope(qp, fb.positions, rope_table)
        _C.mla_q_quant(qa, qp, q8, qs)
    return _mla_core(q8, qs, cache, kv_scale, fb, softmax_scale, page_size, topk)


def _mla_core(q8, qs, cache, kv_scale, fb, softmax_scale, page_size, topk, lse_out=None, comp=None):
    T, H, _ = q8.shape
    L = 512
    dev = q8.device
    out = torch.empty(T, H, L, dtype=torch.bfloat16, device=dev)
    keys = int(fb.max_seq_len) if fb.max_seq_len else 4096
    if topk is not None:
        keys = min(keys, int(topk.shape[1]))
        topk = topk.to(torch.int32).contiguous()
    nsplit = mla_splits(T, H, keys) if (fb.is_decode or topk is not None) else 1
    po = pl = None
    if nsplit > 1:
        po = torch.empty(nsplit, T, H, L, dtype=torch.float32, device=dev)
        pl = torch.empty(nsplit, T, H, dtype=torch.float32, device=dev)
    if comp is not None:
        # compressed blocks (entries >= COMP_FLAG) are gathered from the
        # compressed rows; the selection keeps them in aligned groups of four
        _C.mla_tc(q8, qs, cache.view(torch.uint8), kv_scale, fb.block_table, fb.q_seq, fb.positions, page_size,
                  softmax_scale, nsplit, out, po, pl, topk, mla_hb(H), lse_out=lse_out,
                  cache2=comp[0].view(torch.uint8), ratio2=int(comp[1]))
        return out
    _C.mla_tc(q8, qs, cache.view(torch.uint8), kv_scale, fb.block_table, fb.q_seq, fb.positions, page_size,
              softmax_scale, nsplit, out, po, pl, topk, mla_hb(H), lse_out=lse_out)
    return out


# ---------------------------------------------------------------------------
def _gate_bf16(gate: torch.Tensor) -> torch.Tensor:
    """bf16 copy of a router gate, kept on the gate tensor itself (it lives
    and dies with the weights; an in-place weight update bumps the tensor's
    version and refreshes it)."""
    hit = getattr(gate, "_b200_bf16", None)
    if hit is None or hit[1].shape != gate.shape:
        hit = [gate._version, gate.to(torch.bfloat16).contiguous()]
        gate._b200_bf16 = hit
    elif hit[0] != gate._version:
        hit[1].copy_(gate)            # same buffer: captured decode graphs read the new values
        hit[0] = gate._version
    return hit[1]


def router(x: torch.Tensor, gate: torch.Tensor, bias: torch.Tensor, cfg):
    """Router logits on the tensor cores (bf16 inputs, fp32 accumulate and
    output), then the fused sigmoid / group-limited top-k kernel."""
    g16 = _gate_bf16(gate)
    xb = x.to(torch.bfloat16)
    T = xb.shape[0]
    E, Kd = g16.shape
    if E % 128 == 0 and Kd % 64 == 0 and xb.stride(-1) == 1:
        # tcgen05 split-K GEMM (fp32 accumulate across splits)
        logits = torch.zeros(T, E, dtype=torch.float32, device=x.device)
        splits = max(1, min(32, (Kd // 64) // 4, 148 // max(1, (E // 128) * -(-T // 128))))
        if levers.on("deterministic"):
            splits = 1             # fp32 atomics from several splits sum in any order
        _C.bf16_absorb(g16.view(1, E, Kd), xb.view(T, 1, Kd), 3, logits.view(T, 1, E), None, None, None, None,
                       None, None, None, splits=splits)
    else:
        logits = torch.mm(xb, g16.t(), out_dtype=torch.float32)
    K = cfg.num_experts_per_tok
    w = torch.empty(T, K, dtype=torch.float32, device=x.device)
    ids = torch.empty(T, K, dtype=torch.int32, device=x.device)
    _C.router(logits.contiguous(), bias.float(), cfg.n_group, cfg.topk_group, K, cfg.routed_scaling_factor,
              cfg.norm_topk_prob, w, ids, scoring=1 if cfg.scoring_func == "sqrtsoftplus" else 0)
    return w, ids


def moe_tile_n(rows_per_expert: float, cap: int) -> int:
    """Token tile of the grouped GEMMs from the expected rows per expert."""
    bn = cap
    for b in (16, 32, 64, 128):
        if rows_per_expert * 1.5 <= b or b == cap:
            bn = b
            break
    return tactics.pick("moe_tile", bn, cap=cap, rows_per_expert=rows_per_expert)


def moe_tiles(rows_per_expert: float):
    """(FC1, FC2) token tiles of the grouped GEMMs.  Decode-sized experts
    take the smallest tile that holds their rows (weight streaming); from 128
    rows per expert FC1 runs 128-token tiles (gate + up into one TMEM
    accumulator).  FC2 stays at 128 tokens: N = 256 block-scaled MMAs need
    the B scale factors of tokens 128-255 in a TMEM layout this kernel does
    not stage (the 256-token tile produced wrong sums)."""
    bn1 = 128 if rows_per_expert >= 128 else moe_tile_n(rows_per_expert, 64)
    bn2 = moe_tile_n(rows_per_expert, 128)
    return (tactics.pick("moe_tile_fc1", bn1, rows_per_expert=rows_per_expert),
            tactics.pick("moe_tile_fc2", bn2, rows_per_expert=rows_per_expert))


def _fused(bn1: int, bn2: int) -> bool:
    return levers.on("moe_fused") and bn1 == bn2 and bn1 <= 64


def _pulls(bn1: int, bn2: int) -> bool:
    """The fused kernel reads FC1 rows straight from the activations /
    dispatch buffer (switch moe_pull; off keeps the separate gather)."""
    return levers.on("moe_pull") and _fused(bn1, bn2)


def _moe_ws(ex, dev) -> torch.Tensor:
    """Work counters of the fused expert kernel ([2 + E] int32, zero; the
    kernel leaves them zero)."""
    ws = getattr(ex, "_fused_ws", None)
    if ws is None or ws.device != dev:
        ws = torch.zeros(2 + ex.count, dtype=torch.int32, device=dev)
        ex._fused_ws = ws
        ex._fused_err = torch.zeros(1, dtype=torch.int32, device=dev)
        _ERR_WORDS.append(weakref.ref(ex._fused_err))
    return ws


# device error words of kernels with in-kernel waits (weak: a word lives as
# long as its expert set)
_ERR_WORDS: List[weakref.ref] = []


def check_device_errors() -> None:
    """Raise if a bounded in-kernel wait (dependency between CTAs) ran out.
    One device read for all live error words (one per expert set)."""
    words = [w() for w in _ERR_WORDS]
    words = [w for w in words if w is not None]
    if len(words) != len(_ERR_WORDS):
        _ERR_WORDS[:] = [weakref.ref(w) for w in words]
    if not words:
        return
    v = int(torch.cat(words).max().item()) if len(words) > 1 else int(words[0].item())
    if v:
        raise RuntimeError(f"fused expert GEMM: in-kernel dependency wait timed out (code {v})")


def _expert_gemms(ex, xq, xsf, xg, hq, hsf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight, fp4,
                  pull=None):
    """FC1 (SwiGLU + requant into hq) and FC2 (routing-weighted into y): one
    fused persistent launch when both use the same token tile (decode), else
    two grouped launches.  pull (fused only): dict of the FC1 row sources
    (row_token, src_q / src_sf / src_g addresses, src_rows, optional
    src_epoch / src_epoch_add / src_par_bytes) read in place of xq."""
    E, I = ex.count, ex.inter
    w13, w2 = ex.w13, ex.w2
    g2 = float(ex.fc2_act_scale)
    if _fused(bn1, bn2):
        ws = _moe_ws(ex, y.device)
        if pull is not None:
            xq, xsf, xg = hq, hsf, None      # unused operands (rows come from the sources)
        _C.moe_fused(w13.data, w13.sf, w2.data, w2.sf, xq, xsf, hq, hsf, y, E, Hd, I, bn1, seg_start, seg_count, tt1,
                     row_weight, ws, ex._fused_err, 0, True, ex.tiled,
                     xg if fp4 else None, w13.global_scale if fp4 else None, w2.global_scale if fp4 else None, g2,
                     **(pull or {}))
        return
    assert pull is None, "pulled rows need the fused expert kernel"
    if fp4:
        _C.gemm_grouped(w13.data, w13.sf, xq, xsf, 2 * I, Hd, E, I, bn1, seg_start, seg_count, tt1, 2,
                        None, 0, hq, hsf, I, None, 0, True, w_g=w13.global_scale, x_g=xg, out_g=g2, a_tiled=ex.tiled)
        _C.gemm_grouped(w2.data, w2.sf, hq, hsf, Hd, I, E, 0, bn2, seg_start, seg_count, tt2, 3,
                        y, Hd, None, None, 0, row_weight, 0, True, w_g=w2.global_scale, x_g_const=g2, a_tiled=ex.tiled)
        return
    _C.gemm_grouped(w13.data, w13.sf, xq, xsf, 2 * I, Hd, E, I, bn1, seg_start, seg_count, tt1, 2,
                    None, 0, hq, hsf, I, None, 0, True, a_tiled=ex.tiled)
    _C.gemm_grouped(w2.data, w2.sf, hq, hsf, Hd, I, E, 0, bn2, seg_start, seg_count, tt2, 3,
                    y, Hd, None, None, 0, row_weight, 0, True, a_tiled=ex.tiled)



def moe_experts(h, w: torch.Tensor, ids: torch.Tensor, ex, out_dtype=torch.bfloat16, n_experts_total=None,
                combine: bool = True):
    """Local-expert MoE: routing layout -> row gather -> persistent FC1
    (SwiGLU + MXFP8 requant) -> persistent FC2 (routing-weighted) -> combine.
    No host synchronisation: buffers are sized for the worst case."""
    from . import QAct
    a = h if isinstance(h, QAct) else quant(h)
    T, Hd = a.q.shape
    K = ids.shape[1]
    E = ex.count
    dev = a.q.device
    I = ex.inter
    e_tot = n_experts_total or E
    exp_rows = T * K / e_tot
    bn1, bn2 = moe_tiles(exp_rows)
    max_rows = round_up(T * K, 128) + E * 128   # 128-aligned segments
    seg_start = torch.empty(E, dtype=torch.int32, device=dev)
    seg_count = torch.empty(E, dtype=torch.int32, device=dev)
    tt1 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    tt2 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    row_token = torch.empty(max_rows, dtype=torch.int32, device=dev)
    row_weight = torch.empty(max_rows, dtype=torch.float32, device=dev)
    pair_row = torch.empty(T, K, dtype=torch.int32, device=dev)
    total = torch.empty(1, dtype=torch.int32, device=dev)
    ids = ids if ids.dtype == torch.int32 else ids.int()
    _C.moe_align(ids.contiguous(), w.float().contiguous(), ex.first, E, seg_start, seg_count, row_token, row_weight,
                 pair_row, total, bn1, tt1, bn2, tt2)
    hq = alloc_qact(max_rows, I, dev)
    y = torch.empty(max_rows, Hd, dtype=torch.bfloat16, device=dev)
    if _pulls(bn1, bn2):
        pull = dict(row_token=row_token, src_q=[a.q.data_ptr()], src_sf=[a.sf.data_ptr()], src_rows=max(T, 1))
        _expert_gemms(ex, None, None, None, hq.q, hq.sf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight,
                      False, pull)
    else:
        xs = alloc_qact(max_rows, Hd, dev)
        _C.moe_gather(a.q, a.sf, pair_row, xs.q, xs.sf)
        _expert_gemms(ex, xs.q, xs.sf, None, hq.q, hq.sf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight,
                      False)
    if not combine:
        from . import MoEPartial
        return MoEPartial(y, pair_row, None)
    out = torch.empty(T, Hd, dtype=out_dtype, device=dev)
    _C.moe_combine(y, pair_row, None, out)
    return out


def nvfp4_quant(x: torch.Tensor):
    """bf16/fp32 rows -> (packed e2m1 [T, K/2], e4m3 scales (chunk layout),
    per-row fp32 global scale [T])."""
    T, K = x.shape
    dev = x.device
    q = torch.empty(T, K // 2, dtype=torch.uint8, device=dev)
    sf = torch.empty(round_up(max(T, 1), 128) * (K // 16), dtype=torch.uint8, device=dev)
    g = torch.empty(T, dtype=torch.float32, device=dev)
    _C.nvfp4_quant(x if x.stride(-1) == 1 else x.contiguous(), q, sf, g)
    return q, sf, g


def moe_experts_nvfp4(h, w, ids, ex, out_dtype=torch.bfloat16, n_experts_total=None, combine: bool = True):
    """NVFP4 routed experts: per-token NVFP4 quantization of the MoE input ->
    routing layout -> row gather -> persistent FC1 (kind::mxf4nvf4, SwiGLU,
    NVFP4 requant) -> FC2 (routing-weighted) -> combine."""
    from . import QAct
    x = h.hf if isinstance(h, QAct) and h.hf is not None else (h if not isinstance(h, QAct) else None)
    if x is None:
        from .quant import dequant_mxfp8
        x = dequant_mxfp8(h.q, h.sf).to(torch.bfloat16)
    T, Hd = x.shape
    K = ids.shape[1]
    E = ex.count
    dev = x.device
    I = ex.inter
    e_tot = n_experts_total or E
    exp_rows = T * K / e_tot
    bn1, bn2 = moe_tiles(exp_rows)
    max_rows = round_up(T * K, 128) + E * 128
    xq, xsf, xg = nvfp4_quant(x)
    seg_start = torch.empty(E, dtype=torch.int32, device=dev)
    seg_count = torch.empty(E, dtype=torch.int32, device=dev)
    tt1 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    tt2 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    row_token = torch.empty(max_rows, dtype=torch.int32, device=dev)
    row_weight = torch.empty(max_rows, dtype=torch.float32, device=dev)
    pair_row = torch.empty(T, K, dtype=torch.int32, device=dev)
    total = torch.empty(1, dtype=torch.int32, device=dev)
    ids = ids if ids.dtype == torch.int32 else ids.int()
    _C.moe_align(ids.contiguous(), w.float().contiguous(), ex.first, E, seg_start, seg_count, row_token, row_weight,
                 pair_row, total, bn1, tt1, bn2, tt2)
    hq = torch.empty(max_rows, I // 2, dtype=torch.uint8, device=dev)
    hsf = torch.empty(max_rows * (I // 16), dtype=torch.uint8, device=dev)
    y = torch.empty(max_rows, Hd, dtype=torch.bfloat16, device=dev)
    if _pulls(bn1, bn2):
        pull = dict(row_token=row_token, src_q=[xq.data_ptr()], src_sf=[xsf.data_ptr()], src_g=[xg.data_ptr()],
                    src_rows=max(T, 1))
        _expert_gemms(ex, None, None, None, hq, hsf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight, True,
                      pull)
    else:
        xs_q = torch.empty(max_rows, Hd // 2, dtype=torch.uint8, device=dev)
        xs_sf = torch.empty(max_rows * (Hd // 16), dtype=torch.uint8, device=dev)
        xs_g = torch.empty(max_rows, dtype=torch.float32, device=dev)
        _C.moe_gather4(xq, xsf, xg, pair_row, xs_q, xs_sf, xs_g)
        _expert_gemms(ex, xs_q, xs_sf, xs_g, hq, hsf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight,
                      True)
    if not combine:
        from . import MoEPartial
        return MoEPartial(y, pair_row, None)
    out = torch.empty(T, Hd, dtype=out_dtype, device=dev)
    _C.moe_combine(y, pair_row, None, out)
    return out


def moe_experts_ep(h, w, ids, ex, T_step: int, n_experts_total: int, ep, far=None):
    """Expert-parallel MoE: ep_dispatch (P2P push of routed rows) -> ep_align
    (bounded wait + routing layout over all ranks' tokens) -> persistent
    FC1 (SwiGLU + requant; its producer reads the received rows in place) ->
    FC2 (routing-weighted); the combine + reduce-scatter runs fused in the
    following norm step.  Unfused (prefill tiles): ep_gather copies the rows
    into an expert-sorted operand first."""
    from . import EPPartial, QAct
    from .quant import NVFP4Tensor
    fp4 = isinstance(ex.w13, NVFP4Tensor)
    if fp4:
        x = h.hf if isinstance(h, QAct) and h.hf is not None else h
        q, sf, g = nvfp4_quant(x)
        T_r, Hd = x.shape
    else:
        a = h if isinstance(h, QAct) else quant(h)
        q, sf, g = a.q, a.sf, None
        T_r, Hd = a.q.shape
    K = ids.shape[1]
    E = ex.count
    dev = q.device
    I = ex.inter
    Tg = ep.world * T_step
    exp_rows = Tg * K / n_experts_total
    bn1, bn2 = moe_tiles(exp_rows)
    max_rows = round_up(Tg * K, 128) + E * 128
    ids = (ids if ids.dtype == torch.int32 else ids.int()).contiguous()
    # peer pull (fused expert kernel only): the rows stay in their source
    # rank's region and the producer warps of the owners read them over NVLink
    peer = _pulls(bn1, bn2) and levers.on("ep_peer_pull") and ep.world <= 8
    _C.ep_dispatch(q, sf, g, Hd, ids, w.float().contiguous(), T_step, n_experts_total // ep.world, ep.bases,
                   ep.rank, ep.max_t, ep.epoch, ep.push_ticket, peer_pull=peer)
    seg_start = torch.empty(E, dtype=torch.int32, device=dev)
    seg_count = torch.empty(E, dtype=torch.int32, device=dev)
    tt1 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    tt2 = torch.empty(E + 1, dtype=torch.int32, device=dev)
    row_token = torch.empty(max_rows, dtype=torch.int32, device=dev)
    row_weight = torch.empty(max_rows, dtype=torch.float32, device=dev)
    pair_row = torch.empty(Tg, K, dtype=torch.int32, device=dev)
    total = torch.empty(1, dtype=torch.int32, device=dev)
    pulls = _pulls(bn1, bn2)
    # the combine fused into the FC2 epilogue (pair rows stored straight into
    # the owners' slots of the expert-parallel all-reduce workspace)
    comb = (pulls and far is not None and getattr(far, "topk", 0) == K and far.supports(T_step)
            and levers.on("ep_combine_epilogue"))
    row_pair = torch.empty(max_rows, dtype=torch.int32, device=dev) if comb else None
    _C.ep_align(ep.bases, ep.rank, ep.max_t, Hd, K, T_step, ex.first, E, seg_start, seg_count, row_token, row_weight,
                pair_row, total, bn1, tt1, bn2, tt2, ep.epoch, ep.err, release=pulls, row_pair=row_pair)
    y = torch.empty(max_rows if not comb else 1, Hd, dtype=torch.bfloat16, device=dev)
    if pulls:
        # received rows read in place (row index = owner rank * T_step + t);
        # ep_align advanced the epoch, so they sit at parity (epoch + 1) & 1
        if peer:
            # row g = source rank * T_step + t sits at row t of the source's region
            pull = dict(row_token=row_token, src_q=ep.src_q, src_sf=ep.src_sf, src_g=ep.src_g if fp4 else [],
                        src_rows=T_step, src_epoch=ep.epoch, src_epoch_add=1, src_par_bytes=ep.par_bytes)
        else:
            pull = dict(row_token=row_token, src_q=[ep.recv_q], src_sf=[ep.recv_sf],
                        src_g=[ep.recv_g] if fp4 else [], src_rows=ep.world * ep.max_t, src_epoch=ep.epoch,
                        src_epoch_add=1, src_par_bytes=ep.par_bytes)
        if comb:
            pull.update(c_row_pair=row_pair, c_K=K, c_T_step=T_step, c_bases=far.bases, c_rank=far.rank,
                        c_max_t=far.max_tokens, c_off=far.comb_off, c_epoch=far.epoch)
        if fp4:
            hq = torch.empty(max_rows, I // 2, dtype=torch.uint8, device=dev)
            hsf = torch.empty(max_rows * (I // 16), dtype=torch.uint8, device=dev)
        else:
            h_ = alloc_qact(max_rows, I, dev)
            hq, hsf = h_.q, h_.sf
        _expert_gemms(ex, None, None, None, hq, hsf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight, fp4,
                      pull)
        if comb:
            return EPPartial(None, pair_row, T_step, T_r, pushed=True, ids=ids[:T_r].contiguous())
        return EPPartial(y, pair_row, T_step, T_r)
    if fp4:
        xs_q = torch.empty(max_rows, Hd // 2, dtype=torch.uint8, device=dev)
        xs_sf = torch.empty(max_rows * (Hd // 16), dtype=torch.uint8, device=dev)
        xs_g = torch.empty(max_rows, dtype=torch.float32, device=dev)
        _C.ep_gather(ep.bases, ep.rank, ep.max_t, Hd, K, T_step, pair_row, xs_q, xs_sf, xs_g, ep.epoch,
                     ep.gather_ticket)
        hq = torch.empty(max_rows, I // 2, dtype=torch.uint8, device=dev)
        hsf = torch.empty(max_rows * (I // 16), dtype=torch.uint8, device=dev)
        _expert_gemms(ex, xs_q, xs_sf, xs_g, hq, hsf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight,
                      True)
        return EPPartial(y, pair_row, T_step, T_r)
    xs = alloc_qact(max_rows, Hd, dev)
    _C.ep_gather(ep.bases, ep.rank, ep.max_t, Hd, K, T_step, pair_row, xs.q, xs.sf, None, ep.epoch,
                 ep.gather_ticket)
    hq = alloc_qact(max_rows, I, dev)
    _expert_gemms(ex, xs.q, xs.sf, None, hq.q, hq.sf, y, Hd, bn1, bn2, seg_start, seg_count, tt1, tt2, row_weight,
                  False)
    return EPPartial(y, pair_row, T_step, T_r)


# ---------------------------------------------------------------------------
def index_k_store(k, ln_w, ln_b, eps, table, pos, cache, scale, slots):
    _C.ix_k_store(k, ln_w, ln_b, eps, pos, table, slots, cache.view(torch.uint8), scale)


def ix_splits(T: int, max_len: int) -> int:
    """Key splits of the indexer score grid: cover ~2 waves of SMs, at least
    two 128-key tiles per CTA."""
    tiles = max(1, -(-max_len // 128))
    return max(1, min(64, -(-296 // max(T, 1)), max(1, tiles // 2)))


_IX_SCORE_BYTES = 512 << 20      # cap on the fp32 score scratch per call


def indexer_topk(q_raw, w_raw, w_factor, table, k_cache, k_scale, fb, page_size, topk, swa=0):
    """Indexer: RoPE + e4m3 queries, tcgen05 scores, radix top-k.  Queries are
    processed in slices so the [T, capacity] fp32 score scratch stays bounded."""
    T, nh = w_raw.shape
    dev = q_raw.device
    cap = int(fb.block_table.shape[1]) * page_size
    out = torch.empty(T, topk, dtype=torch.int32, device=dev)
    kc = k_cache.view(torch.uint8)
    step = max(1, min(T, _IX_SCORE_BYTES // (cap * 4)))
    max_len = int(fb.max_seq_len) if fb.max_seq_len else cap
    for t0 in range(0, T, step):
        t1 = min(T, t0 + step)
        n = t1 - t0
        q8 = torch.empty(n * nh, 128, dtype=torch.uint8, device=dev)
        wq = torch.empty(n, nh, dtype=torch.float32, device=dev)
        pos = fb.positions[t0:t1]
        _C.ix_q_quant(q_raw[t0:t1], w_raw[t0:t1], nh, w_factor, pos, table, q8, wq)
        scores = torch.empty(n, cap, dtype=torch.float32, device=dev)
        _C.ix_score(q8, wq, kc, k_scale, fb.block_table, fb.q_seq[t0:t1], pos, page_size,
                    ix_splits(n, max_len), scores)
        if swa > 0:
            # the last `swa` positions up to each query always survive the top-k
            j = torch.arange(cap, device=dev).unsqueeze(0)
            p = pos.long().unsqueeze(1)
            scores.masked_fill_((j > p - swa) & (j <= p), float("inf"))
        _C.topk_select(scores, pos, out[t0:t1], max_len)
    return out


def indexer_topk_compressed(q_raw, w_raw, w_factor, table, cik, cis, fb, page_size, r, topk, swa):
    """Selection of a compressed-attention layer [T, swa + topk]: the window
    (built on the device from the positions), then the indexer's top blocks
    among those ending before the window: tcgen05 scores over the compressed
    keys (paged page_size / r rows a page, key j of sequence b at
    table[b, j*r // page] * (page / r) + j mod (page / r)) and the radix
    top-k, tagged COMP_FLAG + block."""
    from .ref import COMP_FLAG
    T, nh = w_raw.shape
    dev = q_raw.device
    if swa % 4 or topk % 4:
        raise ValueError("compressed attention needs window and top-k sizes that are multiples of 4")
    cpg = page_size // r
    cap = int(fb.block_table.shape[1]) * cpg
    pos = fb.positions
    out = torch.empty(T, swa + topk, dtype=torch.int32, device=dev)
    win = pos.view(-1, 1) - (swa - 1) + torch.arange(swa, dtype=torch.int32, device=dev)
    out[:, :swa] = torch.where(win >= 0, win, torch.full_like(win, -1))
    # last whole block before the window (-1: none yet)
    cpos = (torch.div(pos + 1 - swa, r, rounding_mode="floor") - 1).clamp(min=-1).to(torch.int32)
    ck = cik.view(torch.uint8)
    step = max(1, min(T, _IX_SCORE_BYTES // (cap * 4)))
    max_len = max(1, (int(fb.max_seq_len) if fb.max_seq_len else cap * r) // r)
    sel = torch.empty(T, topk, dtype=torch.int32, device=dev)
    for t0 in range(0, T, step):
        t1 = min(T, t0 + step)
        n = t1 - t0
        q8 = torch.empty(n * nh, 128, dtype=torch.uint8, device=dev)
        wq = torch.empty(n, nh, dtype=torch.float32, device=dev)
        _C.ix_q_quant(q_raw[t0:t1], w_raw[t0:t1], nh, w_factor, pos[t0:t1], table, q8, wq)
        scores = torch.empty(n, cap, dtype=torch.float32, device=dev)
        _C.ix_score(q8, wq, ck, cis, fb.block_table, fb.q_seq[t0:t1], cpos[t0:t1], cpg, ix_splits(n, max_len),
                    scores)
        _C.topk_select(scores, cpos[t0:t1], sel[t0:t1], max_len)
    out[:, swa:] = torch.where(sel >= 0, sel + COMP_FLAG, torch.full_like(sel, -1))
    return out


def compress_store(g, bias, fb, r, kv_cache, kv_scale, ix_cache, ix_scale, gate, ckv, cik, cis, page_size):
    _C.compress_store(g, bias, fb.positions, fb.out_slots, fb.q_seq, fb.block_table, page_size, r,
                      kv_cache.view(torch.uint8), kv_scale, ix_cache.view(torch.uint8), ix_scale, gate,
                      ckv.view(torch.uint8), cik.view(torch.uint8), cis)


SAMPLE_CANDIDATES = 64


def sample_tokens(local_logits, vocab_off, temperature, top_p, top_k, uniform, ps):
    """Per-rank top-64 candidates + (max, sum-exp) of the local vocab shard
    (radix select), exchanged through the fused all-reduce slots when TP > 1
    (NCCL all-gather of the small candidate buffer otherwise), then one
    sorting / top-k / top-p / draw kernel per row."""
    B, n = local_logits.shape
    dev = local_logits.device
    Kc = SAMPLE_CANDIDATES
    temperature = temperature.float().contiguous()
    top_p = top_p.float().contiguous()
    top_k = top_k.to(torch.int32).contiguous()
    uniform = uniform.float().contiguous()
    tokens = torch.empty(B, dtype=torch.int64, device=dev)
    world = ps.tp_size
    far = getattr(ps, "fused_ar", None) if world > 1 else None
    logits = local_logits if local_logits.stride(-1) == 1 else local_logits.contiguous()
    if far is not None and far.world == world and B * (Kc + 1) * 8 <= far.max_tokens * far.hidden * 2:
        _C.lm_candidates(logits, Kc, vocab_off, temperature, None, far.bases, far.rank, far.max_tokens, far.hidden,
                         far.epoch, far.push_ticket)
        _C.sample_final(None, B, Kc, world, far.bases, far.rank, far.max_tokens, far.hidden, far.epoch, far.ticket,
                        temperature, top_p, top_k, uniform, tokens, far.err)
        return tokens
    cand = torch.empty(B, Kc + 1, dtype=torch.int64, device=dev)       # uint2 entries
    _C.lm_candidates(logits, Kc, vocab_off, temperature, cand, [], 0, 0, 0, None, None)
    if world > 1:
        parts = [torch.empty_like(cand) for _ in range(world)]
        dist.all_gather(parts, cand, group=ps.tp_group)
        cand = torch.stack(parts)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _C.sample_final(cand, B, Kc, world, [], 0, 0, 0, None, None, temperature, top_p, top_k, uniform, tokens, err)
    return tokens


def sample(logits, temperature, top_p, top_k, uniform):
    """Vectorised temperature / top-k / top-p sampling with given uniforms."""
    greedy = temperature <= 0
    t = torch.where(greedy, torch.ones_like(temperature), temperature)
    p = torch.softmax(logits.float() / t.unsqueeze(-1), -1)
    sp, si = p.sort(-1, descending=True)
    V = p.shape[-1]
    ar = torch.arange(V, device=p.device).unsqueeze(0)
    keep = torch.ones_like(sp, dtype=torch.bool)
    k = top_k.long().unsqueeze(-1)
    keep &= (k <= 0) | (ar < k)
    c = sp.cumsum(-1)
    keep &= (c - sp) < top_p.unsqueeze(-1)
    sp = torch.where(keep, sp, torch.zeros_like(sp))
    c = sp.cumsum(-1)
    u = (uniform * c[:, -1]).unsqueeze(-1)
    j = torch.searchsorted(c, u).clamp(max=V - 1)
    tok = si.gather(1, j).squeeze(-1)
    return torch.where(greedy, logits.argmax(-1), tok)


# ---------------------------------------------------------------------------
# DeepSeek-V4 family
# ---------------------------------------------------------------------------

def hc_fn_parts(fn: torch.Tensor) -> torch.Tensor:
    """fp32 [M, K] -> bf16 [128, K]: rows p*M + j hold the p-th bf16 part of
    fn[j] (hi, mid, lo: fn = hi + mid + lo to ~24 bits), zero rows after."""
    M, K = fn.shape
    assert 3 * M <= 128
    out = torch.zeros(128, K, dtype=torch.bfloat16, device=fn.device)
    rest = fn.float()
    for p in range(3):
        part = rest.to(torch.bfloat16)
        out[p * M:(p + 1) * M] = part
        rest = rest - part.float()
    return out


def hc_embed(embed, ids, hc):
    T, D = ids.shape[0], embed.shape[1]
    X = torch.empty(T, hc, D, dtype=torch.bfloat16, device=embed.device)
    ss = torch.empty(T, dtype=torch.float32, device=embed.device)
    _C.hc_embed(embed, ids.int() if ids.dtype != torch.int32 else ids, X, ss)
    return X, ss


def hc_post(X, y, post, comb):
    ss = torch.empty(X.shape[0], dtype=torch.float32, device=X.device)
    yb = y if y.dtype == torch.bfloat16 else y.to(torch.bfloat16)
    _C.hc_post(X, yb, post, comb, ss)
    return ss


def hc_pre(X, sumsq, hw, norm_w, eps, cfg, next_linear, head, keep_hf):
    T, hc, D = X.shape
    K = hc * D
    parts = hw.fn_parts
    if parts is None:
        parts = hw.fn_parts = hc_fn_parts(hw.fn)
    raw = torch.zeros(T, 128, dtype=torch.float32, device=X.device)
    splits = max(1, min(32, (K // 64) // 4, 148 // max(1, -(-T // 128))))
    if levers.on("deterministic"):
        splits = 1
    _C.bf16_absorb(parts.view(1, 128, K), X.view(T, 1, K), 3, raw.view(T, 1, 128), None, None, None, None, None,
                   None, None, splits=splits)
    quantized = next_linear is not None and getattr(next_linear, "quantized", False)
    post = comb = None
    if not head:
        post = torch.empty(T, hc, dtype=torch.float32, device=X.device)
        comb = torch.empty(T, hc * hc, dtype=torch.float32, device=X.device)
    a = alloc_qact(T, D, X.device) if quantized else None
    hb = torch.empty(T, D, dtype=torch.bfloat16, device=X.device) if (keep_hf or not quantized) else None
    _C.hc_pre(raw, 3, hw.m, sumsq, hw.scale, hw.base, 1 if head else 0, cfg.hc_sinkhorn_iters, cfg.hc_eps, X,
              norm_w, eps, post, comb, a.q if a else None, a.sf if a else None, hb, None)
    if a is not None:
        a.hf = hb
        return a, post, comb
    return hb, post, comb


HC_BOUNDARY_MAX_T = 256      # above: the tcgen05 stats GEMM (fn read once per 128 rows)


def hc_boundary_ok(X) -> bool:
    T, hc, D = X.shape
    return levers.on("hc_boundary") and T <= HC_BOUNDARY_MAX_T and hc == 4 and D % 256 == 0


def hc_boundary(X, carry, hw, norm_w, eps, cfg, next_linear, head, keep_hf):
    """One kernel for the boundary: hc_post of carry = (y, post, comb) (None:
    X is up to date), the mixes in fp32, the coefficients and the normed
    sublayer input, a cluster of CTAs per row."""
    T, hc, D = X.shape
    y = post_in = comb_in = None
    if carry is not None:
        y, post_in, comb_in = carry
        y = y if y.dtype == torch.bfloat16 else y.to(torch.bfloat16)
    quantized = next_linear is not None and getattr(next_linear, "quantized", False)
    post = comb = None
    if not head:
        post = torch.empty(T, hc, dtype=torch.float32, device=X.device)
        comb = torch.empty(T, hc * hc, dtype=torch.float32, device=X.device)
    a = alloc_qact(T, D, X.device) if quantized else None
    hb = torch.empty(T, D, dtype=torch.bfloat16, device=X.device) if (keep_hf or not quantized) else None
    _C.hc_boundary(X, y, post_in, comb_in, hw.fn, hw.scale, hw.base, 1 if head else 0, cfg.hc_sinkhorn_iters,
                   cfg.hc_eps, norm_w, eps, post, comb, a.q if a else None, a.sf if a else None, hb, None)
    if a is not None:
        a.hf = hb
        return a, post, comb
    return hb, post, comb


def hc_mean(X):
    out = torch.empty(X.shape[0], X.shape[2], dtype=torch.bfloat16, device=X.device)
    _C.hc_mean(X, out)
    return out


def kv_store_v4(kv, w, eps, table, pos, cache, slots, kv_scale, rd):
    _C.kv_store_v4(kv, w, eps, pos, table, cache.view(torch.uint8), slots, kv_scale, rd)


def mqa_attention(q, cache, kv_scale, fb, softmax_scale, page_size, sink, table, rd, topk=None, comp=None):
    """Heads per rank below a multiple of 16 (e.g. 64 heads over 8 ranks) are
    padded with zero queries up to the latent-attention kernel's head block;
    the padded heads' outputs are dropped."""
    T, H, L = q.shape
    dev = q.device
    Hp = -(-H // 16) * 16
    q8 = (torch.zeros if Hp != H else torch.empty)(T, Hp, 576, dtype=torch.uint8, device=dev)
    qs = (torch.ones if Hp != H else torch.empty)(T, Hp, dtype=torch.float32, device=dev)
    qb = q if q.dtype == torch.bfloat16 else q.to(torch.bfloat16)
    _C.mqa_q_prep(qb, fb.positions, table, rd, q8, qs)
    lse = torch.empty(T, Hp, dtype=torch.float32, device=dev) if sink is not None else None
    out = _mla_core(q8, qs, cache, kv_scale, fb, softmax_scale, page_size, topk, lse_out=lse, comp=comp)
    if Hp != H and sink is not None:
        sink = torch.cat([sink.float(), sink.new_zeros(Hp - H)])
    _C.attn_fixup(out, lse, sink, rd, fb.positions, table)
    return out if Hp == H else out[:, :H].contiguous()


def e5_prune(w, ids, cfg, n_experts):
    w = w.contiguous()
    ids = ids.contiguous()
    _C.e5_prune(ids, w, n_experts, cfg.prune_budget, cfg.prune_max_count)
    return w, ids


def engram_ids(fb, tok_cache, cfg, mults, page_size):
    out = torch.empty(fb.num_tokens, cfg.engram_heads, dtype=torch.int32, device=fb.input_ids.device)
    _C.engram_hash(fb.input_ids, fb.positions, fb.q_seq, fb.block_table, fb.out_slots, page_size, tok_cache,
                   cfg.engram_heads, cfg.engram_rows, cfg.engram_max_ngram, mults, out)
    return out


def engram_update(X, ids, ew, cfg, ps):
    T = X.shape[0]
    nh = ids.shape[1]
    emb = torch.empty(T, nh * 256, dtype=torch.bfloat16, device=X.device)
    _C.engram_gather(ew.table, ew.scale, ids.contiguous(), ew.row_lo, emb)
    if ps.tp_size > 1:
        ps.tp_all_reduce(emb)
    from . import linear
    kv = linear(emb, ew.wkv.w, torch.bfloat16)
    ss = torch.empty(T, dtype=torch.float32, device=X.device)
    _C.engram_gate(X, kv, ew.q_w, ew.k_w, cfg.rms_norm_eps, cfg.engram_clamp, ss)
    return ss


# ---------------------------------------------------------------------------
# self-checks of the switchable fast paths (run once at engine start)
# ---------------------------------------------------------------------------

def _moe_check_case():
    from . import ExpertWeights
    g = torch.Generator(device="cuda").manual_seed(11)
    E, H, I, K, T = 8, 512, 256, 2, 24

    def mx(n, k):
        a = quant((torch.randn(E * n, k, device="cuda", generator=g) * 0.05).to(torch.bfloat16))
        return MXFP8Tensor(a.q.view(E, n, k), a.sf.view(E, -1), n)
    ex = ExpertWeights(0, E, mx(2 * I, H), mx(H, I), I)
    x = quant(torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16))
    ids = torch.stack([torch.randperm(E, device="cuda", generator=g)[:K] for _ in range(T)]).int()
    w = torch.rand(T, K, device="cuda", generator=g)
    return ex, x, ids, w


def _check_moe(switch: str) -> bool:
    """moe_fused: one persistent launch == the two grouped launches;
    moe_pull: in-place row reads == the pre-gathered operand (bitwise)."""
    ex, x, ids, w = _moe_check_case()
    keep = {n: levers.on(n) for n in ("moe_fused", "moe_pull")}
    try:
        if switch == "moe_fused":
            levers.set_switch("moe_fused", False)
            ref_out = moe_experts(x, w, ids, ex, torch.float32)
            levers.set_switch("moe_fused", True)
            levers.set_switch("moe_pull", False)
        else:
            levers.set_switch("moe_fused", True)
            levers.set_switch("moe_pull", False)
            ref_out = moe_experts(x, w, ids, ex, torch.float32)
            levers.set_switch("moe_pull", True)
        out = moe_experts(x, w, ids, ex, torch.float32)
        torch.cuda.synchronize()
        check_device_errors()
        return bool(torch.equal(out, ref_out))
    finally:
        for n, v in keep.items():
            levers.set_switch(n, v)


def register_selfchecks() -> None:
    for name in ("moe_fused", "moe_pull"):
        sw = levers._REGISTRY[name]
        if not sw.checks:
            levers.add_check(name, lambda n=name: _check_moe(n))
