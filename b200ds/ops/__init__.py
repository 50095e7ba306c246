"""Op surface of the engine.

Every function takes plain tensors / weight containers.  CUDA tensors run the
hand-written sm_100a kernels of the in-tree extension (``b200ds._C``); a CUDA
call with the extension missing raises (no silent fallback).  CPU tensors run
the fp32 references in :mod:`b200ds.ops.ref`, which is how the engine is
tested without a GPU.  ``set_impl("torch")`` selects the library baseline on
the GPU (cuBLAS block-scaled GEMM via torch._scaled_mm, NCCL collectives),
the comparison arm for the benchmarks.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn.functional as F

from . import ref
from .quant import MXFP8Tensor, quant_mxfp8_ref, dequant_mxfp8, NVFP4Tensor

_IMPL = "native"


def set_impl(impl: str) -> None:
    assert impl in ("native", "torch")
    global _IMPL
    _IMPL = impl


def get_impl() -> str:
    return _IMPL


def _native():
    from . import cuda as _c
    return _c


def _use_native(t: torch.Tensor) -> bool:
    return t.is_cuda and _IMPL == "native"


def _use_baseline(t: torch.Tensor) -> bool:
    return t.is_cuda and _IMPL == "torch"


@dataclass
class QAct:
    """Activation quantized to MXFP8 (q e4m3 [T, K], sf packed sf128x4),
    optionally with the un-quantized bf16/fp32 copy ``hf``."""
    q: torch.Tensor
    sf: torch.Tensor
    hf: Optional[torch.Tensor] = None

    @property
    def shape(self):
        return self.q.shape


@dataclass
class ExpertWeights:
    """Stacked local experts.  w13 [E, 2I, h] (gate rows then up rows),
    w2 [E, h, I]; either float tensors or MXFP8 (data + per-expert sf)."""
    first: int
    count: int
    w13: object
    w2: object
    inter: int
    # NVFP4 experts: fixed fp32 global scale of the FC2 input (the SwiGLU
    # output), so e4m3 block scales cover block maxima up to 448*6*scale.
    fc2_act_scale: float = 1.0 / 32
    # weights stored as contiguous 128-row x 128-byte tiles (GPU serving
    # layout, see ops.quant.tile_rows128)
    tiled: bool = False
    # random-init bytes (benchmarks): any layout reads as the same distribution
    random_init: bool = False


@dataclass
class PendingLinear:
    """y = x W^T left uncomputed so the following all-reduce can run inside
    the GEMM's epilogue (fused GEMM + all-reduce)."""
    x: object
    w: object
    n_out: int


@dataclass
class MoEPartial:
    """Rank-partial MoE output before the combine: weighted expert rows
    y[rows, h], their per-(token, k) row index pair_row[T, K] (-1 = expert on
    another rank), and an optional additive partial (shared expert)."""
    y: torch.Tensor
    pair_row: torch.Tensor
    add: Optional[torch.Tensor] = None


@dataclass
class EPPartial:
    """Expert-parallel MoE output before its combine + reduce-scatter: weighted
    expert rows y over the world * T_step received tokens, their (token, k)
    row index pair_row [world * T_step, K], this rank's T_r own tokens and an
    optional additive partial for them (shared expert).  Consumed by the
    fused reduce-scatter + residual + RMSNorm."""
    y: Optional[torch.Tensor]
    pair_row: torch.Tensor
    T_step: int
    T_r: int
    add: Optional[torch.Tensor] = None
    # combine already stored by the experts' FC2 epilogue into the owners'
    # slots (y unused): the owner sums its tokens' K pair rows (ids [T_r, K],
    # < 0 = no expert)
    pushed: bool = False
    ids: Optional[torch.Tensor] = None


def materialize(a, out_dtype=torch.bfloat16) -> torch.Tensor:
    if isinstance(a, PendingLinear):
        y = linear(a.x, a.w, out_dtype)
        return y if y.shape[-1] == a.n_out else y[..., : a.n_out]
    if isinstance(a, MoEPartial):
        from . import cuda
        T = a.pair_row.shape[0]
        out = torch.empty(T, a.y.shape[1], dtype=out_dtype, device=a.y.device)
        add = a.add.to(torch.bfloat16).contiguous() if a.add is not None else None
        cuda._C.moe_combine(a.y, a.pair_row, add, out)
        return out
    return a


def to_float(x) -> torch.Tensor:
    if isinstance(x, QAct):
        if x.hf is not None:
            return x.hf.float()
        return dequant_mxfp8(x.q, x.sf)
    return x.float()


def quant(x: torch.Tensor) -> QAct:
    if _use_native(x):
        return _native().quant(x)
    q, sf = quant_mxfp8_ref(x.float())
    return QAct(q, sf, None)


# ---------------------------------------------------------------------------
# norms
# ---------------------------------------------------------------------------

def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    if _use_native(x):
        return _native().rmsnorm(x, w, eps)
    if _use_baseline(x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)
    return ref.rmsnorm(x, w, eps)


def rmsnorm_act(x: torch.Tensor, w: torch.Tensor, eps: float, next_linear=None, keep_hf: bool = True):
    """RMSNorm producing the operand format the next linear consumes."""
    if next_linear is not None and getattr(next_linear, "quantized", False):
        if _use_native(x):
            return _native().rmsnorm_quant(x, w, eps, keep_hf)
        if x.is_cuda:
            from . import baseline
            return baseline.rmsnorm_quant(x, w, eps, keep_hf)
        y = rmsnorm(x, w, eps)
        a = quant(y)
        a.hf = y if keep_hf else None
        return a
    return rmsnorm(x, w, eps)


def allreduce_add_rmsnorm(a: torch.Tensor, residual: torch.Tensor, w: torch.Tensor, eps: float,
                          ps, kind: str, next_linear=None):
    """All-reduce the rank-partial output ``a`` over the TP group, add it to
    the residual stream, RMSNorm, and quantize for ``next_linear``.
    Returns (normalized activation, new residual).  ``a`` may be a
    PendingLinear / MoEPartial, which the fused path folds into its GEMM or
    combine kernel."""
    if residual.is_cuda and _IMPL == "native" and (ps.tp_size > 1 or isinstance(a, EPPartial)):
        return _native().allreduce_add_rmsnorm(a, residual, w, eps, ps, next_linear)
    a = materialize(a, torch.float32 if not residual.is_cuda else torch.bfloat16)
    if ps.tp_size > 1 or (kind == "ffn" and ps.ep_size > 1):
        if ps.tp_size > 1:
            ps.tp_all_reduce(a)
        else:
            ps.ep_all_reduce(a)
    if a.is_cuda:
        if _IMPL == "native":
            return _native().add_rmsnorm_act(a, residual, w, eps, next_linear)
        residual = (residual.float() + a.float()).to(residual.dtype)
        return rmsnorm_act(residual, w, eps, next_linear), residual
    residual = residual.float() + a.float()
    return rmsnorm_act(residual, w, eps, next_linear), residual


# ---------------------------------------------------------------------------
# GEMM
# ---------------------------------------------------------------------------

def linear(x, w, out_dtype=torch.bfloat16) -> torch.Tensor:
    if isinstance(w, MXFP8Tensor):
        a = x if isinstance(x, QAct) else quant(x)
        if a.q.is_cuda:
            if _IMPL == "native":
                return _native().gemm(a, w, out_dtype)
            from . import baseline
            return baseline.gemm(a, w, out_dtype)
        return ref.gemm_mxfp8(a.q, a.sf, w.data, w.sf).to(out_dtype)
    xf = to_float(x)
    if xf.is_cuda:
        return (xf.to(w.dtype) @ w.T).to(out_dtype)
    return (xf @ w.float().T).to(out_dtype)


def gate_up_swiglu(x, gate_up) -> object:
    """silu(x Wg^T) * (x Wu^T) for a [2I, h] gate_up weight; returns the
    operand the down projection consumes (QAct for quantized weights)."""
    if gate_up.quantized:
        a = x if isinstance(x, QAct) else quant(x)
        if a.q.is_cuda and _IMPL == "native":
            return _native().gemm_swiglu_quant(a, gate_up.w)
        y = linear(a, gate_up.w, torch.float32)
        h = ref.swiglu(y)
        return quant(h.to(torch.bfloat16) if h.is_cuda else h)
    y = gate_up(x, out_dtype=torch.float32)
    return ref.swiglu(y)


# ---------------------------------------------------------------------------
# rope / kv cache / attention
# ---------------------------------------------------------------------------

def rope(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    if _use_native(x):
        return _native().rope(x, pos, table)
    return ref.rope(x, pos, table)


def kv_store(kv_a: torch.Tensor, ln_w: torch.Tensor, eps: float, table: torch.Tensor, pos: torch.Tensor,
             cache: torch.Tensor, slots: torch.Tensor, kv_scale: float, kv_lora: int) -> None:
    """cache[slots] = quant([rmsnorm(kv_a[:, :kv_lora]) | rope(kv_a[:, kv_lora:])] / kv_scale)."""
    if _use_native(kv_a):
        return _native().kv_store(kv_a, ln_w, eps, table, pos, cache, slots, kv_scale, kv_lora)
    ckv = ref.rmsnorm(kv_a[:, :kv_lora], ln_w, eps)
    kpe = ref.rope(kv_a[:, kv_lora:], pos, table)
    if cache.dtype == torch.float8_e4m3fn:
        cache[slots.long()] = ref.kv_quant(ckv, kpe, kv_scale)
    else:
        cache[slots.long()] = (torch.cat([ckv, kpe], -1) / kv_scale).to(cache.dtype)


def absorb_q(q_nope: torch.Tensor, w_uk: torch.Tensor) -> torch.Tensor:
    """[T, H, nope] x [H, nope, L] -> [T, H, L]."""
    if q_nope.is_cuda:
        return torch.bmm(q_nope.transpose(0, 1).to(w_uk.dtype), w_uk).transpose(0, 1)
    return torch.einsum("thd,hdc->thc", q_nope.float(), w_uk.float())


def absorb_o(o_lat: torch.Tensor, w_uv: torch.Tensor, quantize: bool = False):
    """[T, H, L] x [H, v, L] -> [T, H*v].  With quantize=True on the native
    path the result comes back as the MXFP8 operand of the output projection
    (quantized straight from the head-major batched-GEMM output)."""
    T, H, L = o_lat.shape
    if o_lat.is_cuda:
        if (quantize and _IMPL == "native" and w_uv.dtype == torch.bfloat16 and w_uv.shape[1] % 128 == 0
                and o_lat.dtype == torch.bfloat16):
            return _native().absorb_o_mx(o_lat, w_uv.contiguous())
        y = torch.bmm(o_lat.transpose(0, 1).to(w_uv.dtype), w_uv.transpose(1, 2))      # [H, T, v]
        if quantize and _IMPL == "native":
            return _native().quant_heads(y)
        return y.transpose(0, 1).reshape(T, -1)
    return torch.einsum("thc,hdc->thd", o_lat.float(), w_uv.float()).reshape(T, -1)


def mla_from_q(q_nope, q_pe, w_uk, w_uk_t, cache, kv_scale, fb, softmax_scale, page_size, topk, rope_table):
    """Absorbed MLA from the projected query: q_nope [T,H,nope] is absorbed
    into the latent space (w_uk [H,nope,L]; w_uk_t = its [H,L,nope] copy used
    by the fused tensor-core kernel), q_pe [T,H,rope] is rotated here."""
    if (_use_native(q_nope) and w_uk_t is not None and q_nope.dtype == torch.bfloat16 and page_size == 64
            and w_uk_t.shape[1] == 512 and q_nope.shape[1] % 16 == 0 and q_pe.shape[-1] == 64):
        return _native().mla_decode_from_q(q_nope, q_pe, w_uk_t, cache, kv_scale, fb, softmax_scale, page_size,
                                           topk, rope_table)
    q_abs = absorb_q(q_nope, w_uk)
    return mla_attention(q_abs, q_pe, cache, kv_scale, fb, softmax_scale, page_size, topk, rope_table=rope_table)


def mla_attention(q_abs, q_pe, cache, kv_scale, fb, softmax_scale, page_size, topk=None, rope_table=None):
    """Absorbed MLA.  With rope_table, q_pe is the un-rotated rope part and
    RoPE is applied here (fused into the native kernel's query prep)."""
    if _use_native(q_abs):
        return _native().mla_attention(q_abs, q_pe, cache, kv_scale, fb, softmax_scale, page_size, topk,
                                       rope_table=rope_table)
    if rope_table is not None:
        q_pe = ref.rope(q_pe, fb.positions, rope_table)
    if _use_baseline(q_abs) and topk is None and cache.dtype == torch.float8_e4m3fn:
        from . import baseline
        if fb.is_decode and page_size in (32, 64) and baseline.flashinfer_ok():
            return baseline.mla_decode_flashinfer(q_abs, q_pe, cache, kv_scale, fb, softmax_scale, page_size)
        if fb.is_decode and int(q_abs.shape[0]) == int(fb.block_table.shape[0]):
            return baseline.mla_decode_torch(q_abs, q_pe, cache, kv_scale, fb, softmax_scale, page_size)
        return baseline.mla_prefill_torch(q_abs, q_pe, cache, kv_scale, fb, softmax_scale, page_size)
    out = ref.mla_attention(q_abs, q_pe, cache, kv_scale, fb.block_table, fb.seq_lens, fb.q_seq,
                            fb.positions, softmax_scale, page_size, topk)
    return out.to(q_abs.dtype) if q_abs.is_cuda else out


def index_k_store(k, ln_w, ln_b, eps: float, table, pos, cache: torch.Tensor, scale: torch.Tensor,
                  slots: torch.Tensor) -> None:
    """Indexer keys: LayerNorm -> RoPE on the first rope dims -> per-token
    e4m3 (fp32 scale) into the paged indexer cache."""
    if _use_native(k):
        return _native().index_k_store(k, ln_w, ln_b, eps, table, pos, cache, scale, slots)
    hd = k.shape[-1]
    rd = table.shape[-1]
    kf = torch.nn.functional.layer_norm(to_float(k), (hd,), ln_w.float(), ln_b.float(), eps)
    kf = torch.cat([ref_rope(kf[:, :rd], pos, table), kf[:, rd:]], -1)
    if cache.dtype == torch.float8_e4m3fn:
        s = kf.abs().amax(-1).clamp(min=1e-12) / 448.0
        cache[slots.long()] = (kf / s.unsqueeze(-1)).to(cache.dtype)
        scale[slots.long()] = s
    else:
        cache[slots.long()] = kf.to(cache.dtype)
        scale[slots.long()] = 1.0


def indexer_topk(q_raw, w_raw, w_factor: float, table, k_cache, k_scale, fb, page_size: int, topk: int,
                 swa: int = 0):
    """Top-k cache positions [T, topk] (-1 padded, ascending) of the lightning
    indexer: q_raw [T, NH*hd] before RoPE, w_raw [T, NH] head weights before
    the w_factor scaling."""
    if _use_native(q_raw):
        return _native().indexer_topk(q_raw, w_raw, w_factor, table, k_cache, k_scale, fb, page_size, topk, swa)
    T, nh = w_raw.shape
    rd = table.shape[-1]
    q = to_float(q_raw).reshape(T, nh, -1)
    q = torch.cat([ref_rope(q[..., :rd], fb.positions, table), q[..., rd:]], -1)
    w = to_float(w_raw) * w_factor
    return ref.indexer_scores(q, w, k_cache, k_scale, fb.block_table, fb.q_seq, fb.positions, page_size, topk, swa)


def ref_rope(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    from ..models.rope import apply_rope_ref
    return apply_rope_ref(x.float(), pos, table)


# ---------------------------------------------------------------------------
# MoE
# ---------------------------------------------------------------------------

def router(h, gate: torch.Tensor, bias: torch.Tensor, cfg):
    x = to_float(h) if not (isinstance(h, QAct) and h.hf is not None and h.hf.is_cuda) else h.hf
    if _use_native(x):
        return _native().router(x, gate, bias, cfg)
    logits = x.float() @ gate.float().T
    if cfg.scoring_func == "sqrtsoftplus":
        return ref.router_sqrtsoftplus(logits, bias, cfg.num_experts_per_tok, cfg.routed_scaling_factor)
    return ref.router_topk(logits, bias, cfg.num_experts_per_tok, cfg.n_group, cfg.topk_group,
                           cfg.routed_scaling_factor, cfg.norm_topk_prob)


def moe_experts_ep(h, w: torch.Tensor, ids: torch.Tensor, ex: ExpertWeights, T_step: int, n_experts_total: int,
                   ep, far=None) -> EPPartial:
    """Expert-parallel MoE on the fused NVLink path: dispatch this rank's
    routed tokens to the expert owners, run the grouped GEMMs over the
    received tokens; returns the partial for the fused combine (with `far`,
    the expert-parallel all-reduce workspace, the FC2 epilogue stores each
    pair's row straight into its owner's slot)."""
    return _native().moe_experts_ep(h, w, ids, ex, T_step, n_experts_total, ep, far)


def moe_experts(h, w: torch.Tensor, ids: torch.Tensor, ex: ExpertWeights, out_dtype=torch.float32,
                n_experts_total=None, combine: bool = True):
    """Local-expert part of the MoE: sum_k w[t,k] * expert_{ids[t,k]}(h[t]) over
    the experts this rank owns (others contribute on their ranks)."""
    if isinstance(ex.w13, NVFP4Tensor):
        x = h.hf if isinstance(h, QAct) and h.hf is not None else h
        if (x.q if isinstance(x, QAct) else x).is_cuda and _IMPL == "native":
            return _native().moe_experts_nvfp4(h, w, ids, ex, out_dtype, n_experts_total, combine)
        return _moe_nvfp4_ref(to_float(h), w, ids, ex).to(out_dtype)
    if isinstance(ex.w13, MXFP8Tensor) and (h.q if isinstance(h, QAct) else h).is_cuda:
        if _IMPL == "native":
            return _native().moe_experts(h, w, ids, ex, out_dtype, n_experts_total, combine)
        from . import baseline
        xb = h.hf if isinstance(h, QAct) and h.hf is not None else (
            dequant_mxfp8(h.q, h.sf).to(torch.bfloat16) if isinstance(h, QAct) else h.to(torch.bfloat16))
        if baseline.flashinfer_ok() and n_experts_total is not None:
            return baseline.moe_experts_flashinfer(xb.contiguous(), w, ids, ex, n_experts_total).to(out_dtype)
        if baseline.grouped_mx_ok(xb.device):
            return baseline.moe_experts_grouped(xb, w, ids, ex, out_dtype)
        return baseline.moe_experts(h if isinstance(h, QAct) else quant(h), w, ids, ex, out_dtype)
    xf = to_float(h)
    T = xf.shape[0]
    out = torch.zeros(T, xf.shape[1], dtype=torch.float32, device=xf.device)
    quantized = isinstance(ex.w13, MXFP8Tensor)
    for e in range(ex.count):
        gid = ex.first + e
        hit = (ids == gid)
        tok = hit.any(-1).nonzero().flatten()
        if tok.numel() == 0:
            continue
        we = (w * hit).sum(-1)[tok].unsqueeze(-1)
        if quantized:
            a = QAct(*quant_mxfp8_ref(xf[tok]))
            w13 = MXFP8Tensor(ex.w13.data[e], ex.w13.sf[e])
            w2 = MXFP8Tensor(ex.w2.data[e], ex.w2.sf[e])
            y = ref.swiglu(ref.gemm_mxfp8(a.q, a.sf, w13.data, w13.sf))
            a2 = QAct(*quant_mxfp8_ref(y))
            o = ref.gemm_mxfp8(a2.q, a2.sf, w2.data, w2.sf)
        else:
            y = ref.swiglu(xf[tok] @ ex.w13[e].float().T)
            o = y @ ex.w2[e].float().T
        out.index_add_(0, tok, we * o)
    return out.to(out_dtype)


def _moe_nvfp4_ref(xf: torch.Tensor, w: torch.Tensor, ids: torch.Tensor, ex: ExpertWeights) -> torch.Tensor:
    """fp32 reference of the NVFP4 experts, with the activations quantized as
    the kernels do (FC1 input: per-token global scale; FC2 input: the fixed
    fc2_act_scale)."""
    from .quant import dequant_nvfp4_rows, quant_nvfp4_rows
    T = xf.shape[0]
    out = torch.zeros(T, xf.shape[1], dtype=torch.float32, device=xf.device)
    for e in range(ex.count):
        gid = ex.first + e
        hit = (ids == gid)
        tok = hit.any(-1).nonzero().flatten()
        if tok.numel() == 0:
            continue
        we = (w.float() * hit).sum(-1)[tok].unsqueeze(-1)
        a = dequant_nvfp4_rows(*quant_nvfp4_rows(xf[tok]))
        w13 = dequant_nvfp4_rows(ex.w13.data[e], ex.w13.sf[e], ex.w13.global_scale[e])[: 2 * ex.inter]
        y = ref.swiglu(a @ w13.T)
        a2 = dequant_nvfp4_rows(*quant_nvfp4_rows(y, ex.fc2_act_scale))
        w2 = dequant_nvfp4_rows(ex.w2.data[e], ex.w2.sf[e], ex.w2.global_scale[e])[: xf.shape[1]]
        out.index_add_(0, tok, we * (a2 @ w2.T))
    return out


# ---------------------------------------------------------------------------
# LM head / sampling
# ---------------------------------------------------------------------------

def lm_head_local(x, head) -> torch.Tensor:
    """This rank's vocabulary shard of the logits [B, V_local] (bf16 from
    the MXFP8 tensor-core GEMM for a quantized head, else fp32)."""
    if isinstance(head, MXFP8Tensor):
        y = linear(x if isinstance(x, QAct) else to_float(x), head, torch.bfloat16)
        n = head.rows if head.rows is not None else head.data.shape[0]
        return y if y.shape[-1] == n else y[..., :n]
    xf = to_float(x)
    if xf.is_cuda:
        return (xf.to(head.dtype) @ head.T).float()
    return xf.float() @ head.float().T


def lm_head_logits(x, head, ps) -> torch.Tensor:
    """Full-vocabulary fp32 logits (vocab shards all-gathered over TP)."""
    return ps.tp_all_gather(lm_head_local(x, head).float().contiguous(), dim=-1)


def sample_tokens(local_logits: torch.Tensor, vocab_off: int, temperature, top_p, top_k, uniform, ps) -> torch.Tensor:
    """Token ids [B] sampled from the vocab-parallel logits without gathering
    them: native kernels exchange per-rank candidates only; the reference
    path gathers and samples the full logits."""
    if _use_native(local_logits):
        return _native().sample_tokens(local_logits, vocab_off, temperature, top_p, top_k, uniform, ps)
    full = ps.tp_all_gather(local_logits.float().contiguous(), dim=-1)
    return sample(full, temperature, top_p, top_k, uniform)


def sample(logits: torch.Tensor, temperature, top_p, top_k, uniform) -> torch.Tensor:
    if _use_native(logits):
        return _native().sample(logits, temperature, top_p, top_k, uniform)
    if _use_baseline(logits):
        from . import baseline
        return baseline.sample_torch(logits, temperature, top_p, top_k, uniform)
    return ref.sample(logits, temperature, top_p, top_k, uniform)


# ---------------------------------------------------------------------------
# DeepSeek-V4 family: mHC residual streams, MQA with sinks, E5, Engram
# ---------------------------------------------------------------------------

@dataclass
class HcWeights:
    """Coefficient weights of one hyper-connection (a sublayer's or the
    head's): fn [M, hc*D] fp32, scale [3] (sublayer) or [1] (head), base [M].
    fn_parts (GPU): [128, hc*D] bf16 holding fn as hi / mid / lo bf16 parts
    (rows p*M + j), the weight operand of the tcgen05 stats GEMM."""
    fn: torch.Tensor
    scale: torch.Tensor
    base: torch.Tensor
    fn_parts: Optional[torch.Tensor] = None

    @property
    def m(self) -> int:
        return self.fn.shape[0]


@dataclass
class EngramWeights:
    """Engram table shard (rows [row_lo, row_lo + rows) of the layer's
    table, e4m3 bytes [rows, dim] + UE8M0 [rows, dim/32], in pinned host
    memory on GPU ranks), the kv projection and the gate norms."""
    table: torch.Tensor
    scale: torch.Tensor
    row_lo: int
    wkv: object            # Linear [2D, heads*dim]
    q_w: torch.Tensor
    k_w: torch.Tensor


def hc_embed(embed: torch.Tensor, ids: torch.Tensor, hc: int):
    """Residual streams of the first layer: every stream = the token's
    embedding row.  Returns (X [T, hc, D], sum of squares [T])."""
    if _use_native(embed):
        return _native().hc_embed(embed, ids, hc)
    e = embed[ids.long()].float()
    X = e.unsqueeze(1).expand(-1, hc, -1).contiguous()
    return X, X.pow(2).sum((1, 2))


def hc_post(X: torch.Tensor, y: torch.Tensor, post: torch.Tensor, comb: torch.Tensor) -> torch.Tensor:
    """X <- post * y + comb^T X (in place); returns the new sum of squares [T]."""
    if _use_native(X):
        return _native().hc_post(X, y, post, comb)
    hc = X.shape[1]
    out = ref.hc_post(X, y, post, comb.reshape(-1, hc, hc))
    X.copy_(out)
    return out.pow(2).sum((1, 2))


def hc_pre(X: torch.Tensor, sumsq: torch.Tensor, hw: HcWeights, norm_w: torch.Tensor, eps: float, cfg,
           next_linear=None, head: bool = False, keep_hf: bool = False):
    """Sublayer coefficients from the streams and the sublayer input
    RMSNorm(sum_c pre_c X_c) * norm_w in the operand format of next_linear.
    Returns (h, post, comb) (head=True: post and comb are None)."""
    if _use_native(X):
        return _native().hc_pre(X, sumsq, hw, norm_w, eps, cfg, next_linear, head, keep_hf)
    hc, D = X.shape[1], X.shape[2]
    raw = X.float().flatten(1) @ hw.fn.float().T
    if head:
        pre = ref.hc_head_coeffs(raw, sumsq, hw.scale, hw.base, hc, hc * D, cfg.hc_eps)
        post = comb = None
    else:
        pre, post, comb = ref.hc_coeffs(raw, sumsq, hw.scale, hw.base, hc, hc * D, cfg.hc_sinkhorn_iters,
                                        cfg.hc_eps)
        comb = comb.reshape(-1, hc * hc)
    x = ref.hc_combine(X, pre)
    if X.is_cuda:
        x = x.to(torch.bfloat16)
    return rmsnorm_act(x, norm_w, eps, next_linear, keep_hf), post, comb


def hc_boundary(X: torch.Tensor, carry, hw: HcWeights, norm_w: torch.Tensor, eps: float, cfg, next_linear=None,
                head: bool = False, keep_hf: bool = False, sumsq: Optional[torch.Tensor] = None):
    """A whole hyper-connection boundary: hc_post of the previous sublayer's
    output carry = (y, post, comb) into X (None: X is already up to date and
    sumsq holds its row sums of squares), then hc_pre.  Returns (h, post,
    comb) like hc_pre.  On GPUs decode-sized batches run it as one kernel."""
    if _use_native(X) and _native().hc_boundary_ok(X):
        return _native().hc_boundary(X, carry, hw, norm_w, eps, cfg, next_linear, head, keep_hf)
    if carry is not None:
        sumsq = hc_post(X, *carry)
    return hc_pre(X, sumsq, hw, norm_w, eps, cfg, next_linear, head=head, keep_hf=keep_hf)


def hc_mean(X: torch.Tensor) -> torch.Tensor:
    if _use_native(X):
        return _native().hc_mean(X)
    return X.float().mean(1)


def kv_store_v4(kv: torch.Tensor, w: torch.Tensor, eps: float, table: torch.Tensor, pos: torch.Tensor,
                cache: torch.Tensor, slots: torch.Tensor, kv_scale: float, rd: int) -> None:
    """cache[slots, :L] = (rmsnorm(kv) with RoPE on its last rd dims) /
    kv_scale; the row's rope-key part stays zero (K = V = the latent row)."""
    if _use_native(kv):
        return _native().kv_store_v4(kv, w, eps, table, pos, cache, slots, kv_scale, rd)
    L = kv.shape[1]
    x = ref.rmsnorm(kv, w, eps)
    x = torch.cat([x[:, :L - rd], ref.rope(x[:, L - rd:], pos, table)], -1)
    row = torch.zeros(x.shape[0], cache.shape[1], dtype=torch.float32)
    row[:, :L] = x / kv_scale
    if cache.dtype == torch.float8_e4m3fn:
        cache[slots.long()] = row.clamp(-448, 448).to(cache.dtype)
    else:
        cache[slots.long()] = row.to(cache.dtype)


def mqa_attention(q: torch.Tensor, cache: torch.Tensor, kv_scale: float, fb, softmax_scale: float, page_size: int,
                  sink: Optional[torch.Tensor], table: torch.Tensor, rd: int, topk=None, comp=None) -> torch.Tensor:
    """MQA over the paged latent rows (K = V = row[:L]) with RoPE on the
    query tails, per-head sinks, and the output tails rotated back to
    position 0.  q [T, H, L] -> o [T, H, L].  comp = (compressed rows,
    ratio): selection entries >= ref.COMP_FLAG name compressed blocks."""
    if _use_native(q):
        return _native().mqa_attention(q, cache, kv_scale, fb, softmax_scale, page_size, sink, table, rd, topk,
                                       comp=comp)
    T, H, L = q.shape
    qf = q.float()
    qf = torch.cat([qf[..., :L - rd], ref.rope(qf[..., L - rd:], fb.positions, table)], -1)
    o = ref.mqa_sink_attention(qf, cache, kv_scale, fb.block_table, fb.q_seq, fb.positions, softmax_scale, page_size,
                               sink, L, topk, comp=comp)
    return ref.inv_rope_tail(o, fb.positions, table, rd)


def compress_store(g: torch.Tensor, bias: torch.Tensor, fb, r: int, kv_cache: torch.Tensor, kv_scale: float,
                   ix_cache: torch.Tensor, ix_scale: torch.Tensor, gate: torch.Tensor, ckv: torch.Tensor,
                   cik: torch.Tensor, cis: torch.Tensor, page_size: int) -> None:
    """Compressed attention: store this step's gate logits g [T] and write
    the compressed latent rows / indexer keys of the blocks the step
    completes (ref.compress_store)."""
    if _use_native(kv_cache):
        return _native().compress_store(g, bias, fb, r, kv_cache, kv_scale, ix_cache, ix_scale, gate, ckv, cik, cis,
                                        page_size)
    ref.compress_store(to_float(g), bias, fb.positions, fb.out_slots, fb.q_seq, fb.block_table, r, kv_cache,
                       kv_scale, ix_cache, ix_scale, gate, ckv, cik, cis, page_size)


def indexer_topk_compressed(q_raw, w_raw, w_factor: float, table, cik, cis, fb, page_size: int, r: int, topk: int,
                            swa: int):
    """Selection of a compressed-attention layer [T, swa + topk]: the window
    positions, then the indexer's top compressed blocks before the window
    (entries COMP_FLAG + block)."""
    if _use_native(q_raw):
        return _native().indexer_topk_compressed(q_raw, w_raw, w_factor, table, cik, cis, fb, page_size, r, topk,
                                                 swa)
    T, nh = w_raw.shape
    rd = table.shape[-1]
    q = to_float(q_raw).reshape(T, nh, -1)
    q = torch.cat([ref_rope(q[..., :rd], fb.positions, table), q[..., rd:]], -1)
    w = to_float(w_raw) * w_factor
    return ref.indexer_select_compressed(q, w, cik, cis, fb.block_table, fb.q_seq, fb.positions, page_size, r,
                                         topk, swa)


def e5_prune(w: torch.Tensor, ids: torch.Tensor, cfg, n_experts: int):
    """E5 routed-expert prune of a decode batch (returns new (w, ids))."""
    if _use_native(ids):
        return _native().e5_prune(w, ids, cfg, n_experts)
    return ref.e5_prune(ids, w, cfg.prune_budget, cfg.prune_max_count)


def engram_ids(fb, tok_cache: torch.Tensor, cfg, mults: torch.Tensor, page_size: int) -> torch.Tensor:
    """Hash ids [T, heads] of each token's n-grams (the tokens before this
    batch come from tok_cache, the token stored at every KV slot, which this
    call updates with the batch's tokens)."""
    if _use_native(fb.input_ids):
        return _native().engram_ids(fb, tok_cache, cfg, mults, page_size)
    T = fb.num_tokens
    n = cfg.engram_max_ngram
    ctx = torch.full((T, n), -1, dtype=torch.int64)
    ids = fb.input_ids.long()
    pos, qs = fb.positions.long(), fb.q_seq.long()
    for t in range(T):
        p, b = int(pos[t]), int(qs[t])
        for i in range(n):
            pp = p - i
            if pp < 0:
                continue
            if i == 0:
                ctx[t, i] = ids[t]
            elif t - i >= 0 and int(qs[t - i]) == b and int(pos[t - i]) == pp:
                ctx[t, i] = ids[t - i]
            else:
                page = int(fb.block_table[b, pp // page_size])
                ctx[t, i] = int(tok_cache[page * page_size + pp % page_size])
    tok_cache[fb.out_slots.long()] = fb.input_ids.to(tok_cache.dtype)
    return ref.engram_hash(ctx, cfg.engram_heads, cfg.engram_rows, n)


def engram_update(X: torch.Tensor, ids: torch.Tensor, ew: EngramWeights, cfg, ps) -> torch.Tensor:
    """Gather the hashed rows (this rank's shard; all-reduced over TP), project
    to [k | v], gate v into every stream (X in place).  Returns the new sum
    of squares of X [T]."""
    if _use_native(X):
        return _native().engram_update(X, ids, ew, cfg, ps)
    emb = ref.engram_gather(ew.table, ew.scale, ids, ew.row_lo, ew.row_lo + ew.table.shape[0])
    emb = emb.flatten(1)
    if ps.tp_size > 1:
        ps.tp_all_reduce(emb)
    kv = linear(emb, ew.wkv.w, torch.float32)
    out = ref.engram_gate(X, kv, ew.q_w, ew.k_w, cfg.rms_norm_eps, cfg.engram_clamp)
    X.copy_(out)
    return out.pow(2).sum((1, 2))
