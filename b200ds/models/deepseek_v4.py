"""DeepSeek-V4-family decoder for the serving engine (arch="deepseek_v4").

Per token the residual state is hc streams X [hc, D] (bf16 on the GPU).  Each
sublayer (attention, then FFN) runs three kernels around its body:
  * hc_post (previous sublayer): X <- post * y + comb^T X, with the sum of
    squares of the new streams (the RMS of the coefficients);
  * the stats GEMM on the tensor cores: raw = X_flat . fn^T with fn split in
    bf16 hi / mid / lo parts (split-K, fp32 accumulation);
  * hc_pre: pre / post / comb (row softmax + Sinkhorn on 16 lanes) and the
    sublayer input RMSNorm(sum_c pre_c X_c) * w as the next GEMM's MXFP8
    operand.
Attention is MQA over one latent row per token (K = V, RoPE on its tail)
through the tcgen05 latent-attention kernel, with per-head sinks and the
inverse RoPE of the output tail in one fix-up kernel; the output projection
is the grouped low-rank wo_a on the bf16 tensor-core batched GEMM (its
epilogue writes wo_b's MXFP8 operand) then wo_b.  MoE: sqrt-softplus router
(+ E5 prune at decode) into the fused expert kernels.  Engram layers gate
hashed host-table rows into every stream before their attention.

Parallelism: TP over heads / output groups / FFN columns with an all-reduce
after each sublayer, routed experts EP-split over the same ranks (one
all-reduce for routed + shared), Engram tables row-sharded (zeros for rows
owned elsewhere, summed by the all-reduce), vocab-parallel LM head.

Reference parity: fork_loop.py:59-226 (layer loop with hc_broadcast /
hc_combine head), hq_layer.py:32-101 / fg_layer.py (hyper-connection
sublayers), fork_attn.py:380-553 (MQA, sinks, inverse rope, wo_a / wo_b),
moe_fwd.py:67-263 (MoE), eg.py:355-390 (Engram), aux.py (stream means).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from .. import ops
from ..config import EngineConfig, ModelConfig
from ..ops import EngramWeights, HcWeights
from ..parallel.state import ParallelState
from .batch import ForwardBatch
from .deepseek import DenseWeights, Linear, MoEWeights, _drain
from .rope import cos_sin_table


@dataclass
class V4AttnWeights:
    wqkv_a: Linear                # [q_lora + L, D]
    q_norm: torch.Tensor
    kv_norm: torch.Tensor
    wq_b: Linear                  # [Hl * L, q_lora]
    wo_a: torch.Tensor            # [Gl, R, (H/G) * L]
    wo_b: Linear                  # [D, Gl * R]
    sink: Optional[torch.Tensor]  # [Hl]
    # sparse attention: the lightning indexer's projections ride on the
    # attention GEMMs (wk and weights_proj rows appended to wqkv_a, the
    # indexer's wq_b rows to wq_b)
    ix_k_norm_w: Optional[torch.Tensor] = None
    ix_k_norm_b: Optional[torch.Tensor] = None
    # compressed sparse attention: the compressor's gate row rides on wqkv_a
    # (after the indexer rows); per-position-in-block gate bias [ratio]
    comp_bias: Optional[torch.Tensor] = None


@dataclass
class V4LayerWeights:
    attn_hc: HcWeights
    ffn_hc: HcWeights
    in_ln: torch.Tensor
    post_ln: torch.Tensor
    attn: V4AttnWeights
    ffn: object                   # DenseWeights | MoEWeights
    engram: Optional[EngramWeights] = None


@dataclass
class _Partial:
    """A sublayer output that is still this rank's partial sum (tensor
    parallelism): its all-reduce runs fused with the hyper-connection post."""
    y: torch.Tensor


class DeepseekV4Model:
    supports_cp = True        # context-parallel prefill under DP attention (parallel/cp.py)
    supports_tbo = True       # two-batch overlap of DP-attention prefill steps (forward_tbo)
    _tbo_live = False         # forward_tbo is interleaving micro-batches

    @property
    def tbo_splits_decode(self) -> bool:
        """Whether a decode batch may be cut into two micro-batches: not with
        the E5 prune, whose routing depends on the whole decode batch."""
        return not self.cfg.prune_budget > 0

    def __init__(self, cfg: ModelConfig, ecfg: EngineConfig, ps: ParallelState, layers: List[V4LayerWeights],
                 embed: torch.Tensor, hc_head: HcWeights, final_ln: torch.Tensor, lm_head, device,
                 kv_dtype=torch.float8_e4m3fn):
        assert cfg.is_v4 and cfg.hc_mult > 0
        self.cfg, self.ecfg, self.ps = cfg, ecfg, ps
        self.layers = layers
        self.embed = embed
        self.hc_head = hc_head
        self.final_ln = final_ln
        self.lm_head = lm_head
        self.device = torch.device(device)
        self.kv_dtype = kv_dtype
        self.heads = cfg.num_attention_heads // ps.tp_size
        self.groups = cfg.o_groups // ps.tp_size
        # DP attention: each rank runs attention, mHC, Engram, dense / shared
        # FFNs and the LM head for its own requests with replicated weights
        # (tp_size 1); only the routed experts are EP-split
        self.dp = bool(ecfg.dp_attention) and ps.ep_size > 1
        self.rope_table = cos_sin_table(cfg, cfg.max_position_embeddings, device=self.device)
        self.kv_scale = [1.0] * len(layers)
        self.kv_cache: List[torch.Tensor] = []
        self.tok_cache: Optional[torch.Tensor] = None
        self.page_size = ecfg.page_size
        self.aux: List[torch.Tensor] = []
        self.tail_skipped = 0            # rows the last prefill tail left out of the window layers
        from ..utils.trace import null_tracer
        self.tracer = null_tracer()
        from ..ops.ref import engram_multipliers
        m = [v - (1 << 64) if v >= (1 << 63) else v for v in engram_multipliers(max(cfg.engram_heads, 1))]
        self.engram_mults = torch.tensor(m, dtype=torch.int64, device=self.device)
        # tensor parallelism on GPUs: each sublayer's all-reduce runs fused
        # with the hyper-connection post (csrc/elementwise/v4.cu ar_hc_post)
        from ..utils import levers
        if (self.device.type == "cuda" and ps.tp_size > 1 and not self.dp and ecfg.comm_impl == "fused"
                and levers.on("fused_comm") and getattr(ps, "fused_ar", None) is None):
            from ..parallel.symm import FusedAllReduce
            # the V4 boundary kernel reads the push protocol's per-source slots
            ps.fused_ar = FusedAllReduce(ps, cfg.hidden_size, max_tokens=max(ecfg.max_num_seqs, 256),
                                         allow_nvls=False)

    # ------------------------------------------------------------------
    def allocate_kv(self, num_pages: int):
        c = self.cfg
        slots = num_pages * self.page_size
        self.kv_cache = [torch.zeros(slots, c.kv_cache_dim, dtype=self.kv_dtype, device=self.device)
                         for _ in self.layers]
        if c.index_n_heads:
            self.ix_cache = [torch.zeros(slots, c.index_head_dim, dtype=self.kv_dtype, device=self.device)
                             for _ in self.layers]
            self.ix_scale = [torch.ones(slots, dtype=torch.float32, device=self.device) for _ in self.layers]
        if c.engram_layers:
            self.tok_cache = torch.full((slots,), -1, dtype=torch.int32, device=self.device)
        # compressed sparse attention: per compressed layer the gate logit of
        # every slot, and one compressed latent row / indexer key (+ scale) per
        # r slots, paged with the same page ids (page_size / r rows a page)
        self.comp = {}
        for i in range(len(self.layers)):
            r = c.compress_ratio(i)
            if r:
                if r > 8 or self.page_size % r:
                    # a block lives in one page; the compressed keys' TMA
                    # boxes are whole 8-row swizzle atoms
                    raise ValueError(f"compress ratio {r} must divide the page size and be at most 8")
                n = slots // r
                self.comp[i] = dict(
                    ratio=r,
                    gate=torch.zeros(slots, dtype=torch.float32, device=self.device),
                    kv=torch.zeros(n, c.kv_cache_dim, dtype=self.kv_dtype, device=self.device),
                    ik=torch.zeros(n, c.index_head_dim, dtype=self.kv_dtype, device=self.device),
                    iks=torch.ones(n, dtype=torch.float32, device=self.device))

    def kv_tensors(self) -> List[torch.Tensor]:
        """Every cache tensor indexed by slot (slot = page * page_size +
        offset) or, for the compressed rows, by page * page_size / r + offset:
        what one KV page holds across the model."""
        out = list(self.kv_cache)
        out += list(getattr(self, "ix_cache", []) or []) + list(getattr(self, "ix_scale", []) or [])
        if self.tok_cache is not None:
            out.append(self.tok_cache)
        for cc in getattr(self, "comp", {}).values():
            out += [cc["gate"], cc["kv"], cc["ik"], cc["iks"]]
        return out

    def kv_bytes_per_token(self) -> int:
        c = self.cfg
        es = torch.tensor([], dtype=self.kv_dtype).element_size()
        per = c.kv_cache_dim * es + ((c.index_head_dim * es + 4) if c.index_n_heads else 0)
        total = per * len(self.layers) + (4 if c.engram_layers else 0)
        for i in range(len(self.layers)):
            r = c.compress_ratio(i)
            if r:
                total += 4 + (c.kv_cache_dim * es + c.index_head_dim * es + 4) // r
        return total

    def vocab_offset(self) -> int:
        rows = getattr(self.lm_head, "rows", None)
        n = rows if rows is not None else self.lm_head.shape[0]
        return self.ps.tp_rank * n

    # ------------------------------------------------------------------
    def _out_dtype(self):
        return torch.float32 if self.device.type == "cpu" else torch.bfloat16

    def _fused_post(self, T: int) -> bool:
        """The sublayer all-reduce is left to the fused all-reduce + hc_post."""
        far = getattr(self.ps, "fused_ar", None)
        return (far is not None and not self.dp and self.ps.tp_size > 1 and ops.get_impl() == "native"
                and far.supports(T))

    def _post(self, X, y, post, comb):
        """hc_post of a sublayer output y (a rank partial when the fused
        boundary runs, else already reduced); returns the row sum of squares."""
        if isinstance(y, _Partial):
            return self.ps.fused_ar.allreduce_hc_post(y.y, X, post, comb)
        return ops.hc_post(X, y, post, comb)

    def _reduce(self, y: torch.Tensor) -> torch.Tensor:
        if self.dp:                 # replicated weights, this rank's own tokens: nothing to sum
            return y
        if self._fused_post(y.shape[0]):
            return _Partial(y)
        if self.ps.tp_size > 1:
            self.ps.tp_all_reduce(y)
        elif self.ps.ep_size > 1:
            self.ps.ep_all_reduce(y)
        return y

    def _attention(self, i: int, lw: V4LayerWeights, h, fb: ForwardBatch) -> torch.Tensor:
        c = self.cfg
        aw = lw.attn
        T = fb.num_tokens
        L, rd, ql = c.kv_lora_rank, c.qk_rope_head_dim, c.q_lora_rank
        od = self._out_dtype()
        qkv = aw.wqkv_a(h, out_dtype=od)
        q_lat = ops.rmsnorm_act(qkv[:, :ql], aw.q_norm, c.rms_norm_eps, aw.wq_b, keep_hf=False)
        ops.kv_store_v4(qkv[:, ql:ql + L], aw.kv_norm, c.rms_norm_eps, self.rope_table, fb.positions,
                        self.kv_cache[i], fb.out_slots, self.kv_scale[i], rd)
        qo = aw.wq_b(q_lat, out_dtype=od)
        q = qo[:, : self.heads * L].view(T, self.heads, L)
        topk, comp = None, None
        cp_done = fb.cp is None
        if c.is_window_layer(i):
            # window-only layer: the selection is the last late_window positions
            # (built on the device from the positions, graph-safe)
            W = c.late_window
            topk = fb.positions.view(-1, 1).to(torch.int32) - torch.arange(W, dtype=torch.int32, device=fb.positions.device)
            topk = torch.where(topk >= 0, topk, torch.full_like(topk, -1))
        elif c.index_n_heads:
            nh, hd = c.index_n_heads, c.index_head_dim
            base = ql + L
            ops.index_k_store(qkv[:, base: base + hd], aw.ix_k_norm_w, aw.ix_k_norm_b, 1e-6, self.rope_table,
                              fb.positions, self.ix_cache[i], self.ix_scale[i], fb.out_slots)
            q_ix = qo[:, self.heads * L: self.heads * L + nh * hd]
            w_ix = qkv[:, base + hd: base + hd + nh]
            if c.compress_ratio(i):
                # the gate logits (the row after the indexer's), then the
                # compressed rows of the blocks this step completes, then the
                # window + top compressed blocks
                cc = self.comp[i]
                g, cfb = qkv[:, base + hd + nh], fb
                if not cp_done:
                    # context parallel: every rank's rows and gate logits first;
                    # then each rank compresses the chunk's blocks itself
                    g, cfb = self._cp_gather(i, fb, g), fb.cp.whole(fb)
                    cp_done = True
                ops.compress_store(g, aw.comp_bias, cfb, cc["ratio"], self.kv_cache[i],
                                   self.kv_scale[i], self.ix_cache[i], self.ix_scale[i], cc["gate"], cc["kv"],
                                   cc["ik"], cc["iks"], self.page_size)
                topk = ops.indexer_topk_compressed(q_ix, w_ix, (nh * hd) ** -0.5, self.rope_table, cc["ik"],
                                                   cc["iks"], fb, self.page_size, cc["ratio"], c.compress_topk,
                                                   c.index_swa)
                comp = (cc["kv"], cc["ratio"])
            else:
                if not cp_done:
                    self._cp_gather(i, fb)
                    cp_done = True
                topk = ops.indexer_topk(q_ix, w_ix, (nh * hd) ** -0.5, self.rope_table, self.ix_cache[i],
                                        self.ix_scale[i], fb, self.page_size, c.index_topk, c.index_swa)
        if not cp_done:
            self._cp_gather(i, fb)
        o = ops.mqa_attention(q, self.kv_cache[i], self.kv_scale[i], fb, c.softmax_scale, self.page_size, aw.sink,
                              self.rope_table, rd, topk, comp=comp)
        z = ops.absorb_o(o.reshape(T, self.groups, -1), aw.wo_a, quantize=aw.wo_b.quantized)
        y = aw.wo_b(z, out_dtype=od)
        return self._reduce(y)

    def _cp_gather(self, i: int, fb: ForwardBatch, gate: Optional[torch.Tensor] = None):
        """Context-parallel chunk: every rank's new cache rows of layer i (the
        latent row; the indexer key + scale where the layer stores one) into
        this rank's cache before any query of the chunk attends; a compressed
        layer's gate logits travel along (returned for the whole chunk)."""
        from ..parallel.cp import gather_rows
        c = self.cfg
        bufs = [self.kv_cache[i]]
        if c.index_n_heads and not c.is_window_layer(i):
            bufs += [self.ix_cache[i], self.ix_scale[i]]
        return gather_rows(bufs, fb, self.ps, extra=gate)

    def _ffn(self, i: int, lw: V4LayerWeights, h, fb: ForwardBatch) -> torch.Tensor:
        c = self.cfg
        od = self._out_dtype()
        if isinstance(lw.ffn, DenseWeights):
            return self._reduce(lw.ffn.down(ops.gate_up_swiglu(h, lw.ffn.gate_up), out_dtype=od))
        mw: MoEWeights = lw.ffn
        w, ids = ops.router(h, mw.gate, mw.bias, c)
        if fb.is_decode and c.prune_budget > 0:
            w, ids = ops.e5_prune(w, ids, c, c.n_routed_experts)
        if self.dp:
            return _drain(self._moe_dp_steps(mw, h, w, ids, fb))
        out = ops.moe_experts(h, w, ids, mw.experts, out_dtype=od, n_experts_total=c.n_routed_experts)
        if mw.shared_gate_up is not None:
            out = out + mw.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up), out_dtype=od)
        return self._reduce(out.to(od))

    def _ffn_steps(self, i: int, lw: V4LayerWeights, h, fb: ForwardBatch):
        """`_ffn` as a generator (yields inside the DP MoE exchange)."""
        if not (self.dp and isinstance(lw.ffn, MoEWeights)):
            return self._ffn(i, lw, h, fb)
        c, mw = self.cfg, lw.ffn
        w, ids = ops.router(h, mw.gate, mw.bias, c)
        if fb.is_decode and c.prune_budget > 0:
            w, ids = ops.e5_prune(w, ids, c, c.n_routed_experts)
        return (yield from self._moe_dp_steps(mw, h, w, ids, fb))

    def _moe_dp_steps(self, mw: MoEWeights, h, w: torch.Tensor, ids: torch.Tensor, fb: ForwardBatch):
        """Routed experts under DP attention.  Each rank has routed (and, in
        decode, E5-pruned over its own batch) its T_r tokens; tokens, weights
        and expert ids are all-gathered over the EP group, padded to the
        step's agreed T_step rows per rank (padding rows carry no expert),
        every rank runs its local experts over all ranks' rows, the partial
        sums are reduce-scattered (all-reduced on gloo) and each rank keeps
        its own rows plus its replicated shared expert.  A generator that
        yields right after issuing each collective: asynchronously while two
        micro-batches interleave (forward_tbo), in place otherwise."""
        import torch.distributed as dist
        c, ps = self.cfg, self.ps
        od = self._out_dtype()
        T_r = fb.num_tokens
        T_step = max(int(fb.dp_tmax or 0), T_r)
        x = ops.to_float(h).to(od)
        w = w.float()
        from ..parallel.ep_a2a import a2a_moe_steps, a2a_ok
        if a2a_ok(x, T_step):
            # rows travel only to their experts' owners
            overlap = self._tbo_live and not (x.is_cuda and torch.cuda.is_current_stream_capturing())

            def run(xr, wr, ir):
                return ops.moe_experts(xr, wr, ir, mw.experts, out_dtype=torch.float32,
                                       n_experts_total=c.n_routed_experts)
            out = yield from a2a_moe_steps(x.contiguous(), w, ids, ps, mw.experts.count, run, overlap)
            if mw.shared_gate_up is not None:
                out = out + mw.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up), out_dtype=torch.float32).float()
            return out.to(od)
        if T_step > T_r:
            pad = T_step - T_r
            x = torch.cat([x, x.new_zeros(pad, x.shape[1])], 0)
            w = torch.cat([w, w.new_zeros(pad, w.shape[1])], 0)
            ids = torch.cat([ids, ids.new_full((pad, ids.shape[1]), -1)], 0)
        overlap = self._tbo_live and not (x.is_cuda and torch.cuda.is_current_stream_capturing())
        srcs = [x.contiguous(), w.contiguous(), ids.contiguous()]
        outs = [[torch.empty_like(t) for _ in range(ps.ep_size)] for t in srcs]
        works = [dist.all_gather(o, t, group=ps.ep_group, async_op=overlap) for o, t in zip(outs, srcs)]
        yield
        if overlap:
            for wk in works:
                wk.wait()
        g, gw, gi = (torch.cat(o, 0) for o in outs)
        part = ops.moe_experts(g, gw, gi, mw.experts, out_dtype=torch.float32, n_experts_total=c.n_routed_experts)
        if dist.get_backend(ps.ep_group) == "nccl":
            red = torch.empty(T_step, part.shape[1], dtype=part.dtype, device=part.device)
            work = dist.reduce_scatter_tensor(red, part.contiguous(), group=ps.ep_group, async_op=overlap)
        else:
            red = None
            work = dist.all_reduce(part, group=ps.ep_group, async_op=overlap)
        shared = None
        if mw.shared_gate_up is not None:
            shared = mw.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up), out_dtype=torch.float32).float()
        yield
        if overlap:
            work.wait()
        out = red[:T_r] if red is not None else part[ps.ep_rank * T_step: ps.ep_rank * T_step + T_r]
        if shared is not None:
            out = out + shared
        return out.to(od)

    def _ffn_first_linear(self, lw: V4LayerWeights):
        if isinstance(lw.ffn, DenseWeights):
            return lw.ffn.gate_up
        return lw.ffn.shared_gate_up

    def _hidden(self, fb: ForwardBatch):
        """All layers + the head combine; returns (normed hidden, batch) where
        the batch is the prefill tail's when window-only late layers ran on
        a subset of the rows."""
        return _drain(self._hidden_steps(fb))

    @torch.no_grad()
    def forward_tbo(self, fbs: List[ForwardBatch]) -> List[torch.Tensor]:
        """Two-batch overlap (DP attention prefill): the micro-batches' layer
        stacks run interleaved, each handing over right after it issues a
        collective of the MoE exchange, so one micro-batch's all-gather /
        reduce-scatter overlaps the other's kernels; collectives are issued
        in the same order on every rank.  Returns each micro-batch's logits.

        Reference parity: `_can_run_tbo` / `_forward_layers_tbo` in the V4
        layer loop (fork_loop.py:121,151-158)."""
        gens = [self._hidden_steps(fb) for fb in fbs]
        res = [None] * len(gens)
        live = list(range(len(gens)))
        self._tbo_live = True
        try:
            while live:
                for k in list(live):
                    try:
                        next(gens[k])
                    except StopIteration as e:
                        res[k] = e.value
                        live.remove(k)
        finally:
            self._tbo_live = False
        return [ops.lm_head_logits(self._last_hidden(h, fb), self.lm_head, self.ps) for h, fb in res]

    def _hidden_steps(self, fb: ForwardBatch):
        """`_hidden` as a generator: yields inside the DP MoE exchanges."""
        c = self.cfg
        eps = c.rms_norm_eps
        tr = self.tracer
        tr.reset()
        tr.mark("embed")
        X, ss = ops.hc_embed(self.embed, fb.input_ids, c.hc_mult)
        eids = None
        if c.engram_layers:
            if fb.cp is not None:
                # context parallel: a row's n-gram predecessors sit on other
                # ranks; the whole chunk's tokens go to the token cache first
                w = fb.cp.whole(fb)
                self.tok_cache[w.out_slots] = w.input_ids.to(self.tok_cache.dtype)
            eids = ops.engram_ids(fb, self.tok_cache, c, self.engram_mults, self.page_size)
        self.aux = []
        self.tail_skipped = 0
        carry = None
        for i, lw in enumerate(self.layers):
            tr.mark(f"L{i}.attn")
            tail = i == c.late_layer_start and fb.tail_from is not None
            if carry is not None and (tail or lw.engram is not None or isinstance(carry[0], _Partial)):
                # the post runs on its own where something acts on X before
                # the coefficients (or fused with the TP all-reduce)
                ss = self._post(X, *carry)
                carry = None
            if tail:
                # prefill tail: the window-only layers need only the rows within
                # reach of each prompt's end (ForwardBatch.tail_rows)
                rows = fb.tail_rows()
                self.tail_skipped = fb.num_tokens - int(rows.numel())
                X, ss = X[rows].contiguous(), ss[rows].contiguous()
                eids = eids[rows].contiguous() if eids is not None else None
                fb = fb.take_rows(rows)
            if lw.engram is not None:
                ss = ops.engram_update(X, eids, lw.engram, c, self.ps)
            # hc_post of the previous FFN + the attention coefficients + its input
            h, post, comb = ops.hc_boundary(X, carry, lw.attn_hc, lw.in_ln, eps, c, lw.attn.wqkv_a, sumsq=ss)
            if i in c.aux_layers:
                self.aux.append(ops.hc_mean(X))
            y = self._attention(i, lw, h, fb)
            carry, ss = (y, post, comb), None
            if isinstance(y, _Partial):
                ss = self._post(X, *carry)
                carry = None
            tr.mark(f"L{i}.ffn")
            moe = isinstance(lw.ffn, MoEWeights)
            h, post, comb = ops.hc_boundary(X, carry, lw.ffn_hc, lw.post_ln, eps, c, self._ffn_first_linear(lw),
                                            keep_hf=moe, sumsq=ss)
            f = yield from self._ffn_steps(i, lw, h, fb)
            carry, ss = (f, post, comb), None
        tr.mark("head")
        if isinstance(carry[0], _Partial):
            ss = self._post(X, *carry)
            carry = None
        h, _, _ = ops.hc_boundary(X, carry, self.hc_head, self.final_ln, eps, c, None, head=True, sumsq=ss)
        return h, fb

    def _last_hidden(self, h, fb: ForwardBatch) -> torch.Tensor:
        x = ops.to_float(h)
        if x.is_cuda:
            x = x.to(torch.bfloat16)
        if fb.is_decode and int(fb.last_idx.shape[0]) == int(x.shape[0]):
            return x
        return x[fb.last_idx]

    @torch.no_grad()
    def forward(self, fb: ForwardBatch) -> torch.Tensor:
        """Logits [B, V] (full vocab) of each sequence's last token."""
        h, fb = self._hidden(fb)
        return ops.lm_head_logits(self._last_hidden(h, fb), self.lm_head, self.ps)

    @torch.no_grad()
    def forward_tokens(self, fb: ForwardBatch, temperature, top_p, top_k, uniform) -> torch.Tensor:
        h, fb = self._hidden(fb)
        local = ops.lm_head_local(self._last_hidden(h, fb), self.lm_head)
        out = ops.sample_tokens(local, self.vocab_offset(), temperature, top_p, top_k, uniform, self.ps)
        self.tracer.mark("end")
        return out


# ---------------------------------------------------------------------------
# construction from a full state dict (names of models/reference_v4.py)
# ---------------------------------------------------------------------------

def host_mapped_copy(t: torch.Tensor) -> torch.Tensor:
    """Copy of a CPU tensor in device-mapped host memory."""
    from .. import _C
    buf = _C.host_mapped(t.numel() * t.element_size()).view(t.dtype).view(t.shape)
    buf.copy_(t)
    return buf


def build_model_v4(cfg: ModelConfig, ecfg: EngineConfig, ps: ParallelState, sd: Dict[str, torch.Tensor],
                   device="cpu", kv_dtype=None) -> DeepseekV4Model:
    """This rank's V4 model from a FULL (unsharded) fp32 state dict:

      model.embed_tokens.weight, model.norm.weight, lm_head.weight,
      model.hc_head.{fn, scale, base},
      model.layers.i.{attn_hc, ffn_hc}.{fn, scale, base},
      model.layers.i.{input_layernorm, post_attention_layernorm}.weight,
      model.layers.i.self_attn.{wqkv_a, wq_b, wo_a, wo_b}.weight,
        .{q_norm, kv_norm}.weight, .attn_sink,
      model.layers.i.mlp.* (DeepSeek-V3 names),
      model.layers.i.engram.{table, table_scale, wkv.weight, q_norm.weight,
        k_norm.weight}.
    """
    from .loader import _quantize, build_ffn
    assert not ecfg.dp_attention or ps.tp_size == 1, "DP attention replicates the non-expert weights (tp_size 1)"
    dev = torch.device(device)
    tp, tr = ps.tp_size, ps.tp_rank
    H, L, G, R = cfg.num_attention_heads, cfg.kv_lora_rank, cfg.o_groups, cfg.o_lora_rank
    assert H % tp == 0 and G % tp == 0 and H % G == 0
    Hl, Gl = H // tp, G // tp
    fmt_d = cfg.dense_format
    wdt = torch.bfloat16 if dev.type == "cuda" else torch.float32

    def get(name) -> torch.Tensor:
        t = sd[name]
        si = sd.get(name + "_scale_inv")
        if si is None:
            return t.float()
        from ..ops.quant import dequant_blocked
        if dev.type == "cuda":       # fp8 bytes cross the host link; dequantize on the device
            t, si = t.to(dev), si.to(dev)
        return dequant_blocked(t, si)

    def split(t, dim, n, r):
        return t.chunk(n, dim)[r].contiguous() if n > 1 else t

    def hcw(prefix) -> HcWeights:
        w = HcWeights(get(prefix + "fn").to(dev).contiguous(), get(prefix + "scale").to(dev),
                      get(prefix + "base").to(dev))
        if dev.type == "cuda":
            from ..ops.cuda import hc_fn_parts
            w.fn_parts = hc_fn_parts(w.fn)
        return w

    layers: List[V4LayerWeights] = []
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        wq_b = split(get(a + "wq_b.weight").view(H, L, -1), 0, tp, tr).reshape(Hl * L, -1)
        a_rows, b_rows = [get(a + "wqkv_a.weight")], [wq_b]
        if cfg.index_n_heads:
            ix = a + "indexer."
            a_rows += [get(ix + "wk.weight"), get(ix + "weights_proj.weight")]
            b_rows += [get(ix + "wq_b.weight")]
        if cfg.compress_ratio(i):
            a_rows += [get(a + "compressor.wgate.weight")]
        wo_a = split(get(a + "wo_a.weight").view(G, R, -1), 0, tp, tr).to(dev, wdt).contiguous()
        wo_b = split(get(a + "wo_b.weight"), 1, tp, tr)
        sink = split(get(a + "attn_sink"), 0, tp, tr).to(dev).contiguous() if cfg.attn_sink else None
        aw = V4AttnWeights(wqkv_a=Linear(_quantize(torch.cat(a_rows, 0), fmt_d, dev)),
                           q_norm=get(a + "q_norm.weight").to(dev), kv_norm=get(a + "kv_norm.weight").to(dev),
                           wq_b=Linear(_quantize(torch.cat(b_rows, 0), fmt_d, dev)), wo_a=wo_a,
                           wo_b=Linear(_quantize(wo_b, fmt_d, dev)), sink=sink)
        if cfg.index_n_heads:
            aw.ix_k_norm_w = get(a + "indexer.k_norm.weight").to(dev)
            aw.ix_k_norm_b = get(a + "indexer.k_norm.bias").to(dev)
        if cfg.compress_ratio(i):
            aw.comp_bias = get(a + "compressor.pos_bias").float().to(dev).contiguous()
        eng = None
        if i in cfg.engram_layers:
            e = p + "engram."
            table, scale = sd[e + "table"], sd[e + "table_scale"]
            rows = table.shape[0]
            lo, hi = tr * rows // tp, (tr + 1) * rows // tp
            t_sh, s_sh = table[lo:hi].contiguous(), scale[lo:hi].contiguous()
            if dev.type == "cuda":
                # host-resident tables (mapped host memory), read by the gather
                # kernel over the host link
                t_sh, s_sh = host_mapped_copy(t_sh), host_mapped_copy(s_sh)
            eng = EngramWeights(table=t_sh, scale=s_sh, row_lo=lo,
                                wkv=Linear(_quantize(get(e + "wkv.weight"), fmt_d, dev)),
                                q_w=get(e + "q_norm.weight").to(dev), k_w=get(e + "k_norm.weight").to(dev))
        layers.append(V4LayerWeights(attn_hc=hcw(p + "attn_hc."), ffn_hc=hcw(p + "ffn_hc."),
                                     in_ln=get(p + "input_layernorm.weight").to(dev),
                                     post_ln=get(p + "post_attention_layernorm.weight").to(dev), attn=aw,
                                     ffn=build_ffn(cfg, sd, get, split, p + "mlp.", i, ps, dev), engram=eng))
    emb_dt = torch.bfloat16 if dev.type == "cuda" else torch.float32
    embed = get("model.embed_tokens.weight").to(dev, emb_dt).contiguous()
    head_full = sd["model.embed_tokens.weight"] if cfg.tie_word_embeddings else sd["lm_head.weight"]
    head = split(head_full.float(), 0, tp, tr)
    head = _quantize(head, "mxfp8", dev) if fmt_d == "mxfp8" and dev.type == "cuda" else head.to(dev, emb_dt)
    if kv_dtype is None:
        kv_dtype = torch.float8_e4m3fn if dev.type == "cuda" else torch.float32
    return DeepseekV4Model(cfg, ecfg, ps, layers, embed, hcw("model.hc_head."), get("model.norm.weight").to(dev),
                           head, dev, kv_dtype=kv_dtype)
