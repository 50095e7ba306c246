"""Production DeepSeek-V3(.2) decoder for the serving engine.

Layout per rank (one process per GPU):
  * attention: TP over heads; q_a/kv_a projections fused into one replicated
    GEMM; absorbed MLA over a paged e4m3 latent cache (kv_lora + rope per
    token, one per-layer scale); o_proj row-parallel followed by the TP
    all-reduce, fused with the residual add + next RMSNorm + MXFP8 quant;
  * dense FFN: column/row parallel, SwiGLU + requant fused into the gate_up
    GEMM epilogue, all-reduce fused as above;
  * MoE: sigmoid group-limited router, routed experts expert-parallel (each
    rank owns n_experts/ep contiguous experts), shared expert TP-split; one
    fused combine + all-reduce + residual + norm + quant per layer;
  * data-parallel attention (dp_attention): each rank runs attention for its
    own requests with all heads; the MoE boundary all-gathers tokens and
    reduce-scatters the combined result.

Reference parity: fork_loop.py:229-400 (layer loop), fork_attn.py:75-553
(attention), moe_fwd.py:67-263 (MoE), fin.py:384 (fused finalize +
all-reduce + norm + quant), epa.py:1208 (o_proj GEMM + all-reduce).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

from .. import ops
from ..config import EngineConfig, ModelConfig
from ..parallel.state import ParallelState
from ..ops.quant import MXFP8Tensor
from .batch import ForwardBatch
from .rope import cos_sin_table


def _drain(gen):
    """Run a generator to completion; returns its return value."""
    while True:
        try:
            next(gen)
        except StopIteration as e:
            return e.value


class Linear:
    """y = x W^T with W either a float tensor (tiny/CPU) or an MXFP8Tensor."""

    def __init__(self, w):
        self.w = w

    @property
    def quantized(self) -> bool:
        return isinstance(self.w, MXFP8Tensor)

    @property
    def out_features(self) -> int:
        rows = getattr(self.w, "rows", None)
        return rows if rows is not None else self.w.shape[0]

    def __call__(self, x, out_dtype=torch.bfloat16) -> torch.Tensor:
        y = ops.linear(x, self.w, out_dtype)
        n = self.out_features
        return y if y.shape[-1] == n else y[..., :n]


@dataclass
class AttnWeights:
    qkv_a: Linear                 # [q_lora + kv_lora + rope, h] (or q_proj-less variant)
    q_a_ln: Optional[torch.Tensor]
    kv_a_ln: torch.Tensor
    q_b: Linear                   # [Hl * qk_head, q_lora]
    w_uk: torch.Tensor            # [Hl, nope, kv_lora]
    w_uv: torch.Tensor            # [Hl, v, kv_lora]
    o_proj: Linear                # [h, Hl * v]
    w_uk_t: Optional[torch.Tensor] = None   # [Hl, kv_lora, nope] (GPU serving copy of w_uk)
    # Sparse indexer (optional).  Its projections ride on the attention GEMMs:
    # qkv_a has [wk (index_head_dim); weights_proj (index_n_heads)] appended
    # after the q_lora + kv rows, and q_b has the indexer's wq_b rows appended
    # after this rank's q heads, so no extra GEMM launches are needed.
    ix_k_norm_w: Optional[torch.Tensor] = None
    ix_k_norm_b: Optional[torch.Tensor] = None


@dataclass
class MoEWeights:
    gate: torch.Tensor            # [E, h] fp32 router
    bias: torch.Tensor            # [E]
    experts: "ops.ExpertWeights"  # local experts, stacked
    shared_gate_up: Optional[Linear]
    shared_down: Optional[Linear]


@dataclass
class DenseWeights:
    gate_up: Linear               # [2 * I_local, h] (gate rows then up rows)
    down: Linear                  # [h, I_local]


@dataclass
class LayerWeights:
    in_ln: torch.Tensor
    post_ln: torch.Tensor
    attn: AttnWeights
    ffn: object                   # DenseWeights | MoEWeights


class DeepseekModel:
    supports_cp = True        # context-parallel prefill under DP attention (parallel/cp.py)
    supports_tbo = True       # two-batch overlap of DP-attention prefill steps (forward_tbo)
    _tbo_live = False         # forward_tbo is interleaving micro-batches

    def __init__(self, cfg: ModelConfig, ecfg: EngineConfig, ps: ParallelState,
                 layers: List[LayerWeights], embed: torch.Tensor, final_ln: torch.Tensor,
                 lm_head: torch.Tensor, device, kv_dtype=torch.float8_e4m3fn):
        self.cfg, self.ecfg, self.ps = cfg, ecfg, ps
        self.layers = layers
        self.embed = embed
        self.final_ln = final_ln
        self.lm_head = lm_head            # [V_local, h] (vocab-parallel over TP)
        self.device = torch.device(device)
        self.kv_dtype = kv_dtype
        attn_tp = 1 if ecfg.dp_attention else ps.tp_size
        self.attn_tp = attn_tp
        self.heads = cfg.num_attention_heads // attn_tp
        self.rope_table = cos_sin_table(cfg, cfg.max_position_embeddings, device=self.device)
        self.kv_scale = [1.0] * len(layers)
        self.kv_cache: List[torch.Tensor] = []
        self.ix_cache: List[torch.Tensor] = []
        self.ix_scale: List[torch.Tensor] = []
        self.page_size = ecfg.page_size
        from ..utils.trace import null_tracer
        self.tracer = null_tracer()       # the engine installs a Tracer when tracing is on
        self.mtp = None                   # MTP draft module (models/mtp.py), attached by the loader
        self.last_residual = None
        if self.device.type == "cuda":
            for lw in layers:       # [H, L, nope] copy of W_uk for the tensor-core absorption
                w = lw.attn.w_uk
                if w.dtype == torch.bfloat16 and getattr(lw.attn, "w_uk_t", None) is None:
                    lw.attn.w_uk_t = w.transpose(1, 2).contiguous()
        # DP attention: each rank serves its own requests with replicated
        # attention / dense / shared-expert / LM-head weights (tp_size 1);
        # only the routed experts are split (EP) and exchanged at the MoE
        # boundary.  ps_local is the single-rank view for local reductions.
        assert cfg.late_layer_start is None, "window-only late layers are a DeepSeek-V4-family option"
        self.dp = bool(ecfg.dp_attention) and ps.ep_size > 1
        self.ps_local = ParallelState(device=self.device) if self.dp else ps
        from ..utils import levers
        fused_comm = ecfg.comm_impl == "fused" and levers.on("fused_comm")
        if (self.device.type == "cuda" and ps.tp_size > 1 and fused_comm
                and getattr(ps, "fused_ar", None) is None):
            from ..parallel.symm import FusedAllReduce
            ps.fused_ar = FusedAllReduce(ps, cfg.hidden_size, max_tokens=max(ecfg.max_num_seqs, 256))
        if (self.device.type == "cuda" and self.dp and fused_comm and cfg.n_routed_experts
                and getattr(ps, "fused_ep", None) is None):
            from ..parallel.symm import EPDispatch, FusedAllReduce
            cap = max(ecfg.max_num_seqs, 256)
            ps.fused_ar = FusedAllReduce(ps, cfg.hidden_size, max_tokens=cap, group="ep",
                                         topk=cfg.num_experts_per_tok)
            ps.fused_ep = EPDispatch(ps, cfg.hidden_size, cfg.num_experts_per_tok, cap)

    # ------------------------------------------------------------------
    def allocate_kv(self, num_pages: int):
        c = self.cfg
        slots = num_pages * self.page_size
        self.kv_cache = [torch.zeros(slots, c.kv_cache_dim, dtype=self.kv_dtype, device=self.device)
                         for _ in self.layers]
        if c.index_n_heads:
            idt = self.kv_dtype
            self.ix_cache = [torch.zeros(slots, c.index_head_dim, dtype=idt, device=self.device)
                             for _ in self.layers]
            self.ix_scale = [torch.ones(slots, dtype=torch.float32, device=self.device)
                             for _ in self.layers]

    def kv_tensors(self) -> List[torch.Tensor]:
        """Every per-slot cache tensor ([slots, ...], slot = page * page_size +
        offset): what one KV page holds across the model."""
        out = list(self.kv_cache)
        out += list(getattr(self, "ix_cache", []) or []) + list(getattr(self, "ix_scale", []) or [])
        return out

    def kv_bytes_per_token(self) -> int:
        c = self.cfg
        per = c.kv_cache_dim * torch.tensor([], dtype=self.kv_dtype).element_size()
        if c.index_n_heads:
            per += c.index_head_dim * torch.tensor([], dtype=self.kv_dtype).element_size() + 4
        return per * len(self.layers)

    # ------------------------------------------------------------------
    def _attention(self, i: int, lw: LayerWeights, h, fb: ForwardBatch) -> torch.Tensor:
        c = self.cfg
        aw = lw.attn
        T = fb.num_tokens
        qkv = aw.qkv_a(h, out_dtype=torch.float32 if self.device.type == "cpu" else torch.bfloat16)
        ql = c.q_lora_rank
        q_lat = ops.rmsnorm_act(qkv[:, :ql], aw.q_a_ln, c.rms_norm_eps, aw.q_b,
                                keep_hf=bool(c.index_n_heads))
        ops.kv_store(qkv[:, ql:ql + c.kv_cache_dim], aw.kv_a_ln, c.rms_norm_eps, self.rope_table, fb.positions,
                     self.kv_cache[i], fb.out_slots, self.kv_scale[i], c.kv_lora_rank)
        if fb.cp is not None and not c.index_n_heads:
            self._cp_gather(i, fb)
        qo = aw.q_b(q_lat, out_dtype=torch.float32 if self.device.type == "cpu" else torch.bfloat16)
        q = qo[:, : self.heads * c.qk_head_dim].view(T, self.heads, c.qk_head_dim)
        topk = None
        if c.index_n_heads:
            topk = self._indexer(i, aw, qkv, qo, fb)
        # weights the layer streams after attention go to L2 meanwhile
        self._prefetch(i, lw, fb)
        # absorption of q_nope into the latent space, RoPE of the (un-rotated)
        # rope part and the e4m3 query prep run fused ahead of the attention
        o_lat = ops.mla_from_q(q[..., : c.qk_nope_head_dim], q[..., c.qk_nope_head_dim:], aw.w_uk,
                               getattr(aw, "w_uk_t", None), self.kv_cache[i], self.kv_scale[i], fb,
                               c.softmax_scale, self.page_size, topk, self.rope_table)
        self._prefetch_join()
        o = ops.absorb_o(o_lat, aw.w_uv, quantize=aw.o_proj.quantized)   # [T, Hl*v] (MXFP8 when quantized)
        if self.device.type == "cuda" and self.attn_tp > 1:
            # leave the o_proj GEMM to the all-reduce so it can run fused
            return ops.PendingLinear(o, aw.o_proj.w, aw.o_proj.out_features)
        return aw.o_proj(o, out_dtype=torch.float32 if self.device.type == "cpu" else torch.bfloat16)

    def _indexer(self, i, aw: AttnWeights, qkv, qo, fb: ForwardBatch):
        """Lightning indexer: keys from the qkv_a GEMM's appended rows, queries
        from q_b's appended rows; returns top-k cache positions [T, topk]."""
        c = self.cfg
        nh, hd = c.index_n_heads, c.index_head_dim
        base = c.q_lora_rank + c.kv_cache_dim
        k_raw = qkv[:, base: base + hd]
        w_raw = qkv[:, base + hd: base + hd + nh]
        q_raw = qo[:, self.heads * c.qk_head_dim: self.heads * c.qk_head_dim + nh * hd]
        ops.index_k_store(k_raw, aw.ix_k_norm_w, aw.ix_k_norm_b, 1e-6, self.rope_table, fb.positions,
                          self.ix_cache[i], self.ix_scale[i], fb.out_slots)
        if fb.cp is not None:
            self._cp_gather(i, fb)
        return ops.indexer_topk(q_raw, w_raw, (nh * hd) ** -0.5, self.rope_table, self.ix_cache[i],
                                self.ix_scale[i], fb, self.page_size, c.index_topk, c.index_swa)

    def _cp_gather(self, i: int, fb: ForwardBatch) -> None:
        """Context-parallel chunk: every rank's new cache rows of layer i
        (latent + rope, and the indexer key + scale of sparse models) into
        this rank's cache before any query of the chunk attends."""
        from ..parallel.cp import gather_rows
        bufs = [self.kv_cache[i]]
        if self.cfg.index_n_heads:
            bufs += [self.ix_cache[i], self.ix_scale[i]]
        gather_rows(bufs, fb, self.ps)

    def _ffn(self, i: int, lw: LayerWeights, h, fb: ForwardBatch) -> torch.Tensor:
        c = self.cfg
        out_dt = torch.float32 if self.device.type == "cpu" else torch.bfloat16
        fuse = self.device.type == "cuda" and self.ps.tp_size > 1
        if isinstance(lw.ffn, DenseWeights):
            a = ops.gate_up_swiglu(h, lw.ffn.gate_up)
            if fuse:
                return ops.PendingLinear(a, lw.ffn.down.w, lw.ffn.down.out_features)
            return lw.ffn.down(a, out_dtype=out_dt)
        mw: MoEWeights = lw.ffn
        if self.dp:
            return self._moe_dp(mw, h, fb)
        w, ids = ops.router(h, mw.gate, mw.bias, c)
        if fuse and ops.get_impl() == "native":
            # The shared expert is independent of the routed experts: run it on
            # a side stream (a parallel branch of the captured graph) while the
            # routing + grouped GEMMs run on the main stream.
            shared = None
            if mw.shared_gate_up is not None:
                shared = self._fork(lambda: lw.ffn.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up),
                                                               out_dtype=out_dt), h)
            part = ops.moe_experts(h, w, ids, mw.experts, out_dtype=out_dt, n_experts_total=c.n_routed_experts,
                                   combine=False)
            if shared is not None:
                part.add = self._join(shared)
            return part
        out = ops.moe_experts(h, w, ids, mw.experts, out_dtype=out_dt, n_experts_total=c.n_routed_experts)
        if mw.shared_gate_up is not None:
            s = lw.ffn.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up), out_dtype=out_dt)
            out = out + s
        return out

    def _moe_dp_fused_ok(self, fb: ForwardBatch) -> bool:
        """Whether this step's MoE exchange fits the symmetric-memory fused
        path (native kernels, rows per rank within the dispatch buffers)."""
        ps = self.ps
        T_step = max(int(fb.dp_tmax or 0), fb.num_tokens)
        ep, far = getattr(ps, "fused_ep", None), getattr(ps, "fused_ar", None)
        return (self.device.type == "cuda" and ops.get_impl() == "native" and ep is not None and ep.supports(T_step)
                and far is not None and far.supports(T_step))

    def _moe_dp(self, mw: MoEWeights, h, fb: ForwardBatch):
        """MoE under DP attention: this rank's T_r tokens (padded to the
        step's agreed T_step rows per rank) meet the routed experts of every
        rank.  Fused path: router on the local tokens, P2P dispatch to the
        expert owners, grouped GEMMs over the received tokens, and the
        combine + reduce-scatter fused into the next norm.  Host-collective
        path (CPU, baseline ops, steps larger than the symmetric buffers):
        `_moe_dp_host`."""
        c, ps = self.cfg, self.ps
        if self._moe_dp_fused_ok(fb):
            T_step = max(int(fb.dp_tmax or 0), fb.num_tokens)
            out_dt = torch.bfloat16
            shared = None
            if mw.shared_gate_up is not None:
                shared = self._fork(lambda: mw.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up),
                                                           out_dtype=out_dt), h)
            w, ids = ops.router(h, mw.gate, mw.bias, c)
            part = ops.moe_experts_ep(h, w, ids, mw.experts, T_step, c.n_routed_experts, ps.fused_ep, ps.fused_ar)
            if shared is not None:
                part.add = self._join(shared)
            return part
        return _drain(self._moe_dp_host(mw, h, fb))

    def _moe_dp_host(self, mw: MoEWeights, h, fb: ForwardBatch):
        """Host-collective MoE under DP attention, as a generator that yields
        right after issuing each collective (asynchronously while two-batch
        overlap interleaves micro-batches).  Large steps: the all-to-all
        exchange (parallel/ep_a2a.py: rows only to their experts' owners,
        partial sums back).  Smaller ones: all-gather of every rank's rows,
        this rank's experts over all of them, then a reduce-scatter (NCCL;
        all-reduce + own slice on gloo) back to the owners.  The shared
        expert runs during the reduction."""
        import torch.distributed as dist
        c, ps = self.cfg, self.ps
        T_r = fb.num_tokens
        T_step = max(int(fb.dp_tmax or 0), T_r)
        out_dt = torch.float32 if self.device.type == "cpu" else torch.bfloat16
        x = ops.to_float(h)
        # asynchronous only while two micro-batches interleave (never inside a
        # graph capture); otherwise the collectives complete in place
        overlap = self._tbo_live and not (x.is_cuda and torch.cuda.is_current_stream_capturing())
        from ..parallel.ep_a2a import a2a_moe_steps, a2a_ok
        if a2a_ok(x, T_step):
            # rows travel only to their experts' owners (router on the local rows)
            w, ids = ops.router(h, mw.gate, mw.bias, c)

            def run(xr, wr, ir):
                return ops.moe_experts(xr, wr, ir, mw.experts, out_dtype=torch.float32,
                                       n_experts_total=c.n_routed_experts)
            out = yield from a2a_moe_steps(x.to(out_dt).contiguous(), w, ids, ps, mw.experts.count, run, overlap)
            if mw.shared_gate_up is not None:
                out = out + mw.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up), out_dtype=torch.float32).float()
            return out.to(out_dt)
        if T_step > T_r:
            x = torch.cat([x, x.new_zeros(T_step - T_r, x.shape[1])], 0)
        x = x.to(out_dt).contiguous()
        parts = [torch.empty_like(x) for _ in range(ps.ep_size)]
        work = dist.all_gather(parts, x, group=ps.ep_group, async_op=overlap)
        yield
        if overlap:
            work.wait()
        g = torch.cat(parts, 0)
        w, ids = ops.router(g, mw.gate, mw.bias, c)
        part = ops.moe_experts(g, w, ids, mw.experts, out_dtype=torch.float32, n_experts_total=c.n_routed_experts)
        if dist.get_backend(ps.ep_group) == "nccl":
            out = torch.empty(T_step, part.shape[1], dtype=part.dtype, device=part.device)
            work = dist.reduce_scatter_tensor(out, part.contiguous(), group=ps.ep_group, async_op=overlap)
        else:
            out = None
            work = dist.all_reduce(part, group=ps.ep_group, async_op=overlap)
        shared = None
        if mw.shared_gate_up is not None:
            shared = mw.shared_down(ops.gate_up_swiglu(h, mw.shared_gate_up), out_dtype=torch.float32).float()
        yield
        if overlap:
            work.wait()
        out = out[:T_r] if out is not None else part[ps.ep_rank * T_step: ps.ep_rank * T_step + T_r]
        if shared is not None:
            out = out + shared
        return out.to(out_dt)

    # ------------------------------------------------------------------
    L2_PREFETCH_LIMIT = 24 << 20        # bytes per region (L2 is 126 MB; attention reads the KV meanwhile)

    def _prefetch(self, i: int, lw, fb) -> None:
        """Decode steps: issue L2 prefetches of the o-projection weights and
        (MoE layers) the shared expert's gate_up on a low-priority side stream
        that runs next to the attention kernels; `_prefetch_join` rejoins it
        before the o-projection.  The reference warms WO-A / wo_b / the router
        the same way (l2pf.py:4-5, l2pf_unit.cu:22,33)."""
        self._pf_live = False
        if not (self.device.type == "cuda" and fb.is_decode and ops.get_impl() == "native"):
            return
        from ..utils import levers
        if not levers.on("l2_prefetch"):
            return
        ts = []
        for lin in (lw.attn.o_proj, getattr(lw.ffn, "shared_gate_up", None)):
            w = getattr(lin, "w", lin)
            data = getattr(w, "data", None)
            if isinstance(data, torch.Tensor) and data.is_cuda and data.is_contiguous():
                ts.append(data.view(torch.uint8))
        if not ts:
            return
        from .. import _C
        main = torch.cuda.current_stream(self.device)
        if getattr(self, "_pf", None) is None:
            self._pf = torch.cuda.Stream(device=self.device, priority=0)     # lowest priority
        self._pf.wait_stream(main)
        with torch.cuda.stream(self._pf):
            _C.l2_prefetch(ts, self.L2_PREFETCH_LIMIT, 32)
        self._pf_live = True

    def _prefetch_join(self) -> None:
        if getattr(self, "_pf_live", False):
            torch.cuda.current_stream(self.device).wait_stream(self._pf)
            self._pf_live = False

    def _fork(self, fn, *inputs):
        """Run fn() on the side stream after the main stream's pending work;
        returns a handle for `_join`."""
        main = torch.cuda.current_stream(self.device)
        if getattr(self, "_side", None) is None:
            # highest priority: the shared expert is short and joins the MoE
            # combine, so its kernels go ahead of the routed experts' CTAs
            self._side = torch.cuda.Stream(device=self.device, priority=-5)
        side = self._side
        side.wait_stream(main)
        with torch.cuda.stream(side):
            out = fn()
        for t in inputs:
            for x in ((t.q, t.sf, t.hf) if isinstance(t, ops.QAct) else (t,)):
                if isinstance(x, torch.Tensor):
                    x.record_stream(side)
        return out

    def _join(self, out):
        main = torch.cuda.current_stream(self.device)
        main.wait_stream(self._side)
        out.record_stream(main)
        return out

    @torch.no_grad()
    def forward(self, fb: ForwardBatch, x0: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Returns logits [B, V] (full vocab) for each sequence's last token."""
        h = self._hidden(fb, x0)
        return ops.lm_head_logits(self._last_hidden(h, fb), self.lm_head, self.ps)

    def _hidden(self, fb: ForwardBatch, x0: Optional[torch.Tensor] = None):
        """All decoder layers + the final norm; returns the normed hidden.
        x0: the initial residual stream instead of the token embeddings (the
        MTP module).  The pre-norm final residual of every row is kept in
        `last_residual` (the speculative draft's input)."""
        return _drain(self._hidden_steps(fb, x0))

    @torch.no_grad()
    def forward_tbo(self, fbs: List[ForwardBatch]) -> List[torch.Tensor]:
        """Two-batch overlap (DP attention prefill): the micro-batches in
        `fbs` run the layer stack interleaved, each handing over to the next
        right after it issues a collective of the host-collective MoE
        exchange, so one micro-batch's all-gather / reduce-scatter runs
        (NCCL's stream, asynchronously) while the other computes.  Each
        micro-batch's collectives are issued in the same order on every rank.
        Returns the logits of each micro-batch's sequences.

        Reference parity: SGLang's two-batch overlap for expert-parallel
        batches (`_can_run_tbo`, `_forward_layers_tbo`, fork_loop.py:121,
        151-158)."""
        gens = [self._hidden_steps(fb) for fb in fbs]
        hs = [None] * len(gens)
        live = list(range(len(gens)))
        self._tbo_live = True
        try:
            while live:
                for k in list(live):
                    try:
                        next(gens[k])
                    except StopIteration as e:
                        hs[k] = e.value
                        live.remove(k)
        finally:
            self._tbo_live = False
        return [ops.lm_head_logits(self._last_hidden(h, fb), self.lm_head, self.ps) for h, fb in zip(hs, fbs)]

    def _hidden_steps(self, fb: ForwardBatch, x0: Optional[torch.Tensor] = None):
        """`_hidden` as a generator: yields after each asynchronous collective
        of a host-collective MoE exchange (none on the fused paths)."""
        c = self.cfg
        tr = self.tracer
        tr.reset()
        tr.mark("embed")
        residual = (self.embed[fb.input_ids.long()].float() if x0 is None
                    else x0.float().contiguous())                  # fp32 residual stream
        h = ops.rmsnorm_act(residual, self.layers[0].in_ln, c.rms_norm_eps, self.layers[0].attn.qkv_a)
        for i, lw in enumerate(self.layers):
            tr.mark(f"L{i}.attn")
            a = self._attention(i, lw, h, fb)
            h, residual = ops.allreduce_add_rmsnorm(a, residual, lw.post_ln, c.rms_norm_eps,
                                                    self.ps, "tp_attn", self._ffn_first_linear(lw))
            tr.mark(f"L{i}.ffn")
            if self.dp and isinstance(lw.ffn, MoEWeights) and not self._moe_dp_fused_ok(fb):
                f = yield from self._moe_dp_host(lw.ffn, h, fb)
            else:
                f = self._ffn(i, lw, h, fb)
            nxt = self.layers[i + 1] if i + 1 < len(self.layers) else None
            # under DP attention only the fused expert-parallel partial still
            # needs a collective; every other FFN output is already this rank's
            ps_f = self.ps if (not self.dp or isinstance(f, ops.EPPartial)) else self.ps_local
            h, residual = ops.allreduce_add_rmsnorm(
                f, residual, nxt.in_ln if nxt else self.final_ln, c.rms_norm_eps, ps_f,
                "ffn", nxt.attn.qkv_a if nxt else None)
        tr.mark("head")
        self.last_residual = residual
        return h

    def _last_hidden(self, h, fb: ForwardBatch) -> torch.Tensor:
        x = ops.to_float(h)
        if x.is_cuda:
            x = x.to(torch.bfloat16)
        if fb.is_decode and int(fb.last_idx.shape[0]) == int(x.shape[0]):
            return x                 # decode: every token is its sequence's last
        return x[fb.last_idx]

    def vocab_offset(self) -> int:
        rows = getattr(self.lm_head, "rows", None)
        n = rows if rows is not None else self.lm_head.shape[0]
        return self.ps.tp_rank * n

    @torch.no_grad()
    def forward_tokens(self, fb: ForwardBatch, temperature, top_p, top_k, uniform) -> torch.Tensor:
        """Forward + sampling without materialising the full-vocabulary
        logits: returns token ids [B] (greedy for rows with temperature <= 0)."""
        h = self._hidden(fb)
        local = ops.lm_head_local(self._last_hidden(h, fb), self.lm_head)
        out = ops.sample_tokens(local, self.vocab_offset(), temperature, top_p, top_k, uniform, self.ps)
        self.tracer.mark("end")
        return out

    def _ffn_first_linear(self, lw: LayerWeights):
        if isinstance(lw.ffn, DenseWeights):
            return lw.ffn.gate_up
        return lw.ffn.shared_gate_up
