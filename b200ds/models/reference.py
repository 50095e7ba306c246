"""fp32 oracle DeepSeek-V3(.2) decoder in plain PyTorch.

This is the numerics reference every engine path is tested against: naive
(non-absorbed) MLA that up-projects k_nope / v from the cached latent on every
call, explicit sigmoid group-limited top-k routing, per-expert loops, and the
V3.2 lightning indexer as an explicit score matrix + top-k.  It supports
tensor parallelism (heads / FFN columns split, all-reduce after row-parallel
projections; routed experts split across the same ranks with the shared
expert column-split) through :class:`~b200ds.parallel.state.ParallelState`,
so the tiny TP=2 gloo configuration can be checked against a single process.

Reference parity: the served layer loop is fork_loop.py:229-400 (attention
fork_attn.py:75-553, MoE moe_fwd.py:67-263); routing semantics follow the
fused router route_e5.cu:4-12 with V3's sigmoid scoring instead of
sqrtsoftplus.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from ..config import ModelConfig
from ..parallel.state import ParallelState
from .rope import apply_rope_ref, cos_sin_table


# ---------------------------------------------------------------------------
# Random init (HF parameter names)
# ---------------------------------------------------------------------------

def init_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02,
                 dtype=torch.float32) -> Dict[str, torch.Tensor]:
    """Full (unsharded) HF-named state dict, N(0, std) matrices, unit norms."""
    g = torch.Generator().manual_seed(seed)

    def rn(*shape):
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(dtype)

    h, H = cfg.hidden_size, cfg.num_attention_heads
    sd: Dict[str, torch.Tensor] = {"model.embed_tokens.weight": rn(cfg.vocab_size, h)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        sd[p + "input_layernorm.weight"] = torch.ones(h, dtype=dtype)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(h, dtype=dtype)
        a = p + "self_attn."
        if cfg.q_lora_rank:
            sd[a + "q_a_proj.weight"] = rn(cfg.q_lora_rank, h)
            sd[a + "q_a_layernorm.weight"] = torch.ones(cfg.q_lora_rank, dtype=dtype)
            sd[a + "q_b_proj.weight"] = rn(H * cfg.qk_head_dim, cfg.q_lora_rank)
        else:
            sd[a + "q_proj.weight"] = rn(H * cfg.qk_head_dim, h)
        sd[a + "kv_a_proj_with_mqa.weight"] = rn(cfg.kv_cache_dim, h)
        sd[a + "kv_a_layernorm.weight"] = torch.ones(cfg.kv_lora_rank, dtype=dtype)
        sd[a + "kv_b_proj.weight"] = rn(H * (cfg.qk_nope_head_dim + cfg.v_head_dim), cfg.kv_lora_rank)
        sd[a + "o_proj.weight"] = rn(h, H * cfg.v_head_dim)
        if cfg.index_n_heads:
            ix = a + "indexer."
            sd[ix + "wq_b.weight"] = rn(cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank)
            sd[ix + "wk.weight"] = rn(cfg.index_head_dim, h)
            sd[ix + "k_norm.weight"] = torch.ones(cfg.index_head_dim, dtype=dtype)
            sd[ix + "k_norm.bias"] = torch.zeros(cfg.index_head_dim, dtype=dtype)
            sd[ix + "weights_proj.weight"] = rn(cfg.index_n_heads, h)
        m = p + "mlp."
        if cfg.is_moe_layer(i):
            sd[m + "gate.weight"] = rn(cfg.n_routed_experts, h)
            sd[m + "gate.e_score_correction_bias"] = torch.zeros(cfg.n_routed_experts, dtype=dtype)
            for e in range(cfg.n_routed_experts):
                q = m + f"experts.{e}."
                sd[q + "gate_proj.weight"] = rn(cfg.moe_intermediate_size, h)
                sd[q + "up_proj.weight"] = rn(cfg.moe_intermediate_size, h)
                sd[q + "down_proj.weight"] = rn(h, cfg.moe_intermediate_size)
            if cfg.n_shared_experts:
                si = cfg.moe_intermediate_size * cfg.n_shared_experts
                q = m + "shared_experts."
                sd[q + "gate_proj.weight"] = rn(si, h)
                sd[q + "up_proj.weight"] = rn(si, h)
                sd[q + "down_proj.weight"] = rn(h, si)
        else:
            sd[m + "gate_proj.weight"] = rn(cfg.intermediate_size, h)
            sd[m + "up_proj.weight"] = rn(cfg.intermediate_size, h)
            sd[m + "down_proj.weight"] = rn(h, cfg.intermediate_size)
    sd["model.norm.weight"] = torch.ones(h, dtype=dtype)
    if not cfg.tie_word_embeddings:
        sd["lm_head.weight"] = rn(cfg.vocab_size, h)
    if cfg.num_nextn_predict_layers:
        # MTP module (HF layout: one extra decoder layer after the last, with
        # embedding / hidden norms, the [2h -> h] input projection and a head norm)
        L = cfg.num_hidden_layers
        src = init_weights(dataclasses.replace(cfg, num_hidden_layers=L + 1, num_nextn_predict_layers=0,
                                               first_k_dense_replace=min(cfg.first_k_dense_replace, L)),
                           seed + 1, std, dtype)
        m = f"model.layers.{L}."
        for k, v in src.items():
            if k.startswith(m):
                sd[k] = v
        sd[m + "enorm.weight"] = torch.ones(h, dtype=dtype)
        sd[m + "hnorm.weight"] = torch.ones(h, dtype=dtype)
        sd[m + "eh_proj.weight"] = rn(h, 2 * h)
        sd[m + "shared_head.norm.weight"] = torch.ones(h, dtype=dtype)
    return sd


# ---------------------------------------------------------------------------
# Sharding (TP for attention / dense FFN / shared expert, EP for experts)
# ---------------------------------------------------------------------------

def _split(t: torch.Tensor, dim: int, rank: int, n: int) -> torch.Tensor:
    assert t.shape[dim] % n == 0, (t.shape, dim, n)
    return t.chunk(n, dim=dim)[rank].contiguous()


def shard_state_dict(sd: Dict[str, torch.Tensor], cfg: ModelConfig, ps: ParallelState) -> Dict[str, torch.Tensor]:
    """Slice a full state dict for one rank (attention TP = ps.tp_size,
    experts EP = ps.ep_size)."""
    tp, r = ps.tp_size, ps.tp_rank
    out: Dict[str, torch.Tensor] = {}
    H = cfg.num_attention_heads
    for k, v in sd.items():
        if tp > 1 and (k.endswith("q_b_proj.weight") or k.endswith("q_proj.weight")):
            v = _split(v.view(H, cfg.qk_head_dim, -1), 0, r, tp).flatten(0, 1)
        elif tp > 1 and k.endswith("kv_b_proj.weight"):
            v = _split(v.view(H, -1, cfg.kv_lora_rank), 0, r, tp).flatten(0, 1)
        elif tp > 1 and k.endswith("o_proj.weight"):
            v = _split(v, 1, r, tp)
        elif tp > 1 and ("shared_experts" in k or (".mlp." in k and ".experts." not in k and ".gate." not in k)):
            if k.endswith("gate_proj.weight") or k.endswith("up_proj.weight"):
                v = _split(v, 0, r, tp)
            elif k.endswith("down_proj.weight"):
                v = _split(v, 1, r, tp)
        elif ".experts." in k and "shared" not in k and ps.ep_size > 1:
            e = int(k.split(".experts.")[1].split(".")[0])
            per = cfg.n_routed_experts // ps.ep_size
            if not (ps.ep_rank * per <= e < (ps.ep_rank + 1) * per):
                continue
        elif tp > 1 and k == "lm_head.weight":
            v = _split(v, 0, r, tp)
        out[k] = v
    return out


# ---------------------------------------------------------------------------
# Ops
# ---------------------------------------------------------------------------

def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()


def route_ref(logits: torch.Tensor, bias: torch.Tensor, cfg: ModelConfig):
    """Sigmoid group-limited top-k (DeepSeek-V3 noaux_tc).

    logits [T, E] fp32 -> (weights [T, k] fp32, ids [T, k] int64)."""
    scores = logits.float().sigmoid()
    choice = scores + bias.float()
    T, E = scores.shape
    if cfg.n_group > 1:
        g = choice.view(T, cfg.n_group, E // cfg.n_group)
        gscore = g.topk(2, dim=-1).values.sum(-1)                      # [T, G]
        gidx = gscore.topk(cfg.topk_group, dim=-1).indices
        gmask = torch.zeros_like(gscore).scatter_(1, gidx, 1.0)
        emask = gmask.unsqueeze(-1).expand(T, cfg.n_group, E // cfg.n_group).reshape(T, E)
        choice = choice.masked_fill(emask == 0, float("-inf"))
    ids = choice.topk(cfg.num_experts_per_tok, dim=-1).indices
    w = scores.gather(1, ids)
    if cfg.norm_topk_prob and cfg.num_experts_per_tok > 1:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return w * cfg.routed_scaling_factor, ids


# ---------------------------------------------------------------------------
# Model
# ---------------------------------------------------------------------------

class ReferenceModel:
    """fp32 DeepSeek-V3(.2) forward with a contiguous per-sequence latent cache.

    Inputs are batches of equal-length token chunks; `forward(ids [B,S],
    start_pos)` appends S tokens at positions start_pos.. to every sequence
    and returns logits [B, S, V] (full vocab on every rank)."""

    def __init__(self, cfg: ModelConfig, sd: Dict[str, torch.Tensor],
                 ps: Optional[ParallelState] = None, max_len: int = 4096):
        self.cfg = cfg
        self.ps = ps or ParallelState()
        self.w = {k: v.float() for k, v in sd.items()}
        self.max_len = max_len
        self.rope = cos_sin_table(cfg, max_len)
        self.heads = cfg.num_attention_heads // self.ps.tp_size
        self.cache: List[Dict[str, torch.Tensor]] = []
        self.batch = 0

    def reset(self, batch: int):
        c = self.cfg
        self.batch = batch
        self.cache = []
        for _ in range(c.num_hidden_layers):
            d = {"kv": torch.zeros(batch, self.max_len, c.kv_lora_rank),
                 "pe": torch.zeros(batch, self.max_len, c.qk_rope_head_dim)}
            if c.index_n_heads:
                d["ik"] = torch.zeros(batch, self.max_len, c.index_head_dim)
            self.cache.append(d)

    # -- attention --------------------------------------------------------
    def _indexer_select(self, i, x, qr, pos, start, S):
        """V3.2 lightning indexer: score[t, s] = sum_h w[t,h] relu(q[t,h].k[s]),
        keep the top index_topk causal positions. Returns bool mask [B,S,L]."""
        c, w = self.cfg, self.w
        a = f"model.layers.{i}.self_attn.indexer."
        B = x.shape[0]
        nh, hd, rd = c.index_n_heads, c.index_head_dim, c.qk_rope_head_dim
        q = (qr @ w[a + "wq_b.weight"].T).view(B, S, nh, hd)
        q = torch.cat([apply_rope_ref(q[..., :rd], pos, self.rope), q[..., rd:]], -1)
        k = F.layer_norm(x @ w[a + "wk.weight"].T, (hd,), w[a + "k_norm.weight"], w[a + "k_norm.bias"], 1e-6)
        k = torch.cat([apply_rope_ref(k[..., :rd], pos, self.rope), k[..., rd:]], -1)
        L = start + S
        self.cache[i]["ik"][:, start:L] = k
        keys = self.cache[i]["ik"][:, :L]                                   # [B, L, hd]
        hw = (x @ w[a + "weights_proj.weight"].T) * (nh ** -0.5) * (hd ** -0.5)   # [B,S,nh]
        sc = torch.einsum("bshd,bld->bshl", q, keys).relu()
        sc = (sc * hw.unsqueeze(-1)).sum(2)                                 # [B,S,L]
        causal = (torch.arange(L).view(1, L) <= (start + torch.arange(S)).view(S, 1))
        sc = sc.masked_fill(~causal, float("-inf"))
        k_eff = min(c.index_topk, L)
        idx = sc.topk(k_eff, dim=-1).indices
        sel = torch.zeros(B, S, L, dtype=torch.bool).scatter_(2, idx, True)
        return sel & causal

    def _attn(self, i: int, x: torch.Tensor, start: int) -> torch.Tensor:
        c, w = self.cfg, self.w
        a = f"model.layers.{i}.self_attn."
        B, S, _ = x.shape
        Hl = self.heads
        pos = torch.arange(start, start + S).expand(B, S)
        if c.q_lora_rank:
            qr = rms_norm(x @ w[a + "q_a_proj.weight"].T, w[a + "q_a_layernorm.weight"], c.rms_norm_eps)
            q = qr @ w[a + "q_b_proj.weight"].T
        else:
            qr = None
            q = x @ w[a + "q_proj.weight"].T
        q = q.view(B, S, Hl, c.qk_head_dim)
        q_nope, q_pe = q[..., : c.qk_nope_head_dim], q[..., c.qk_nope_head_dim:]
        q_pe = apply_rope_ref(q_pe, pos, self.rope)
        kva = x @ w[a + "kv_a_proj_with_mqa.weight"].T
        ckv = rms_norm(kva[..., : c.kv_lora_rank], w[a + "kv_a_layernorm.weight"], c.rms_norm_eps)
        kpe = apply_rope_ref(kva[..., c.kv_lora_rank:], pos, self.rope)
        L = start + S
        self.cache[i]["kv"][:, start:L] = ckv
        self.cache[i]["pe"][:, start:L] = kpe
        ckv_all = self.cache[i]["kv"][:, :L]
        kpe_all = self.cache[i]["pe"][:, :L]
        kv = (ckv_all @ w[a + "kv_b_proj.weight"].T).view(B, L, Hl, c.qk_nope_head_dim + c.v_head_dim)
        k_nope, v = kv[..., : c.qk_nope_head_dim], kv[..., c.qk_nope_head_dim:]
        scores = torch.einsum("bshd,blhd->bhsl", q_nope, k_nope)
        scores = scores + torch.einsum("bshd,bld->bhsl", q_pe, kpe_all)
        scores = scores * c.softmax_scale
        causal = (torch.arange(L).view(1, L) <= (start + torch.arange(S)).view(S, 1))
        mask = causal.view(1, 1, S, L)
        if c.index_n_heads:
            mask = mask & self._indexer_select(i, x, qr, pos, start, S).unsqueeze(1)
        scores = scores.masked_fill(~mask, float("-inf"))
        p = scores.softmax(-1)
        o = torch.einsum("bhsl,blhd->bshd", p, v).reshape(B, S, Hl * c.v_head_dim)
        out = o @ w[a + "o_proj.weight"].T
        return self.ps.tp_all_reduce(out)

    # -- ffn ----------------------------------------------------------------
    def _mlp(self, pre: str, x: torch.Tensor) -> torch.Tensor:
        w = self.w
        return (F.silu(x @ w[pre + "gate_proj.weight"].T) * (x @ w[pre + "up_proj.weight"].T)) @ w[pre + "down_proj.weight"].T

    def _moe(self, i: int, x: torch.Tensor) -> torch.Tensor:
        c, w = self.cfg, self.w
        m = f"model.layers.{i}.mlp."
        shp = x.shape
        xt = x.reshape(-1, shp[-1])
        logits = xt @ w[m + "gate.weight"].T
        wts, ids = route_ref(logits, w[m + "gate.e_score_correction_bias"], c)
        out = torch.zeros_like(xt)
        per = c.n_routed_experts // self.ps.ep_size
        lo = self.ps.ep_rank * per
        for e in range(lo, lo + per):
            hit = (ids == e)
            tok = hit.any(-1).nonzero().flatten()
            if tok.numel() == 0:
                continue
            we = (wts * hit).sum(-1)[tok].unsqueeze(-1)
            out.index_add_(0, tok, we * self._mlp(m + f"experts.{e}.", xt[tok]))
        if c.n_shared_experts:
            out = out + self._mlp(m + "shared_experts.", xt)
        # Routed experts are EP-split and the shared expert TP-split over the
        # same ranks: one all-reduce combines both.
        if self.ps.tp_size > 1 or self.ps.ep_size > 1:
            out = self.ps.tp_all_reduce(out) if self.ps.ep_size == 1 else self.ps.ep_all_reduce(out)
        return out.view(shp)

    def _ffn(self, i: int, x: torch.Tensor) -> torch.Tensor:
        if self.cfg.is_moe_layer(i):
            return self._moe(i, x)
        return self.ps.tp_all_reduce(self._mlp(f"model.layers.{i}.mlp.", x))

    # -- full forward ------------------------------------------------------------
    @torch.no_grad()
    def forward(self, ids: torch.Tensor, start: int) -> torch.Tensor:
        c, w = self.cfg, self.w
        x = w["model.embed_tokens.weight"][ids]
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            x = x + self._attn(i, rms_norm(x, w[p + "input_layernorm.weight"], c.rms_norm_eps), start)
            x = x + self._ffn(i, rms_norm(x, w[p + "post_attention_layernorm.weight"], c.rms_norm_eps))
        x = rms_norm(x, w["model.norm.weight"], c.rms_norm_eps)
        head = w["model.embed_tokens.weight"] if c.tie_word_embeddings else w["lm_head.weight"]
        logits = x @ head.T
        return self.ps.tp_all_gather(logits, dim=-1)

    @torch.no_grad()
    def greedy(self, prompts: torch.Tensor, new_tokens: int):
        """Greedy decode: returns (tokens [B, new], per-step logits list)."""
        B, S = prompts.shape
        self.reset(B)
        logits = self.forward(prompts, 0)[:, -1]
        outs, all_logits = [], [logits]
        pos = S
        for _ in range(new_tokens):
            nxt = logits.argmax(-1)
            outs.append(nxt)
            if len(outs) == new_tokens:
                break
            logits = self.forward(nxt.view(B, 1), pos)[:, -1]
            all_logits.append(logits)
            pos += 1
        return torch.stack(outs, 1), all_logits
