"""fp32 oracle for the DeepSeek-V4 family (arch="deepseek_v4").

Plain PyTorch, one process, contiguous per-sequence caches: the numerics
reference the engine's V4 model (models/deepseek_v4.py) is tested against.

Architecture (per layer, hc residual streams X [hc, D] per token):
  * each sublayer (attention, then FFN) reads coefficients from its input
    streams: raw = X_flat . fn^T, r = rsqrt(mean(X_flat^2) + eps);
    pre = sigmoid(a0 r raw[:hc] + b), post = 2 sigmoid(a1 r raw[hc:2hc] + b),
    comb = Sinkhorn(a2 r raw[2hc:] + b) (hc x hc);
    the sublayer input is RMSNorm(sum_c pre_c X_c) and the streams become
    X'_c = post_c * y + sum_r comb[r][c] X_r;
  * attention is MQA over one latent row per token: kv = RMSNorm(wqkv_a x
    [q_lora:]) with RoPE on its last rope dims is both key and value; queries
    q = wq_b RMSNorm(wqkv_a x [:q_lora]) per head (RoPE on the same tail);
    softmax with a per-head sink logit in the denominator; the output's rope
    tail is rotated back to position 0; o -> wo_a per head group (low rank)
    -> wo_b;
  * MoE: sqrt(softplus) scores, top-k by score + bias, weights renormalised
    and scaled; at decode the E5 prune drops lightly-used experts;
  * Engram layers first add gated n-gram memory rows to every stream;
  * the head combines the streams with its own sigmoid pre weights, then the
    final RMSNorm and the LM head.

Reference parity: hq_layer.py:32-101 and fg_layer.py (sublayer hyper-
connections), fin.py:218-246 (post), sk_unit.cu:1-15 (coefficients),
fork_attn.py:380-553 (MQA with sinks, inverse rope, wo_a groups, wo_b),
route_e5.cu:4-12 (routing + E5), eg.py:355-390 (Engram), fork_loop.py:195-210
(hc head).  The reference serves the private DeepSeek-V4.1-Flash; the parts
it only calls into (Engram gate, hash) follow our formulation, stated in
ops/ref.py.
"""
from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from ..config import ModelConfig
from ..ops import ref
from .rope import cos_sin_table


def _e4m3_bytes(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-448, 448).to(torch.float8_e4m3fn).view(torch.uint8)


def init_weights_v4(cfg: ModelConfig, seed: int = 0, std: float = 0.02) -> Dict[str, torch.Tensor]:
    """Full (unsharded) fp32 state dict of a V4-family model (our parameter
    names, listed in models/deepseek_v4.py::build_model_v4)."""
    assert cfg.is_v4 and cfg.hc_mult > 0
    g = torch.Generator().manual_seed(seed)

    def rn(*shape, s=std):
        return torch.randn(*shape, generator=g, dtype=torch.float32) * s

    h, H, hc = cfg.hidden_size, cfg.num_attention_heads, cfg.hc_mult
    L, R, G = cfg.kv_lora_rank, cfg.o_lora_rank, cfg.o_groups
    M = (2 + hc) * hc

    def hc_params(prefix, m):
        sd[prefix + "fn"] = rn(m, hc * h, s=std)
        sd[prefix + "scale"] = torch.ones(3 if m > hc else 1)
        base = torch.zeros(m)
        if m > hc:
            base[2 * hc:] = (torch.eye(hc) * 4.0).flatten()       # comb starts near the identity
        sd[prefix + "base"] = base

    sd: Dict[str, torch.Tensor] = {"model.embed_tokens.weight": rn(cfg.vocab_size, h)}
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        hc_params(p + "attn_hc.", M)
        hc_params(p + "ffn_hc.", M)
        sd[p + "input_layernorm.weight"] = torch.ones(h)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(h)
        a = p + "self_attn."
        sd[a + "wqkv_a.weight"] = rn(cfg.q_lora_rank + L, h)
        sd[a + "q_norm.weight"] = torch.ones(cfg.q_lora_rank)
        sd[a + "kv_norm.weight"] = torch.ones(L)
        sd[a + "wq_b.weight"] = rn(H * L, cfg.q_lora_rank)
        sd[a + "wo_a.weight"] = rn(G * R, (H // G) * L)
        sd[a + "wo_b.weight"] = rn(h, G * R)
        if cfg.attn_sink:
            sd[a + "attn_sink"] = rn(H, s=1.0)
        if cfg.index_n_heads:
            ix = a + "indexer."
            sd[ix + "wq_b.weight"] = rn(cfg.index_n_heads * cfg.index_head_dim, cfg.q_lora_rank)
            sd[ix + "wk.weight"] = rn(cfg.index_head_dim, h)
            sd[ix + "k_norm.weight"] = torch.ones(cfg.index_head_dim)
            sd[ix + "k_norm.bias"] = torch.zeros(cfg.index_head_dim)
            sd[ix + "weights_proj.weight"] = rn(cfg.index_n_heads, h)
        r = cfg.compress_ratio(i)
        if r:
            sd[a + "compressor.wgate.weight"] = rn(1, h)
            sd[a + "compressor.pos_bias"] = rn(r, s=0.5)
        m = p + "mlp."
        if cfg.is_moe_layer(i):
            sd[m + "gate.weight"] = rn(cfg.n_routed_experts, h)
            sd[m + "gate.e_score_correction_bias"] = rn(cfg.n_routed_experts, s=0.01)
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
        if i in cfg.engram_layers:
            e = p + "engram."
            d = cfg.engram_dim
            sd[e + "table"] = _e4m3_bytes(rn(cfg.engram_rows, d, s=1.0))
            sd[e + "table_scale"] = torch.full((cfg.engram_rows, d // 32), 127 - 4, dtype=torch.uint8)
            sd[e + "wkv.weight"] = rn(2 * h, cfg.engram_heads * d)
            sd[e + "q_norm.weight"] = torch.ones(h)
            sd[e + "k_norm.weight"] = torch.ones(h)
    hc_params("model.hc_head.", hc)
    sd["model.norm.weight"] = torch.ones(h)
    if not cfg.tie_word_embeddings:
        sd["lm_head.weight"] = rn(cfg.vocab_size, h)
    return sd


def engram_context(tokens: torch.Tensor, n: int) -> torch.Tensor:
    """tokens [S] of one sequence -> [S, n]: column i holds the token at
    position p - i (-1 before the sequence start)."""
    S = tokens.shape[0]
    out = torch.full((S, n), -1, dtype=torch.int64)
    for i in range(n):
        if i < S:
            out[i:, i] = tokens[: S - i].long()
    return out


class ReferenceV4Model:
    """`forward(ids [B, S], start)` appends S tokens to every sequence and
    returns logits [B, S, V]; `decode=True` marks a decode step (E5 prune)."""

    def __init__(self, cfg: ModelConfig, sd: Dict[str, torch.Tensor], max_len: int = 4096):
        self.cfg = cfg
        self.w = {k: (v.float() if v.dtype != torch.uint8 else v) for k, v in sd.items()}
        self.max_len = max_len
        self.rope = cos_sin_table(cfg, max_len)
        self.cache: List[torch.Tensor] = []
        self.tokens: Optional[torch.Tensor] = None
        self.aux: List[torch.Tensor] = []

    def reset(self, batch: int):
        c = self.cfg
        self.cache = [torch.zeros(batch, self.max_len, c.kv_lora_rank) for _ in range(c.num_hidden_layers)]
        self.ik = [torch.zeros(batch, self.max_len, c.index_head_dim) for _ in range(c.num_hidden_layers)]
        self.gate = [torch.zeros(batch, self.max_len) for _ in range(c.num_hidden_layers)]
        self.tokens = torch.full((batch, self.max_len), -1, dtype=torch.int64)

    # -- mHC ------------------------------------------------------------------
    def _coeffs(self, prefix: str, X: torch.Tensor):
        c, w = self.cfg, self.w
        raw, sq = ref.hc_stats(X, w[prefix + "fn"])
        return ref.hc_coeffs(raw, sq, w[prefix + "scale"], w[prefix + "base"], c.hc_mult,
                             c.hc_mult * c.hidden_size, c.hc_sinkhorn_iters, c.hc_eps)

    # -- attention --------------------------------------------------------------
    def _attn(self, i: int, x: torch.Tensor, start: int) -> torch.Tensor:
        c, w = self.cfg, self.w
        a = f"model.layers.{i}.self_attn."
        B, S, _ = x.shape
        H, L, rd = c.num_attention_heads, c.kv_lora_rank, c.qk_rope_head_dim
        pos = torch.arange(start, start + S)
        qkv = x @ w[a + "wqkv_a.weight"].T
        qr = ref.rmsnorm(qkv[..., : c.q_lora_rank], w[a + "q_norm.weight"], c.rms_norm_eps)
        q = (qr @ w[a + "wq_b.weight"].T).view(B, S, H, L)
        kv = ref.rmsnorm(qkv[..., c.q_lora_rank:], w[a + "kv_norm.weight"], c.rms_norm_eps)
        kv = torch.cat([kv[..., :-rd], ref.rope(kv[..., -rd:].reshape(B * S, rd), pos.repeat(B), self.rope)
                        .view(B, S, rd)], -1)
        q = torch.cat([q[..., :-rd], ref.rope(q[..., -rd:].reshape(B * S, H, rd), pos.repeat(B), self.rope)
                       .view(B, S, H, rd)], -1)
        end = start + S
        self.cache[i][:, start:end] = kv
        keys = self.cache[i][:, :end]                                          # [B, end, L]
        if c.compress_ratio(i):
            o = self._compressed_attn(i, x, qr, q, keys, pos, start, S)
            return self._attn_out(i, o, pos)
        s = torch.einsum("bshd,bld->bhsl", q, keys) * c.softmax_scale
        causal = torch.arange(end).view(1, end) <= (start + torch.arange(S)).view(S, 1)
        mask = causal.view(1, 1, S, end)
        if c.is_window_layer(i):          # window-only late layer: the last late_window positions
            win = torch.arange(end).view(1, end) > (start + torch.arange(S)).view(S, 1) - c.late_window
            mask = mask & win.view(1, 1, S, end)
        elif c.index_n_heads:
            mask = mask & self._indexer_select(i, x, qr, pos, start, S).unsqueeze(1)
        s = s.masked_fill(~mask, float("-inf"))
        if c.attn_sink:
            sink = w[a + "attn_sink"].view(1, H, 1, 1).expand(B, H, S, 1)
            p = torch.cat([s, sink], -1).softmax(-1)[..., :-1]
        else:
            p = s.softmax(-1)
        o = torch.einsum("bhsl,bld->bshd", p, keys)                          # [B, S, H, L]
        return self._attn_out(i, o, pos)

    def _attn_out(self, i: int, o: torch.Tensor, pos: torch.Tensor) -> torch.Tensor:
        """Inverse RoPE of the output tails, grouped wo_a, wo_b."""
        c, w = self.cfg, self.w
        a = f"model.layers.{i}.self_attn."
        B, S, H, L = o.shape
        rd = c.qk_rope_head_dim
        o = ref.inv_rope_tail(o.reshape(B * S, H, L), pos.repeat(B), self.rope, rd).view(B, S, H, L)
        G, R = c.o_groups, c.o_lora_rank
        og = o.reshape(B, S, G, (H // G) * L)
        wa = w[a + "wo_a.weight"].view(G, R, (H // G) * L)
        z = torch.einsum("bsgk,grk->bsgr", og, wa).reshape(B, S, G * R)
        return z @ w[a + "wo_b.weight"].T

    def _compressed_attn(self, i, x, qr, q, keys, pos, start, S):
        """Compressed sparse attention of layer i (ratio r): every query
        attends to its window (the last index_swa positions) plus the
        compress_topk compressed blocks before the window with the highest
        indexer scores; a block's row is the gated mean of its r KV rows
        (softmax over the block of wgate . x + pos_bias), its indexer key
        the same mean of the r indexer keys.  Returns o [B, S, H, L]."""
        import torch.nn.functional as F
        from .rope import apply_rope_ref
        c, w = self.cfg, self.w
        a = f"model.layers.{i}.self_attn."
        B, end = keys.shape[0], start + S
        r, swa = c.compress_ratio(i), c.index_swa
        H, L = c.num_attention_heads, c.kv_lora_rank
        nh, hd, rd = c.index_n_heads, c.index_head_dim, c.qk_rope_head_dim
        # gates, indexer queries / keys / head weights
        self.gate[i][:, start:end] = (x @ w[a + "compressor.wgate.weight"].T)[..., 0]
        ix = a + "indexer."
        qi = (qr @ w[ix + "wq_b.weight"].T).view(B, S, nh, hd)
        qi = torch.cat([apply_rope_ref(qi[..., :rd], pos.expand(B, S), self.rope), qi[..., rd:]], -1)
        k = F.layer_norm(x @ w[ix + "wk.weight"].T, (hd,), w[ix + "k_norm.weight"], w[ix + "k_norm.bias"], 1e-6)
        k = torch.cat([apply_rope_ref(k[..., :rd], pos.expand(B, S), self.rope), k[..., rd:]], -1)
        self.ik[i][:, start:end] = k
        hw = (x @ w[ix + "weights_proj.weight"].T) * (nh ** -0.5) * (hd ** -0.5)
        # compressed rows of the complete blocks
        nb = end // r
        g = self.gate[i][:, :nb * r].view(B, nb, r) + w[a + "compressor.pos_bias"].view(1, 1, r)
        wt = torch.softmax(g, -1).unsqueeze(-1)
        ckv = (wt * keys[:, :nb * r].view(B, nb, r, L)).sum(2)                        # [B, nb, L]
        cik = (wt * self.ik[i][:, :nb * r].view(B, nb, r, hd)).sum(2)                # [B, nb, hd]
        qpos = (start + torch.arange(S)).view(S, 1)
        # window mask over full-resolution keys
        j = torch.arange(end).view(1, end)
        win = (j <= qpos) & (j > qpos - swa)                                           # [S, end]
        # candidate blocks (entirely before the window) and their top-k
        jb = torch.arange(nb).view(1, nb)
        cand = jb < (qpos + 1 - swa) // r                                              # [S, nb]
        sc = (torch.einsum("bshd,bjd->bshj", qi, cik).relu() * hw.unsqueeze(-1)).sum(2)  # [B, S, nb]
        sc = sc.masked_fill(~cand.unsqueeze(0), float("-inf"))
        sel = torch.zeros(B, S, nb, dtype=torch.bool)
        if nb:
            kk = min(c.compress_topk, nb)
            idx = sc.topk(kk, dim=-1).indices
            sel = sel.scatter_(2, idx, True) & cand.unsqueeze(0)
        s_w = torch.einsum("bshd,bld->bhsl", q, keys) * c.softmax_scale
        s_w = s_w.masked_fill(~win.view(1, 1, S, end), float("-inf"))
        s_c = torch.einsum("bshd,bjd->bhsj", q, ckv) * c.softmax_scale
        s_c = s_c.masked_fill(~sel.unsqueeze(1), float("-inf"))
        s_all = torch.cat([s_w, s_c], -1)
        if c.attn_sink:
            sink = w[a + "attn_sink"].view(1, H, 1, 1).expand(B, H, S, 1)
            p = torch.cat([s_all, sink], -1).softmax(-1)[..., :-1]
        else:
            p = s_all.softmax(-1)
        return (torch.einsum("bhsl,bld->bshd", p[..., :end], keys)
                + torch.einsum("bhsj,bjd->bshd", p[..., end:], ckv))

    def _indexer_select(self, i, x, qr, pos, start, S):
        """Lightning indexer (as the V3.2 oracle) plus the sliding window:
        top index_topk causal positions by score, the last index_swa always
        kept.  Returns bool mask [B, S, end]."""
        import torch.nn.functional as F
        from .rope import apply_rope_ref
        c, w = self.cfg, self.w
        a = f"model.layers.{i}.self_attn.indexer."
        B = x.shape[0]
        nh, hd, rd = c.index_n_heads, c.index_head_dim, c.qk_rope_head_dim
        q = (qr @ w[a + "wq_b.weight"].T).view(B, S, nh, hd)
        q = torch.cat([apply_rope_ref(q[..., :rd], pos.expand(B, S), self.rope), q[..., rd:]], -1)
        k = F.layer_norm(x @ w[a + "wk.weight"].T, (hd,), w[a + "k_norm.weight"], w[a + "k_norm.bias"], 1e-6)
        k = torch.cat([apply_rope_ref(k[..., :rd], pos.expand(B, S), self.rope), k[..., rd:]], -1)
        end = start + S
        self.ik[i][:, start:end] = k
        keys = self.ik[i][:, :end]
        hw = (x @ w[a + "weights_proj.weight"].T) * (nh ** -0.5) * (hd ** -0.5)
        sc = (torch.einsum("bshd,bld->bshl", q, keys).relu() * hw.unsqueeze(-1)).sum(2)
        qpos = (start + torch.arange(S)).view(S, 1)
        j = torch.arange(end).view(1, end)
        causal = j <= qpos
        sc = sc.masked_fill(~causal, float("-inf"))
        if c.index_swa:
            sc = sc.masked_fill(causal & (j > qpos - c.index_swa), float("inf"))
        idx = sc.topk(min(c.index_topk, end), dim=-1).indices
        sel = torch.zeros(B, S, end, dtype=torch.bool).scatter_(2, idx, True)
        return sel & causal

    # -- ffn ----------------------------------------------------------------------
    def _mlp(self, pre: str, x: torch.Tensor) -> torch.Tensor:
        w = self.w
        return (F.silu(x @ w[pre + "gate_proj.weight"].T) * (x @ w[pre + "up_proj.weight"].T)) \
            @ w[pre + "down_proj.weight"].T

    def _moe(self, i: int, x: torch.Tensor, decode: bool) -> torch.Tensor:
        c, w = self.cfg, self.w
        m = f"model.layers.{i}.mlp."
        shp = x.shape
        xt = x.reshape(-1, shp[-1])
        logits = xt @ w[m + "gate.weight"].T
        wts, ids = ref.router_sqrtsoftplus(logits, w[m + "gate.e_score_correction_bias"], c.num_experts_per_tok,
                                           c.routed_scaling_factor)
        if decode and c.prune_budget > 0:
            wts, ids = ref.e5_prune(ids, wts, c.prune_budget, c.prune_max_count)
        out = torch.zeros_like(xt)
        for e in range(c.n_routed_experts):
            hit = ids == e
            tok = hit.any(-1).nonzero().flatten()
            if tok.numel() == 0:
                continue
            we = (wts * hit).sum(-1)[tok].unsqueeze(-1)
            out.index_add_(0, tok, we * self._mlp(m + f"experts.{e}.", xt[tok]))
        if c.n_shared_experts:
            out = out + self._mlp(m + "shared_experts.", xt)
        return out.view(shp)

    def _ffn(self, i: int, x: torch.Tensor, decode: bool) -> torch.Tensor:
        if self.cfg.is_moe_layer(i):
            return self._moe(i, x, decode)
        return self._mlp(f"model.layers.{i}.mlp.", x)

    # -- engram ---------------------------------------------------------------------
    def _engram(self, i: int, X: torch.Tensor, start: int, S: int) -> torch.Tensor:
        c, w = self.cfg, self.w
        e = f"model.layers.{i}.engram."
        B = X.shape[0] // S
        ids = []
        for b in range(B):
            ctx = engram_context(self.tokens[b, : start + S], c.engram_max_ngram)[start:]
            ids.append(ref.engram_hash(ctx, c.engram_heads, c.engram_rows, c.engram_max_ngram))
        ids = torch.cat(ids, 0)
        emb = ref.engram_gather(w[e + "table"], w[e + "table_scale"], ids)
        kv = emb.flatten(1) @ w[e + "wkv.weight"].T
        return ref.engram_gate(X, kv, w[e + "q_norm.weight"], w[e + "k_norm.weight"], c.rms_norm_eps,
                               c.engram_clamp)

    # -- forward ----------------------------------------------------------------------
    @torch.no_grad()
    def forward(self, ids: torch.Tensor, start: int, decode: Optional[bool] = None) -> torch.Tensor:
        c, w = self.cfg, self.w
        B, S = ids.shape
        decode = (S == 1) if decode is None else decode
        self.tokens[:, start:start + S] = ids.long()
        hc, D = c.hc_mult, c.hidden_size
        X = w["model.embed_tokens.weight"][ids].reshape(B * S, 1, D).expand(B * S, hc, D).clone()
        self.aux = []
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            if i in c.engram_layers:
                X = self._engram(i, X, start, S)
            if i in c.aux_layers:
                self.aux.append(X.mean(1))
            pre, post, comb = self._coeffs(p + "attn_hc.", X)
            xin = ref.rmsnorm(ref.hc_combine(X, pre), w[p + "input_layernorm.weight"], c.rms_norm_eps)
            y = self._attn(i, xin.view(B, S, D), start).reshape(B * S, D)
            X = ref.hc_post(X, y, post, comb)
            pre, post, comb = self._coeffs(p + "ffn_hc.", X)
            xin = ref.rmsnorm(ref.hc_combine(X, pre), w[p + "post_attention_layernorm.weight"], c.rms_norm_eps)
            y = self._ffn(i, xin.view(B, S, D), decode).reshape(B * S, D)
            X = ref.hc_post(X, y, post, comb)
        raw, sq = ref.hc_stats(X, w["model.hc_head.fn"])
        pre = ref.hc_head_coeffs(raw, sq, w["model.hc_head.scale"], w["model.hc_head.base"], hc, hc * D, c.hc_eps)
        x = ref.rmsnorm(ref.hc_combine(X, pre), w["model.norm.weight"], c.rms_norm_eps)
        head = w["model.embed_tokens.weight"] if c.tie_word_embeddings else w["lm_head.weight"]
        return (x @ head.T).view(B, S, -1)

    @torch.no_grad()
    def greedy(self, prompts: torch.Tensor, new_tokens: int):
        B, S = prompts.shape
        self.reset(B)
        logits = self.forward(prompts, 0, decode=False)[:, -1]
        outs = []
        pos = S
        for _ in range(new_tokens):
            nxt = logits.argmax(-1)
            outs.append(nxt)
            if len(outs) == new_tokens:
                break
            logits = self.forward(nxt.view(B, 1), pos, decode=True)[:, -1]
            pos += 1
        return torch.stack(outs, 1)
