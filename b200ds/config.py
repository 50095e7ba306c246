"""Model and engine configuration.

`ModelConfig` carries the DeepSeek-V3 family architecture (MLA attention with
q/kv low-rank projections and a decoupled RoPE key, dense first layers, then
sigmoid-routed MoE with a shared expert) plus the V3.2-style sparse-attention
indexer.  It reads a Hugging Face `config.json` (the fields DeepSeek-V3 ships)
and offers the named presets the benchmarks use.

Reference parity: the served model's facts are recovered in the reference from
kernel constants (hq_unit.cu:36-37, route_e5.cu:4-12, fork_attn.py:174-237,
levers.py:78-80); the reference takes its config from the absent SGLang fork.
"""
from __future__ import annotations

import dataclasses
import json
import math
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class ModelConfig:
    vocab_size: int = 129280
    hidden_size: int = 7168
    intermediate_size: int = 18432          # dense-layer FFN width
    moe_intermediate_size: int = 2048
    num_hidden_layers: int = 61
    first_k_dense_replace: int = 3
    num_attention_heads: int = 128
    q_lora_rank: Optional[int] = 1536
    kv_lora_rank: int = 512
    qk_nope_head_dim: int = 128
    qk_rope_head_dim: int = 64
    v_head_dim: int = 128
    n_routed_experts: int = 256
    n_shared_experts: int = 1
    num_experts_per_tok: int = 8
    n_group: int = 8
    topk_group: int = 4
    routed_scaling_factor: float = 2.5
    scoring_func: str = "sigmoid"
    norm_topk_prob: bool = True
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: Optional[dict] = field(default_factory=lambda: {
        "type": "yarn", "factor": 40.0, "original_max_position_embeddings": 4096,
        "beta_fast": 32.0, "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0})
    max_position_embeddings: int = 163840
    tie_word_embeddings: bool = False
    # multi-token prediction modules after the last layer (DeepSeek-V3 ships 1;
    # the engine uses the first as the speculative-decoding draft)
    num_nextn_predict_layers: int = 0
    # Sparse attention (V3.2-style lightning indexer); 0 heads = dense MLA.
    index_n_heads: int = 0
    index_head_dim: int = 128
    index_topk: int = 2048
    # sliding window always kept by the sparse selection (the last index_swa
    # positions up to the query), on top of the indexer's top-k
    index_swa: int = 0
    # Weight formats: "mxfp8" (e4m3 + UE8M0 per 32 along K), "nvfp4"
    # (e2m1 + e4m3 per 16 along K + fp32 global), "bf16" or "fp32".
    dense_format: str = "mxfp8"
    expert_format: str = "mxfp8"
    # ---- DeepSeek-V4-family architecture (arch="deepseek_v4"; all off for V3) ----
    # mHC: hc_mult residual streams mixed per sublayer by coefficients computed
    # from the streams (pre: combine into the sublayer input, post: spread the
    # output, comb: Sinkhorn-normalised stream mixing).
    arch: str = "deepseek_v3"
    hc_mult: int = 0
    hc_sinkhorn_iters: int = 20
    hc_eps: float = 1e-6
    # MQA latent attention: one shared K=V row of kv_lora_rank per token whose
    # last qk_rope_head_dim dims carry RoPE; queries of kv_lora_rank per head;
    # per-head softmax sinks; the output's rope tail is rotated back; output
    # projection = grouped low-rank wo_a (o_groups x o_lora_rank) then wo_b.
    o_lora_rank: int = 0
    o_groups: int = 0
    attn_sink: bool = False
    # E5 routed-expert prune at decode (budget 0 = off): an expert picked by at
    # most prune_max_count rows is dropped when each picker's cumulative mass up
    # to it (lightest first) stays within prune_budget of the row's mass.
    prune_budget: float = 0.0
    prune_max_count: int = 1
    # Engram: hashed n-gram lookups into host-memory e4m3 tables (rows of
    # engram_dim bytes + UE8M0 per 32) before these layers, gated into every
    # residual stream.
    engram_layers: tuple = ()
    engram_heads: int = 0
    engram_dim: int = 256
    engram_rows: int = 0
    engram_max_ngram: int = 3
    engram_clamp: float = 10.0
    # layers whose residual-stream mean is exported (draft-model taps)
    aux_layers: tuple = ()
    # Compressed sparse attention (V4 family, layers with the indexer): a layer
    # with ratio r > 1 keeps, per sequence, one compressed latent row per r
    # consecutive positions - a learned gated mean of their KV rows (weights =
    # softmax over the block of wgate . x_i + pos_bias[i mod r]) - and compressed
    # indexer keys made the same way.  A query attends to its sliding window
    # (the last index_swa positions) plus the compress_topk compressed blocks
    # before the window that the indexer ranks highest.
    compress_ratios: tuple = ()      # per layer; 0 or 1 = full resolution
    compress_topk: int = 512
    # Window-only late layers: layers >= late_layer_start attend to the last
    # late_window positions (up to and including the query) and skip the
    # indexer.  Prefill then needs those layers only on each prompt's tail.
    late_layer_start: Optional[int] = None
    late_window: int = 0

    # ---- derived -----------------------------------------------------------
    @property
    def is_v4(self) -> bool:
        return self.arch == "deepseek_v4"

    @property
    def qk_head_dim(self) -> int:
        if self.is_v4:
            return self.kv_lora_rank
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def kv_cache_dim(self) -> int:
        """Latent (kv_lora_rank) + decoupled rope key per token."""
        return self.kv_lora_rank + self.qk_rope_head_dim

    def is_moe_layer(self, i: int) -> bool:
        return self.n_routed_experts > 0 and i >= self.first_k_dense_replace

    def compress_ratio(self, i: int) -> int:
        """Compression ratio of layer i (0: full-resolution keys)."""
        if not self.is_v4 or not self.index_n_heads or self.is_window_layer(i) or i >= len(self.compress_ratios):
            return 0
        r = int(self.compress_ratios[i])
        return r if r > 1 else 0

    def is_window_layer(self, i: int) -> bool:
        return self.late_layer_start is not None and self.late_window > 0 and i >= self.late_layer_start

    def tail_rows_needed(self) -> int:
        """Positions before a prompt's end whose window-layer rows a prefill
        must compute so that every later read is exact.  A row left out
        leaves that layer's key row unwritten; a computed row whose window
        reaches an unwritten one is off, and each further window layer
        spreads that late_window - 1 rows forward.  With n window layers the
        last row's output (the logits) and the decode windows' key rows
        (positions >= end - late_window + 1 in every window layer) stay
        exact when the rows from end - n * (late_window - 1) - 1 on are
        computed."""
        n = self.num_hidden_layers - self.late_layer_start
        return n * (self.late_window - 1) + 1

    @property
    def softmax_scale(self) -> float:
        s = 1.0 / math.sqrt(self.qk_head_dim)
        if self.is_v4:
            return s
        rs = self.rope_scaling
        if rs and rs.get("type", rs.get("rope_type")) == "yarn":
            m = yarn_mscale(rs["factor"], rs.get("mscale_all_dim", 0.0))
            s = s * m * m
        return s

    def num_params(self) -> int:
        h = self.hidden_size
        H = self.num_attention_heads
        qr = self.q_lora_rank or 0
        if self.is_v4:
            L = self.kv_lora_rank
            attn = h * (qr + L) + qr * H * L + self.o_groups * self.o_lora_rank * (H // self.o_groups) * L
            attn += h * self.o_groups * self.o_lora_rank
            moe = (self.n_routed_experts + self.n_shared_experts) * 3 * h * self.moe_intermediate_size
            moe += self.n_routed_experts * h
            n_moe = sum(1 for i in range(self.num_hidden_layers) if self.is_moe_layer(i))
            dense = 3 * h * self.intermediate_size
            hc = 2 * (2 + self.hc_mult) * self.hc_mult * self.hc_mult * h if self.hc_mult else 0
            emb = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
            eng = len(self.engram_layers) * 2 * h * self.engram_heads * self.engram_dim
            return (self.num_hidden_layers * (attn + hc) + n_moe * moe + (self.num_hidden_layers - n_moe) * dense
                    + emb + eng)
        attn = (h * qr + qr * H * self.qk_head_dim if qr else h * H * self.qk_head_dim)
        attn += h * self.kv_cache_dim + self.kv_lora_rank * H * (self.qk_nope_head_dim + self.v_head_dim)
        attn += H * self.v_head_dim * h
        dense = 3 * h * self.intermediate_size
        moe = (self.n_routed_experts + self.n_shared_experts) * 3 * h * self.moe_intermediate_size
        moe += self.n_routed_experts * h
        n_moe = sum(1 for i in range(self.num_hidden_layers) if self.is_moe_layer(i))
        n_dense = self.num_hidden_layers - n_moe
        emb = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
        return self.num_hidden_layers * attn + n_dense * dense + n_moe * moe + emb

    # ---- io ----------------------------------------------------------------
    @classmethod
    def from_hf(cls, path_or_dict) -> "ModelConfig":
        """Build from a Hugging Face DeepSeek `config.json` (path or dict); a
        config written by `to_dict` (V4-family fields included) round-trips."""
        if isinstance(path_or_dict, dict):
            d = path_or_dict
        else:
            with open(path_or_dict) as f:
                d = json.load(f)
        names = {f.name for f in dataclasses.fields(cls)}
        # JSON lists of the tuple-valued fields (layer lists, ratios) back to tuples
        kw = {k: (tuple(v) if isinstance(v, list) else v) for k, v in d.items() if k in names}
        if "index_n_heads" not in d and "index_head_dim" in d:
            kw["index_n_heads"] = 64
        qc = d.get("quantization_config") or {}
        if qc.get("quant_method") == "fp8":
            kw.setdefault("dense_format", "mxfp8")
            kw.setdefault("expert_format", "mxfp8")
        return cls(**kw)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


def yarn_mscale(scale: float, mscale: float = 1.0) -> float:
    if scale <= 1.0:
        return 1.0
    return 0.1 * mscale * math.log(scale) + 1.0


# ---------------------------------------------------------------------------
# Presets
# ---------------------------------------------------------------------------

def tiny_config(**over) -> ModelConfig:
    """The tiny CPU / gloo plumbing model: 2 layers (dense FFN 512, then MoE), hidden 256,
    4 heads, q_lora 128, kv_lora 64, nope 32, rope 16, v 32, 8 experts top-2
    sigmoid + 1 shared, moe_intermediate 128, vocab 1024."""
    c = ModelConfig(
        vocab_size=1024, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
        num_hidden_layers=2, first_k_dense_replace=1, num_attention_heads=4,
        q_lora_rank=128, kv_lora_rank=64, qk_nope_head_dim=32, qk_rope_head_dim=16,
        v_head_dim=32, n_routed_experts=8, n_shared_experts=1, num_experts_per_tok=2,
        n_group=1, topk_group=1, routed_scaling_factor=1.0, max_position_embeddings=4096,
        rope_scaling=None, dense_format="fp32", expert_format="fp32")
    return dataclasses.replace(c, **over)


def v3_671b_config(**over) -> ModelConfig:
    """The DeepSeek-V3-shaped 671B decoder (the headline benchmark model)."""
    return dataclasses.replace(ModelConfig(), **over)


def v32_sparse_config(**over) -> ModelConfig:
    """The 671B model with a 64-head fp8 lightning indexer
    selecting top-2048 latent-KV tokens per query."""
    return dataclasses.replace(ModelConfig(index_n_heads=64, index_head_dim=128, index_topk=2048), **over)


def v3_nvfp4_config(**over) -> ModelConfig:
    """The 671B model with routed experts in NVFP4, shared/dense in MXFP8."""
    return dataclasses.replace(ModelConfig(expert_format="nvfp4", dense_format="mxfp8"), **over)


def kimi_k2_config(**over) -> ModelConfig:
    """The DeepSeek-V3 architecture at Kimi-K2 widths (1.04T parameters): 64
    heads, 384 routed experts top-8 in one group, one dense first layer,
    vocab 163840 - the same engine path with more experts per rank."""
    c = ModelConfig(vocab_size=163840, num_attention_heads=64, n_routed_experts=384, n_group=1, topk_group=1,
                    first_k_dense_replace=1, routed_scaling_factor=2.827, rope_theta=50000.0,
                    rope_scaling={"type": "yarn", "factor": 32.0, "original_max_position_embeddings": 4096,
                                  "beta_fast": 1.0, "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0},
                    max_position_embeddings=131072)
    return dataclasses.replace(c, **over)


def small_gpu_config(**over) -> ModelConfig:
    """A V3-shaped model small enough for single-GPU unit tests (4 layers)."""
    c = ModelConfig(
        vocab_size=4096, hidden_size=1024, intermediate_size=2048, moe_intermediate_size=256,
        num_hidden_layers=4, first_k_dense_replace=1, num_attention_heads=16,
        q_lora_rank=384, kv_lora_rank=512, qk_nope_head_dim=128, qk_rope_head_dim=64,
        v_head_dim=128, n_routed_experts=32, n_shared_experts=1, num_experts_per_tok=8,
        n_group=4, topk_group=2, routed_scaling_factor=2.5, max_position_embeddings=8192)
    return dataclasses.replace(c, **over)


def tiny_v4_config(**over) -> ModelConfig:
    """DeepSeek-V4-family CPU/gloo test model: 3 layers (dense, MoE, MoE),
    hidden 256, 4 MQA heads of 64 (rope tail 16), 2 output groups of rank 64,
    4 mHC streams, 8 experts top-2 with sqrt-softplus scoring and the E5
    prune, one Engram layer (4 hash heads)."""
    c = ModelConfig(
        arch="deepseek_v4", vocab_size=1024, hidden_size=256, intermediate_size=512, moe_intermediate_size=128,
        num_hidden_layers=3, first_k_dense_replace=1, num_attention_heads=4, q_lora_rank=128, kv_lora_rank=64,
        qk_nope_head_dim=48, qk_rope_head_dim=16, v_head_dim=64, o_lora_rank=64, o_groups=2, attn_sink=True,
        n_routed_experts=8, n_shared_experts=1, num_experts_per_tok=2, n_group=1, topk_group=1,
        routed_scaling_factor=1.5, scoring_func="sqrtsoftplus", prune_budget=0.4, prune_max_count=1,
        hc_mult=4, hc_sinkhorn_iters=8, engram_layers=(1,), engram_heads=4, engram_dim=256, engram_rows=512,
        aux_layers=(2,), max_position_embeddings=4096, rope_scaling=None, dense_format="fp32",
        expert_format="fp32")
    return dataclasses.replace(c, **over)


def small_v4_gpu_config(**over) -> ModelConfig:
    """A V4-family model for single-GPU tests on the tensor-core paths: 16
    heads of 512 (rope 64) in 4 output groups of rank 512, 32 experts top-6,
    4 mHC streams, Engram at layer 1."""
    c = ModelConfig(
        arch="deepseek_v4", vocab_size=4096, hidden_size=1024, intermediate_size=2048, moe_intermediate_size=256,
        num_hidden_layers=4, first_k_dense_replace=1, num_attention_heads=16, q_lora_rank=384, kv_lora_rank=512,
        qk_nope_head_dim=448, qk_rope_head_dim=64, v_head_dim=512, o_lora_rank=512, o_groups=4, attn_sink=True,
        n_routed_experts=32, n_shared_experts=1, num_experts_per_tok=6, n_group=1, topk_group=1,
        routed_scaling_factor=1.5, scoring_func="sqrtsoftplus", prune_budget=0.4, prune_max_count=1,
        hc_mult=4, hc_sinkhorn_iters=20, engram_layers=(1,), engram_heads=8, engram_dim=256, engram_rows=8192,
        aux_layers=(3,), max_position_embeddings=8192, rope_scaling=None)
    return dataclasses.replace(c, **over)


def v41_flash_config(**over) -> ModelConfig:
    """DeepSeek-V4.1-Flash-shaped decoder (the reference's served model, facts
    from its kernel constants): hidden 5120, 40 layers, 64 MQA heads of 512
    (rope tail 64), q_lora 1280, 8 output groups of rank 1024, 384 routed
    experts top-6 (sqrt-softplus, E5 prune 0.4) + 1 shared, 4 mHC streams,
    Engram at layers 1 and 14 (100 hash heads of 256).  Widths the reference
    does not pin (expert width 2304 from its shared expert, vocab, table
    rows) are stated here."""
    c = ModelConfig(
        arch="deepseek_v4", vocab_size=129280, hidden_size=5120, intermediate_size=12288,
        moe_intermediate_size=2304, num_hidden_layers=40, first_k_dense_replace=0, num_attention_heads=64,
        q_lora_rank=1280, kv_lora_rank=512, qk_nope_head_dim=448, qk_rope_head_dim=64, v_head_dim=512,
        o_lora_rank=1024, o_groups=8, attn_sink=True, n_routed_experts=384, n_shared_experts=1,
        num_experts_per_tok=6, n_group=1, topk_group=1, routed_scaling_factor=2.5, scoring_func="sqrtsoftplus",
        prune_budget=0.4, prune_max_count=1, hc_mult=4, hc_sinkhorn_iters=20, engram_layers=(1, 14),
        engram_heads=100, engram_dim=256, engram_rows=1 << 22, aux_layers=(37, 38, 39),
        max_position_embeddings=163840, rope_scaling=None, expert_format="nvfp4")
    return dataclasses.replace(c, **over)


PRESETS = {
    "tiny": tiny_config,
    "deepseek-v3-671b": v3_671b_config,
    "deepseek-v3.2-sparse-671b": v32_sparse_config,
    "deepseek-v3-671b-nvfp4": v3_nvfp4_config,
    "deepseek-r1-671b": v3_671b_config,
    "kimi-k2-1t": kimi_k2_config,
    "small": small_gpu_config,
    "tiny-v4": tiny_v4_config,
    "small-v4": small_v4_gpu_config,
    "deepseek-v4.1-flash": v41_flash_config,
}


@dataclass
class EngineConfig:
    """Serving-engine knobs (scheduler, KV pool, graphs, parallelism)."""
    tp_size: int = 1                 # attention tensor parallel width
    ep_size: int = 1                 # expert parallel width
    dp_attention: bool = False       # data-parallel attention (tp_size=1 per DP rank) + EP MoE
    page_size: int = 64              # tokens per KV page
    max_model_len: int = 16384       # longest sequence (sizes graph block tables)
    max_num_seqs: int = 256          # concurrent running requests
    max_prefill_tokens: int = 16384  # chunked-prefill budget per step
    schedule_policy: str = "fcfs"    # admission order: "fcfs", "lpm" (longest cached prefix first), "priority"
    mixed_steps: bool = False        # prefill steps also advance running requests by one decode token
    context_parallel: bool = False   # DP attention: long prompts prefill on every rank (rows split round-robin)
    cp_min_tokens: int = 8192        # server: prompts at least this long take the context-parallel path
    tbo: bool = False                # DP attention: two-batch overlap of prefill steps (MoE exchange vs compute)
    tbo_min_tokens: int = 1024       # ... when the largest rank's step has at least this many rows
    prefill_tail: bool = True        # window-only late layers (V4 family) run only on each prompt's tail rows
    kv_cache_fraction: float = 0.85  # of free HBM after weights
    max_kv_pages: Optional[int] = None
    cuda_graphs: bool = True         # capture decode per batch bucket
    extend_graphs: bool = False      # also replay prefill chunks up to 2048 tokens from per-bucket graphs
    graph_batch_sizes: tuple = (1, 2, 4, 8, 16, 32, 64, 128, 256)
    enable_prefix_cache: bool = True
    host_kv_pages: int = 0           # >0: pages of pinned host memory behind the prefix cache (evicted pages move there)
    comm_impl: str = "fused"         # "fused" (own NVLink kernels) or "nccl" (baseline)
    gemm_impl: str = "native"        # "native" (own tcgen05 kernels) or "torch" (baseline)
    seed: int = 0
    weight_sets: int = 0             # >0: cycle this many distinct layer weight sets (when the model exceeds HBM)
    spec_ngram: int = 0              # >0: speculative decoding with n-gram (prompt lookup) drafts up to this n
    spec_k: int = 4                  # draft tokens verified per step
    spec_mtp: bool = False           # speculative decoding with the model's MTP module as the draft
    selfcheck: bool = True           # GPU: check each switchable fast path once at start (fail-closed, ranks agree)
    trace: bool = False              # device timestamps per layer phase (also B200_TRACE=1); adds launches
