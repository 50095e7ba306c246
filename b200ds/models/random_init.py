"""Random-init weights generated directly on the device, per rank, in the
serving formats (for benchmarks of the full-size architectures, whose fp32
state dict would not fit in host memory).

MXFP8 tensors get uniformly random e4m3 codes with the exponent MSB cleared
(finite, |x| <= 1.875, RMS ~0.59) and a constant UE8M0 scale of 2^-5, i.e.
weights with RMS ~0.018; bf16 tensors are N(0, 0.02); norms are ones; the
router gate is N(0, 0.02) so expert load is near uniform.

When the routed experts of all MoE layers do not fit in HBM (the 671B model
on fewer than 8 GPUs), `weight_sets` distinct expert sets are generated and
MoE layer i uses set i % weight_sets.  Every layer still streams its full
expert weights from HBM (one layer's experts are far larger than L2), so the
per-step work is that of the full model.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from ..config import EngineConfig, ModelConfig
from ..ops import ExpertWeights
from ..ops.quant import MXFP8Tensor, NVFP4Tensor, round_up
from ..parallel.state import ParallelState
from .deepseek import AttnWeights, DeepseekModel, DenseWeights, LayerWeights, Linear, MoEWeights

SCALE_BYTE = 127 - 5


def should_generate_on_device(cfg: ModelConfig, device) -> bool:
    return torch.device(device).type == "cuda" and cfg.num_params() > 1_000_000_000


class _Seeder:
    def __init__(self, seed: int):
        self.s = seed * 1_000_003 + 17

    def next(self) -> int:
        self.s += 1
        return self.s


def rand_mx(shape_lead, N: int, K: int, dev, seeder: _Seeder) -> MXFP8Tensor:
    from .. import _C
    Np = round_up(N, 128)
    data = torch.empty(*shape_lead, Np, K, dtype=torch.uint8, device=dev)
    _C.fill_bytes(data, seeder.next(), 0xBF, 0)
    if Np != N:
        data[..., N:, :] = 0
    sf = torch.full((*shape_lead, Np * K // 32), SCALE_BYTE, dtype=torch.uint8, device=dev)
    return MXFP8Tensor(data.view(torch.float8_e4m3fn), sf, N)


# NVFP4 random weights: uniform random e2m1 codes (all 16 are finite, RMS
# 2.93), unit e4m3 block scales (0x38 = 1.0) and a per-expert global scale
# giving RMS ~0.018 like the MXFP8 weights.
NVFP4_SCALE_BYTE = 0x38
NVFP4_GLOBAL = 0.018 / 2.93


def rand_nvfp4(E: int, N: int, K: int, dev, seeder: _Seeder) -> NVFP4Tensor:
    from .. import _C
    Np = round_up(N, 128)
    data = torch.empty(E, Np, K // 2, dtype=torch.uint8, device=dev)
    _C.fill_bytes(data, seeder.next(), 0xFF, 0)
    sf = torch.full((E, Np * K // 16), NVFP4_SCALE_BYTE, dtype=torch.uint8, device=dev)
    g = torch.full((E,), NVFP4_GLOBAL, dtype=torch.float32, device=dev)
    return NVFP4Tensor(data, sf, g, N)


def rand_bf16(shape, dev, gen, std=0.02, dtype=torch.bfloat16):
    t = torch.empty(shape, dtype=dtype, device=dev)
    t.normal_(0.0, std, generator=gen)
    return t


def expert_bytes_per_layer(cfg: ModelConfig, ep: int) -> int:
    per = cfg.n_routed_experts // ep
    h, I = cfg.hidden_size, cfg.moe_intermediate_size
    if cfg.expert_format == "nvfp4":
        return per * (2 * I * h + h * I) * (0.5 + 1 / 16)
    return per * (2 * I * h + h * I) * (1 + 1 / 32)


def auto_weight_sets(cfg: ModelConfig, ps: ParallelState, reserve_bytes: float, dev) -> int:
    n_moe = sum(1 for i in range(cfg.num_hidden_layers) if cfg.is_moe_layer(i))
    if n_moe == 0:
        return 1
    free, _ = torch.cuda.mem_get_info(dev)
    per = expert_bytes_per_layer(cfg, ps.ep_size)
    sets = int((free - reserve_bytes) // per)
    return max(1, min(n_moe, sets))


def build_random_model(cfg: ModelConfig, ecfg: EngineConfig, ps: ParallelState, device, seed: int = 0,
                       reserve_bytes: Optional[float] = None) -> DeepseekModel:
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed + 7919 * ps.rank)
    sd = _Seeder(seed * 131 + ps.rank)
    attn_tp = 1 if ecfg.dp_attention else ps.tp_size
    tp = ps.tp_size
    H = cfg.num_attention_heads
    Hl = H // attn_tp
    h = cfg.hidden_size
    n_moe = sum(1 for i in range(cfg.num_hidden_layers) if cfg.is_moe_layer(i))
    ones = lambda n: torch.ones(n, dtype=torch.float32, device=dev)

    layers: List[LayerWeights] = []
    # attention + dense + shared weights first (distinct per layer)
    attn_list, dense_list, shared_list = [], [], []
    for i in range(cfg.num_hidden_layers):
        ix_rows = cfg.index_head_dim + cfg.index_n_heads if cfg.index_n_heads else 0
        ixq_rows = cfg.index_n_heads * cfg.index_head_dim if cfg.index_n_heads else 0
        qkv_a = Linear(rand_mx((), cfg.q_lora_rank + cfg.kv_cache_dim + ix_rows, h, dev, sd))
        q_b = Linear(rand_mx((), Hl * cfg.qk_head_dim + ixq_rows, cfg.q_lora_rank, dev, sd))
        o = Linear(rand_mx((), h, Hl * cfg.v_head_dim, dev, sd))
        w_uk = rand_bf16((Hl, cfg.qk_nope_head_dim, cfg.kv_lora_rank), dev, gen)
        w_uv = rand_bf16((Hl, cfg.v_head_dim, cfg.kv_lora_rank), dev, gen)
        aw = AttnWeights(qkv_a=qkv_a, q_a_ln=ones(cfg.q_lora_rank), kv_a_ln=ones(cfg.kv_lora_rank), q_b=q_b,
                         w_uk=w_uk, w_uv=w_uv, o_proj=o)
        if cfg.index_n_heads:
            aw.ix_k_norm_w = ones(cfg.index_head_dim)
            aw.ix_k_norm_b = torch.zeros(cfg.index_head_dim, device=dev)
        attn_list.append(aw)
        if cfg.is_moe_layer(i):
            dense_list.append(None)
            if cfg.n_shared_experts:
                si = cfg.moe_intermediate_size * cfg.n_shared_experts // tp
                shared_list.append((Linear(_gate_up(si, h, dev, sd)), Linear(rand_mx((), h, si, dev, sd))))
            else:
                shared_list.append((None, None))
        else:
            I = cfg.intermediate_size // tp
            dense_list.append(DenseWeights(gate_up=Linear(_gate_up(I, h, dev, sd)), down=Linear(rand_mx((), h, I, dev, sd))))
            shared_list.append((None, None))
    embed = rand_bf16((cfg.vocab_size, h), dev, gen)
    v_local = cfg.vocab_size // tp if cfg.vocab_size % tp == 0 else -(-cfg.vocab_size // tp)
    # MXFP8 LM head (vocab-parallel): the tcgen05 GEMM streams half the bytes of bf16
    head = rand_mx((), v_local, h, dev, sd)

    # routed experts: distinct sets as memory allows
    per = cfg.n_routed_experts // ps.ep_size
    first = ps.ep_rank * per
    I = cfg.moe_intermediate_size
    if reserve_bytes is None:
        kv_tokens = ecfg.max_num_seqs * 4096
        reserve_bytes = 24e9 + kv_tokens * cfg.kv_cache_dim * cfg.num_hidden_layers
    sets = ecfg.weight_sets if ecfg.weight_sets > 0 else auto_weight_sets(cfg, ps, reserve_bytes, dev)
    expert_sets = []
    fp4 = cfg.expert_format == "nvfp4"
    for s in range(min(sets, n_moe)):
        if fp4:
            w13 = rand_nvfp4(per, 2 * I, h, dev, sd)
            w2 = rand_nvfp4(per, h, I, dev, sd)
        else:
            w13 = rand_mx((per,), 2 * I, h, dev, sd)
            w2 = rand_mx((per,), h, I, dev, sd)
        # Random bytes need no re-layout: with 64 or fewer experts per GPU
        # the grouped GEMM reads them as contiguous 128 x 128-byte tiles
        # (measured: FC1 at 32 experts/GPU 0.78 -> 0.83 of copy bandwidth).
        expert_sets.append(ExpertWeights(first=first, count=per, w13=w13, w2=w2, inter=I, tiled=per <= 64,
                                         random_init=True))
    moe_idx = 0
    for i in range(cfg.num_hidden_layers):
        if cfg.is_moe_layer(i):
            gate = rand_bf16((cfg.n_routed_experts, h), dev, gen, dtype=torch.float32)
            sgu, sdn = shared_list[i]
            ffn = MoEWeights(gate=gate, bias=torch.zeros(cfg.n_routed_experts, device=dev),
                             experts=expert_sets[moe_idx % len(expert_sets)], shared_gate_up=sgu, shared_down=sdn)
            moe_idx += 1
        else:
            ffn = dense_list[i]
        layers.append(LayerWeights(in_ln=ones(h), post_ln=ones(h), attn=attn_list[i], ffn=ffn))
    m = DeepseekModel(cfg, ecfg, ps, layers, embed, ones(h), head, dev, kv_dtype=torch.float8_e4m3fn)
    m.weight_sets = len(expert_sets)
    return m


def _gate_up(I: int, h: int, dev, sd) -> MXFP8Tensor:
    """[gate; up] stacked rows with I a multiple of 128 per half."""
    assert I % 128 == 0, I
    return rand_mx((), 2 * I, h, dev, sd)


def build_random_model_v4(cfg: ModelConfig, ecfg: EngineConfig, ps: ParallelState, device, seed: int = 0,
                          reserve_bytes: Optional[float] = None):
    """DeepSeek-V4-family model with random weights generated on the device
    in the serving formats (same conventions as above); Engram tables are
    random e4m3 rows in mapped host memory (this rank's row shard)."""
    from ..ops import EngramWeights, HcWeights
    from ..ops.cuda import hc_fn_parts
    from .deepseek_v4 import DeepseekV4Model, V4AttnWeights, V4LayerWeights, host_mapped_copy
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed + 7919 * ps.rank)
    sd = _Seeder(seed * 131 + ps.rank)
    tp, tr = ps.tp_size, ps.tp_rank
    h, hc = cfg.hidden_size, cfg.hc_mult
    H, L, G, R = cfg.num_attention_heads, cfg.kv_lora_rank, cfg.o_groups, cfg.o_lora_rank
    Hl, Gl = H // tp, G // tp
    ones = lambda n: torch.ones(n, dtype=torch.float32, device=dev)

    def hcw(m: int) -> HcWeights:
        fn = rand_bf16((m, hc * h), dev, gen, dtype=torch.float32)
        base = torch.zeros(m, device=dev)
        if m > hc:
            base[2 * hc:] = (torch.eye(hc, device=dev) * 4.0).flatten()
        w = HcWeights(fn, ones(3 if m > hc else 1), base)
        w.fn_parts = hc_fn_parts(fn)
        return w

    M = (2 + hc) * hc
    n_moe = sum(1 for i in range(cfg.num_hidden_layers) if cfg.is_moe_layer(i))
    per = cfg.n_routed_experts // ps.ep_size
    first = ps.ep_rank * per
    I = cfg.moe_intermediate_size
    if reserve_bytes is None:
        kv_tokens = ecfg.max_num_seqs * 4096
        reserve_bytes = 24e9 + kv_tokens * cfg.kv_cache_dim * cfg.num_hidden_layers
    sets = ecfg.weight_sets if ecfg.weight_sets > 0 else auto_weight_sets(cfg, ps, reserve_bytes, dev)
    fp4 = cfg.expert_format == "nvfp4"
    expert_sets = []
    for s in range(min(sets, max(n_moe, 1))):
        if fp4:
            w13, w2 = rand_nvfp4(per, 2 * I, h, dev, sd), rand_nvfp4(per, h, I, dev, sd)
        else:
            w13, w2 = rand_mx((per,), 2 * I, h, dev, sd), rand_mx((per,), h, I, dev, sd)
        expert_sets.append(ExpertWeights(first=first, count=per, w13=w13, w2=w2, inter=I, tiled=per <= 64,
                                         random_init=True))
    layers = []
    moe_idx = 0
    for i in range(cfg.num_hidden_layers):
        aw = V4AttnWeights(wqkv_a=Linear(rand_mx((), cfg.q_lora_rank + L, h, dev, sd)), q_norm=ones(cfg.q_lora_rank),
                           kv_norm=ones(L), wq_b=Linear(rand_mx((), Hl * L, cfg.q_lora_rank, dev, sd)),
                           wo_a=rand_bf16((Gl, R, (H // G) * L), dev, gen),
                           wo_b=Linear(rand_mx((), h, Gl * R, dev, sd)),
                           sink=rand_bf16((Hl,), dev, gen, std=1.0, dtype=torch.float32) if cfg.attn_sink else None)
        if cfg.is_moe_layer(i):
            sgu = sdn = None
            if cfg.n_shared_experts:
                si = cfg.moe_intermediate_size * cfg.n_shared_experts // tp
                sgu, sdn = Linear(_gate_up(si, h, dev, sd)), Linear(rand_mx((), h, si, dev, sd))
            ffn = MoEWeights(gate=rand_bf16((cfg.n_routed_experts, h), dev, gen, dtype=torch.float32),
                             bias=torch.zeros(cfg.n_routed_experts, device=dev),
                             experts=expert_sets[moe_idx % len(expert_sets)], shared_gate_up=sgu, shared_down=sdn)
            moe_idx += 1
        else:
            Id = cfg.intermediate_size // tp
            ffn = DenseWeights(gate_up=Linear(_gate_up(Id, h, dev, sd)), down=Linear(rand_mx((), h, Id, dev, sd)))
        eng = None
        if i in cfg.engram_layers:
            rows = cfg.engram_rows // tp
            cpu_gen = torch.Generator().manual_seed(seed * 7 + i * 131 + tr)
            table = torch.randint(0, 256, (rows, cfg.engram_dim), dtype=torch.uint8, generator=cpu_gen) & 0xBF
            scale = torch.full((rows, cfg.engram_dim // 32), SCALE_BYTE, dtype=torch.uint8)
            eng = EngramWeights(table=host_mapped_copy(table), scale=host_mapped_copy(scale), row_lo=tr * rows,
                                wkv=Linear(rand_mx((), 2 * h, cfg.engram_heads * cfg.engram_dim, dev, sd)),
                                q_w=ones(h), k_w=ones(h))
        layers.append(V4LayerWeights(attn_hc=hcw(M), ffn_hc=hcw(M), in_ln=ones(h), post_ln=ones(h), attn=aw,
                                     ffn=ffn, engram=eng))
    embed = rand_bf16((cfg.vocab_size, h), dev, gen)
    v_local = -(-cfg.vocab_size // tp)
    head = rand_mx((), v_local, h, dev, sd)
    m = DeepseekV4Model(cfg, ecfg, ps, layers, embed, hcw(hc), ones(h), head, dev, kv_dtype=torch.float8_e4m3fn)
    m.weight_sets = len(expert_sets)
    return m
