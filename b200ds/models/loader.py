"""Weight construction: HF state dicts / safetensors checkpoints (block-FP8:
e4m3 with `weight_scale_inv` block scales, fp32 on 128x128 blocks as in
DeepSeek-V3 or UE8M0 on 32x32 blocks as in the V4 family) and random init
generated directly in each rank's shard, in the serving formats.

Reference parity: the reference serves weights loaded by SGLang (absent) and
converts 32x32 ue8m0 block-FP8 to MXFP8 at bind time (dt.py:1-5, fl.py:1-10).
"""
from __future__ import annotations

import glob
import json
import os
from collections.abc import Mapping
from typing import Dict, Iterable, List, Optional

import torch

from ..config import EngineConfig, ModelConfig
from ..ops import ExpertWeights
from ..ops.quant import MXFP8Tensor, dequant_blocked, quant_mxfp8_ref, pack_sf, sf_packed_size, NVFP4Tensor, quant_nvfp4_ref, tile_rows128
from ..parallel.state import ParallelState
from .deepseek import AttnWeights, DeepseekModel, DenseWeights, LayerWeights, Linear, MoEWeights


def _quantize(w: torch.Tensor, fmt: str, device) -> object:
    """float weight [N, K] -> serving format on device (MXFP8 rows padded
    with zeros to a multiple of 128, the GEMM's weight tile)."""
    if fmt in ("fp32", "bf16"):
        return w.to(device=device, dtype=torch.float32 if fmt == "fp32" else torch.bfloat16)
    if fmt == "mxfp8":
        rows = w.shape[0]
        if w.shape[0] % 128:
            w = torch.cat([w, torch.zeros(128 - w.shape[0] % 128, w.shape[1], dtype=w.dtype, device=w.device)], 0)
        wd = w.to(device)
        if wd.is_cuda:
            from .. import ops
            a = ops.quant(wd.to(torch.bfloat16))
            return MXFP8Tensor(a.q, a.sf, rows)
        q, sf = quant_mxfp8_ref(wd.float())
        return MXFP8Tensor(q, sf, rows)
    if fmt == "nvfp4":
        t = quant_nvfp4_ref(w.to(device).float())
        return t
    raise ValueError(f"unknown weight format {fmt}")


def _stack(ws: List[object]) -> object:
    if isinstance(ws[0], MXFP8Tensor):
        return MXFP8Tensor(torch.stack([w.data for w in ws]), torch.stack([w.sf for w in ws]))
    if isinstance(ws[0], NVFP4Tensor):
        return NVFP4Tensor(torch.stack([w.data for w in ws]), torch.stack([w.sf for w in ws]),
                           torch.stack([w.global_scale.reshape(()) for w in ws]), ws[0].rows)
    return torch.stack(ws)


def _maybe_tile(ex: ExpertWeights) -> ExpertWeights:
    """GPU experts with 64 or fewer per rank are stored as contiguous
    128 x 128-byte tiles (the grouped GEMM's TMA boxes)."""
    if ex.count > 64 or not ex.w13.data.is_cuda:
        return ex
    for name in ("w13", "w2"):
        t = getattr(ex, name)
        d = tile_rows128(t.data.view(torch.uint8)).view(t.data.dtype)
        if isinstance(t, MXFP8Tensor):
            setattr(ex, name, MXFP8Tensor(d, t.sf, t.rows))
        else:
            setattr(ex, name, NVFP4Tensor(d, t.sf, t.global_scale, t.rows))
    ex.tiled = True
    return ex


def build_ffn(cfg: ModelConfig, sd, get, split, m: str, i: int, ps: ParallelState, dev):
    """Layer i's FFN from the state dict: routed experts (this rank's EP
    slice, stacked in the expert format) + TP-split shared expert, or the
    TP-split dense SwiGLU FFN."""
    fmt_d = cfg.dense_format
    tp, tr = ps.tp_size, ps.tp_rank
    if cfg.is_moe_layer(i):
        per = cfg.n_routed_experts // ps.ep_size
        first = ps.ep_rank * per
        w13, w2 = [], []
        for e in range(first, first + per):
            q = m + f"experts.{e}."
            w13.append(_quantize(torch.cat([get(q + "gate_proj.weight"), get(q + "up_proj.weight")], 0),
                                 cfg.expert_format, dev))
            w2.append(_quantize(get(q + "down_proj.weight"), cfg.expert_format, dev))
        ex = _maybe_tile(ExpertWeights(first=first, count=per, w13=_stack(w13), w2=_stack(w2),
                                       inter=cfg.moe_intermediate_size))
        sgu = sdn = None
        if cfg.n_shared_experts:
            q = m + "shared_experts."
            g = split(get(q + "gate_proj.weight"), 0, tp, tr)
            u = split(get(q + "up_proj.weight"), 0, tp, tr)
            sgu = Linear(_quantize(torch.cat([g, u], 0), fmt_d, dev))
            sdn = Linear(_quantize(split(get(q + "down_proj.weight"), 1, tp, tr), fmt_d, dev))
        ffn = MoEWeights(gate=get(m + "gate.weight").to(dev),
                         bias=sd[m + "gate.e_score_correction_bias"].float().to(dev),
                         experts=ex, shared_gate_up=sgu, shared_down=sdn)
    else:
        g = split(get(m + "gate_proj.weight"), 0, tp, tr)
        u = split(get(m + "up_proj.weight"), 0, tp, tr)
        ffn = DenseWeights(gate_up=Linear(_quantize(torch.cat([g, u], 0), fmt_d, dev)),
                           down=Linear(_quantize(split(get(m + "down_proj.weight"), 1, tp, tr), fmt_d, dev)))
    return ffn


def build_model(cfg: ModelConfig, ecfg: EngineConfig, ps: ParallelState,
                sd: Dict[str, torch.Tensor], device="cpu", kv_dtype=None) -> DeepseekModel:
    """Build this rank's model from a FULL (unsharded) HF-named state dict of
    float tensors (or fp8 + `<name>_scale_inv`)."""
    dev = torch.device(device)
    attn_tp = 1 if ecfg.dp_attention else ps.tp_size
    attn_rank = 0 if ecfg.dp_attention else ps.tp_rank
    tp, tr = ps.tp_size, ps.tp_rank
    H = cfg.num_attention_heads
    Hl = H // attn_tp

    def get(name) -> torch.Tensor:
        t = sd[name]
        si = sd.get(name + "_scale_inv")
        if dev.type == "cuda":       # fp8 bytes cross the host link; dequantize on the device
            t = t.to(dev)
            si = si.to(dev) if si is not None else None
        if si is not None:
            t = dequant_blocked(t, si)
        return t.float()

    def split(t, dim, n, r):
        return t.chunk(n, dim)[r].contiguous() if n > 1 else t

    fmt_d = cfg.dense_format
    def layer_at(i: int) -> LayerWeights:
        p = f"model.layers.{i}."
        a = p + "self_attn."
        qa = get(a + "q_a_proj.weight")
        kva = get(a + "kv_a_proj_with_mqa.weight")
        qb = split(get(a + "q_b_proj.weight").view(H, cfg.qk_head_dim, -1), 0, attn_tp, attn_rank)
        qb = qb.reshape(Hl * cfg.qk_head_dim, -1)
        a_rows, b_rows = [qa, kva], [qb]
        if cfg.index_n_heads:
            # indexer projections appended to the attention GEMMs (replicated on every rank)
            ix = a + "indexer."
            a_rows += [get(ix + "wk.weight"), get(ix + "weights_proj.weight")]
            b_rows += [get(ix + "wq_b.weight")]
        qkv_a = Linear(_quantize(torch.cat(a_rows, 0), fmt_d, dev))
        q_b = Linear(_quantize(torch.cat(b_rows, 0), fmt_d, dev))
        kvb = split(get(a + "kv_b_proj.weight").view(H, cfg.qk_nope_head_dim + cfg.v_head_dim, -1), 0,
                    attn_tp, attn_rank)
        wdt = torch.bfloat16 if dev.type == "cuda" else torch.float32
        w_uk = kvb[:, : cfg.qk_nope_head_dim].contiguous().to(dev, wdt)
        w_uv = kvb[:, cfg.qk_nope_head_dim:].contiguous().to(dev, wdt)
        o = split(get(a + "o_proj.weight"), 1, attn_tp, attn_rank)
        aw = AttnWeights(qkv_a=qkv_a, q_a_ln=sd[a + "q_a_layernorm.weight"].float().to(dev),
                         kv_a_ln=sd[a + "kv_a_layernorm.weight"].float().to(dev), q_b=q_b,
                         w_uk=w_uk, w_uv=w_uv, o_proj=Linear(_quantize(o, fmt_d, dev)))
        if cfg.index_n_heads:
            ix = a + "indexer."
            aw.ix_k_norm_w = sd[ix + "k_norm.weight"].float().to(dev)
            aw.ix_k_norm_b = sd[ix + "k_norm.bias"].float().to(dev)
        ffn = build_ffn(cfg, sd, get, split, p + "mlp.", i, ps, dev)
        return LayerWeights(in_ln=sd[p + "input_layernorm.weight"].float().to(dev),
                            post_ln=sd[p + "post_attention_layernorm.weight"].float().to(dev), attn=aw, ffn=ffn)

    layers: List[LayerWeights] = [layer_at(i) for i in range(cfg.num_hidden_layers)]
    emb_dt = torch.bfloat16 if dev.type == "cuda" else torch.float32
    embed = sd["model.embed_tokens.weight"].float().to(dev, emb_dt)
    head_full = sd["model.embed_tokens.weight"] if cfg.tie_word_embeddings else sd["lm_head.weight"]
    head = split(head_full.float(), 0, tp, tr)
    # quantized formats serve the LM head in MXFP8 as well (tcgen05 GEMM)
    head = _quantize(head, "mxfp8", dev) if fmt_d == "mxfp8" and dev.type == "cuda" else head.to(dev, emb_dt)
    if kv_dtype is None:
        kv_dtype = torch.float8_e4m3fn if dev.type == "cuda" else torch.float32
    model = DeepseekModel(cfg, ecfg, ps, layers, embed, sd["model.norm.weight"].float().to(dev), head, dev,
                          kv_dtype=kv_dtype)
    L = cfg.num_hidden_layers
    m = f"model.layers.{L}."
    if cfg.num_nextn_predict_layers and (m + "eh_proj.weight") in sd:
        from .mtp import MTPDraft
        block = DeepseekModel(cfg, ecfg, ps, [layer_at(L)], embed, sd[m + "shared_head.norm.weight"].float().to(dev),
                              head, dev, kv_dtype=kv_dtype)
        model.mtp = MTPDraft(block, sd[m + "enorm.weight"].float().to(dev), sd[m + "hnorm.weight"].float().to(dev),
                             Linear(_quantize(get(m + "eh_proj.weight"), fmt_d, dev)))
    return model


# ---------------------------------------------------------------------------
# safetensors checkpoints
# ---------------------------------------------------------------------------

class LazyCheckpoint(Mapping):
    """Read-on-access view of a HF safetensors checkpoint directory: the
    constructor reads only the file headers (tensor name -> file); a tensor
    is read from its (memory-mapped) file when the model builder asks for
    it.  So a rank reads the weights it keeps - its expert slice, the
    replicated / TP-split dense weights - and never the whole checkpoint
    (the 671B fp8 checkpoint is ~690 GB; eight ranks each holding it in host
    memory would not fit).  fp8 tensors keep their `_scale_inv` companions."""

    def __init__(self, path: str, names: Optional[Iterable[str]] = None):
        from safetensors import safe_open
        want = set(names) if names is not None else None
        self.path = path
        self._where: Dict[str, str] = {}
        for f in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
            with safe_open(f, framework="pt") as fh:
                for k in fh.keys():
                    if want is None or k in want or k.replace("_scale_inv", "") in want:
                        self._where[k] = f
        self.reads = 0

    def __getitem__(self, k: str) -> torch.Tensor:
        from safetensors import safe_open
        f = self._where[k]
        self.reads += 1
        with safe_open(f, framework="pt") as fh:
            return fh.get_tensor(k)

    def __iter__(self):
        return iter(self._where)

    def __len__(self) -> int:
        return len(self._where)

    def __contains__(self, k) -> bool:
        return k in self._where


def load_checkpoint(path: str, names: Optional[Iterable[str]] = None) -> LazyCheckpoint:
    """The tensors (or the listed ones) of a HF safetensors checkpoint
    directory, read when accessed (LazyCheckpoint)."""
    return LazyCheckpoint(path, names)


def _fp8_names(k: str, v: torch.Tensor) -> bool:
    """The 2-D projection weights a block-FP8 checkpoint stores in e4m3."""
    if v.dim() != 2:
        return False
    return (k.endswith("proj.weight") or ".experts." in k or k.endswith(("wqkv_a.weight", "wq_b.weight",
                                                                         "wo_b.weight", "wkv.weight")))


def save_checkpoint_fp8(sd: Dict[str, torch.Tensor], path: str, cfg: ModelConfig, shard_bytes: int = 1 << 30,
                        block: int = 128, ue8m0: bool = False):
    """Write a state dict as a block-FP8 checkpoint: every 2-D projection
    weight as e4m3 + `weight_scale_inv` per block x block tile (fp32 scales,
    or UE8M0 powers of two stored as float8_e8m0fnu with ue8m0=True; the V4
    family's checkpoints use 32 x 32 UE8M0)."""
    from safetensors.torch import save_file
    from ..ops.quant import ue8m0_ceil_exponent
    os.makedirs(path, exist_ok=True)
    out: Dict[str, torch.Tensor] = {}
    for k, v in sd.items():
        if _fp8_names(k, v):
            N, K = v.shape
            nb, kb = (N + block - 1) // block, (K + block - 1) // block
            pad = torch.zeros(nb * block, kb * block)
            pad[:N, :K] = v.float()
            blk = pad.view(nb, block, kb, block).abs().amax((1, 3)).clamp(min=1e-12) / 448.0
            if ue8m0:
                e = ue8m0_ceil_exponent(blk)
                blk = torch.ldexp(torch.ones_like(blk), e)
            q = (pad.view(nb, block, kb, block) / blk.view(nb, 1, kb, 1)).view(nb * block, kb * block)[:N, :K]
            out[k] = q.to(torch.float8_e4m3fn).contiguous()
            if ue8m0:
                out[k + "_scale_inv"] = (e + 127).to(torch.uint8).view(torch.float8_e8m0fnu).contiguous()
            else:
                out[k + "_scale_inv"] = blk.float().contiguous()
        else:
            out[k] = v.contiguous()
    save_file(out, os.path.join(path, "model-00001-of-00001.safetensors"))
    d = cfg.to_dict()
    qc = {"quant_method": "fp8", "weight_block_size": [block, block]}
    if ue8m0:
        qc["scale_fmt"] = "ue8m0"
    d["quantization_config"] = qc
    d["architectures"] = ["DeepseekV4ForCausalLM" if cfg.is_v4 else "DeepseekV3ForCausalLM"]
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(d, f)
