"""RoPE frequency tables (plain and YaRN-scaled) for the decoupled rope key.

The rotary dims are rotated as interleaved pairs (x[2i], x[2i+1]) treated as
one complex number, the convention of DeepSeek's own inference code; q and k
use the same convention so scores are unaffected by the layout choice.
"""
from __future__ import annotations

import math

import torch

from ..config import ModelConfig, yarn_mscale


def _yarn_find_correction_dim(num_rot, dim, base, max_pos):
    return (dim * math.log(max_pos / (num_rot * 2 * math.pi))) / (2 * math.log(base))


def _yarn_find_correction_range(low_rot, high_rot, dim, base, max_pos):
    low = math.floor(_yarn_find_correction_dim(low_rot, dim, base, max_pos))
    high = math.ceil(_yarn_find_correction_dim(high_rot, dim, base, max_pos))
    return max(low, 0), min(high, dim - 1)


def inv_freq(cfg: ModelConfig) -> torch.Tensor:
    """Per-pair inverse frequencies [rope_dim/2] in float64 precision."""
    dim = cfg.qk_rope_head_dim
    base = cfg.rope_theta
    freqs = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    rs = cfg.rope_scaling
    if rs and rs.get("type", rs.get("rope_type")) == "yarn":
        factor = rs["factor"]
        orig = rs["original_max_position_embeddings"]
        low, high = _yarn_find_correction_range(rs.get("beta_fast", 32), rs.get("beta_slow", 1), dim, base, orig)
        if low == high:
            high += 0.001
        ramp = ((torch.arange(dim // 2, dtype=torch.float64) - low) / (high - low)).clamp(0, 1)
        smooth = 1 - ramp
        freqs = freqs / factor * (1 - smooth) + freqs * smooth
    return freqs


def attn_mscale(cfg: ModelConfig) -> float:
    """Multiplier applied to cos/sin (1.0 for DeepSeek-V3 where mscale == mscale_all_dim)."""
    rs = cfg.rope_scaling
    if rs and rs.get("type", rs.get("rope_type")) == "yarn":
        return yarn_mscale(rs["factor"], rs.get("mscale", 1.0)) / yarn_mscale(rs["factor"], rs.get("mscale_all_dim", 0.0))
    return 1.0


def cos_sin_table(cfg: ModelConfig, max_pos: int, device=None) -> torch.Tensor:
    """[max_pos, rope_dim] float32: first half cos, second half sin (per pair)."""
    f = inv_freq(cfg)
    t = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(t, f)
    m = attn_mscale(cfg)
    tab = torch.cat([torch.cos(ang) * m, torch.sin(ang) * m], dim=-1).to(torch.float32)
    return tab.to(device) if device is not None else tab


def apply_rope_ref(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """x [*pos.shape, (heads,) rope_dim] rotated at positions pos (fp32 math)."""
    d = x.shape[-1]
    cs = table[pos.long()]                        # [*pos.shape, d]
    cos, sin = cs[..., : d // 2], cs[..., d // 2:]
    while cos.dim() < x.dim():
        cos = cos.unsqueeze(-2)
        sin = sin.unsqueeze(-2)
    xf = x.float()
    x0, x1 = xf[..., 0::2], xf[..., 1::2]
    y0 = x0 * cos - x1 * sin
    y1 = x0 * sin + x1 * cos
    return torch.stack([y0, y1], dim=-1).flatten(-2).to(x.dtype)
