"""Block-scaled weight / activation formats and their PyTorch reference math.

MXFP8 (used for every dense / expert GEMM operand):
  * data: float8_e4m3fn [R, K];
  * scale: one UE8M0 byte per 32 consecutive K elements of a row
    (value 2**(byte-127)), chosen as the smallest power of two with
    amax/scale <= 448 so quantization never saturates;
  * the scale bytes are stored in the tcgen05 scale-factor tile layout
    ("sf128x4"): rows are padded to a multiple of 128 and K/32 scale columns
    are grouped by 4; chunk (row_block, k_chunk) is 512 contiguous bytes in
    which row rb*128 + 32*j + i, scale column 4*kc + c sits at byte
    16*i + 4*j + c.  A GEMM stage of 128 rows x 128 K copies one chunk
    straight into tensor memory with `tcgen05.cp ... 32x128b.warpx4`.

NVFP4 (routed experts in the NVFP4 configuration): e2m1 pairs packed in bytes,
one e4m3 scale per 16 K elements, one fp32 global scale per tensor.

Block-FP8 checkpoints ship e4m3 weights with one scale per block of rows x
columns (`weight_scale_inv`): DeepSeek-V3 uses fp32 scales on 128x128 blocks,
the V4 family UE8M0 (power-of-two) scales on 32x32 blocks.
:func:`dequant_blocked` reads either (the block shape follows from the two
tensors' shapes); the loaders requantize the result to the serving formats.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

E4M3_MAX = 448.0
E2M1_MAX = 6.0
SF_ROWS = 128      # rows per scale-factor chunk
SF_KCHUNK = 128    # K elements per scale-factor chunk (4 blocks of 32)


def round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


# ---------------------------------------------------------------------------
# UE8M0 scale selection
# ---------------------------------------------------------------------------

def ue8m0_ceil_exponent(ratio: torch.Tensor) -> torch.Tensor:
    """ceil(log2(ratio)) for ratio > 0 computed exactly from float32 bits;
    ratio == 0 maps to -127.  Result clamped to [-127, 127]."""
    r = ratio.float().contiguous()
    bits = r.view(torch.int32)
    e = ((bits >> 23) & 0xFF) - 127
    mant = bits & 0x7FFFFF
    e = torch.where(mant != 0, e + 1, e)
    e = torch.where(r > 0, e, torch.full_like(e, -127))
    return e.clamp(-127, 127)


# ---------------------------------------------------------------------------
# sf128x4 layout packing
# ---------------------------------------------------------------------------

def sf_packed_size(rows: int, k: int) -> int:
    return round_up(rows, SF_ROWS) * (k // 32)


def pack_sf(sf: torch.Tensor) -> torch.Tensor:
    """[R, K/32] uint8 (row-major) -> flat sf128x4 layout (uint8)."""
    R, KB = sf.shape
    assert KB % 4 == 0, "K must be a multiple of 128"
    Rp = round_up(R, SF_ROWS)
    if Rp != R:
        sf = torch.cat([sf, torch.full((Rp - R, KB), 127, dtype=sf.dtype, device=sf.device)], 0)
    # [rb, j, i, kc, c] -> [rb, kc, i, j, c]
    t = sf.view(Rp // 128, 4, 32, KB // 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return t.view(-1)


def unpack_sf(packed: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """Inverse of :func:`pack_sf` -> [rows, K/32] uint8."""
    Rp = round_up(rows, SF_ROWS)
    KB = k // 32
    t = packed.view(Rp // 128, KB // 4, 32, 4, 4).permute(0, 3, 2, 1, 4).contiguous()
    return t.view(Rp, KB)[:rows]


def tile_rows128(data: torch.Tensor) -> torch.Tensor:
    """[..., R, C] bytes (R, C multiples of 128) -> the same bytes stored as
    contiguous 128-row x 128-byte tiles, tile order (row block, column block),
    returned with the original shape.  The grouped GEMM reads such weights
    with one contiguous 16 KB block per TMA box."""
    *lead, R, C = data.shape
    t = data.reshape(*lead, R // 128, 128, C // 128, 128).transpose(-3, -2).contiguous()
    return t.reshape(*lead, R, C)


def untile_rows128(data: torch.Tensor) -> torch.Tensor:
    *lead, R, C = data.shape
    t = data.reshape(*lead, R // 128, C // 128, 128, 128).transpose(-3, -2).contiguous()
    return t.reshape(*lead, R, C)


# ---------------------------------------------------------------------------
# MXFP8 tensors
# ---------------------------------------------------------------------------

@dataclass
class MXFP8Tensor:
    """Row-wise MXFP8 matrix: data [R, K] e4m3, scales in sf128x4 layout.
    ``rows`` is the logical row count when R was padded to a multiple of 128."""
    data: torch.Tensor
    sf: torch.Tensor
    rows: Optional[int] = None

    @property
    def shape(self):
        return self.data.shape

    def dequant(self) -> torch.Tensor:
        return dequant_mxfp8(self.data, self.sf)


def quant_mxfp8_ref(x: torch.Tensor, packed: bool = True):
    """Reference MXFP8 quantization of x [R, K] (K % 128 == 0).

    Returns (data e4m3 [R, K], scales uint8 packed sf128x4 or [R, K/32])."""
    R, K = x.shape
    xb = x.float().view(R, K // 32, 32)
    amax = xb.abs().amax(-1)
    e = ue8m0_ceil_exponent(amax / E4M3_MAX)
    inv = torch.pow(2.0, -e.float()).unsqueeze(-1)
    q = (xb * inv).view(R, K).to(torch.float8_e4m3fn)
    sf = (e + 127).to(torch.uint8)
    return q, (pack_sf(sf) if packed else sf)


def dequant_mxfp8(q: torch.Tensor, sf: torch.Tensor, packed: bool = True) -> torch.Tensor:
    R, K = q.shape
    s = unpack_sf(sf, R, K) if packed else sf
    scale = torch.pow(2.0, s.float() - 127.0)
    return (q.float().view(R, K // 32, 32) * scale.unsqueeze(-1)).view(R, K)


def block_scales_float(s: torch.Tensor) -> torch.Tensor:
    """A checkpoint's block scales as fp32 multipliers: float tensors as they
    are, UE8M0 bytes (float8_e8m0fnu, or raw uint8) as 2**(byte - 127)."""
    e8m0 = getattr(torch, "float8_e8m0fnu", None)
    if s.dtype == torch.uint8 or (e8m0 is not None and s.dtype == e8m0):
        e = s.view(torch.uint8).to(torch.int32) - 127
        return torch.ldexp(torch.ones(e.shape, dtype=torch.float32, device=s.device), e)
    return s.float()


def _block_edge(n: int, nb: int) -> int:
    """The block size along a dimension of n elements cut into nb blocks:
    the smallest power of two b with ceil(n / b) == nb."""
    b = 1
    while (n + b - 1) // b > nb:
        b *= 2
    if (n + b - 1) // b != nb:
        raise ValueError(f"{nb} scale blocks do not tile {n} elements with a power-of-two block")
    return b


def dequant_blocked(w: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """fp32 [N, K] of a block-FP8 weight: e4m3 w [N, K] times its block
    scales [ceil(N/bn), ceil(K/bk)] (fp32 or UE8M0; bn x bk = 128 x 128,
    32 x 32, ... inferred from the shapes)."""
    N, K = w.shape
    sn, sk = scale.shape
    bn, bk = _block_edge(N, sn), _block_edge(K, sk)
    s = block_scales_float(scale).repeat_interleave(bn, 0)[:N].repeat_interleave(bk, 1)[:, :K]
    return w.float() * s


def mxfp8_from_blocked(w: torch.Tensor, scale: torch.Tensor) -> MXFP8Tensor:
    """A block-FP8 checkpoint weight [N, K] as MXFP8 (dequantize, then
    requantize per 32 along K)."""
    q, sf = quant_mxfp8_ref(dequant_blocked(w, scale))
    return MXFP8Tensor(q, sf)


# ---------------------------------------------------------------------------
# NVFP4
# ---------------------------------------------------------------------------

_E2M1_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def _e2m1_encode(v: torch.Tensor) -> torch.Tensor:
    """Round |v| <= 6 to the nearest e2m1 value (ties to even code); 4-bit codes."""
    a = v.abs().clamp(max=E2M1_MAX)
    grid = _E2M1_GRID.to(v.device)
    d = (a.unsqueeze(-1) - grid).abs()
    # tie-break towards even code index: add a tiny bias to odd indices
    bias = (torch.arange(8, device=v.device) % 2).float() * 1e-7
    code = (d + bias).argmin(-1)
    sign = (v < 0) & (code != 0)
    return (code | (sign.to(torch.int64) << 3)).to(torch.uint8)


def _e2m1_decode(c: torch.Tensor) -> torch.Tensor:
    grid = _E2M1_GRID.to(c.device)
    v = grid[(c & 7).long()]
    return torch.where((c & 8) != 0, -v, v)


@dataclass
class NVFP4Tensor:
    """NVFP4 matrix (or a stack of E matrices): data uint8 [..., R, K/2]
    packed e2m1 pairs (low nibble = even element); sf uint8 [..., packed] e4m3
    scales per 16 elements in the same 128-row x 4-column chunk layout as the
    MXFP8 scales (K/16 scale columns); global_scale fp32 [...] (per matrix).
    ``rows`` is the logical row count when R was padded to a multiple of 128."""
    data: torch.Tensor
    sf: torch.Tensor
    global_scale: torch.Tensor
    rows: Optional[int] = None

    @property
    def shape(self):
        d = self.data.shape
        return (*d[:-1], d[-1] * 2)

    def dequant(self) -> torch.Tensor:
        return dequant_nvfp4(self.data, self.sf, self.global_scale)


def _nvfp4_encode(x: torch.Tensor, g: torch.Tensor):
    """x [R, K] fp32, g [R, 1] global scales -> (packed codes [R, K/2],
    e4m3 block scales [R, K/16])."""
    R, K = x.shape
    xb = x.view(R, K // 16, 16)
    amax = xb.abs().amax(-1)
    s = (amax / (E2M1_MAX * g)).to(torch.float8_e4m3fn)
    denom = (s.float() * g).unsqueeze(-1)
    v = torch.where(denom > 0, xb / denom, torch.zeros_like(xb)).view(R, K)
    codes = _e2m1_encode(v)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).to(torch.uint8)
    return packed, s


def quant_nvfp4_ref(x: torch.Tensor, global_scale: Optional[torch.Tensor] = None) -> NVFP4Tensor:
    """Weight-style NVFP4: one global scale for the matrix (amax / (448*6)
    unless given), rows padded to a multiple of 128 (zeros)."""
    R, K = x.shape
    xf = x.float()
    if global_scale is None:
        global_scale = (xf.abs().amax() / (E4M3_MAX * E2M1_MAX)).clamp(min=1e-12)
    g = global_scale.float().reshape(())
    Rp = round_up(R, SF_ROWS)
    if Rp != R:
        xf = torch.cat([xf, xf.new_zeros(Rp - R, K)], 0)
    packed, s = _nvfp4_encode(xf, g.view(1, 1).expand(Rp, 1))
    return NVFP4Tensor(packed, pack_sf(s.view(torch.uint8)), g, R)


def quant_nvfp4_rows(x: torch.Tensor, global_scale: Optional[float] = None):
    """Activation-style NVFP4: per-row global scale g_r = amax_r / (448*6)
    (or one fixed value).  Returns (packed [R, K/2], sf packed, g [R])."""
    R, K = x.shape
    xf = x.float()
    if global_scale is None:
        am = xf.abs().amax(-1)
        g = torch.where(am > 0, am / (E4M3_MAX * E2M1_MAX), torch.ones_like(am))
    else:
        g = torch.full((R,), float(global_scale), dtype=torch.float32, device=x.device)
    packed, s = _nvfp4_encode(xf, g.view(R, 1))
    return packed, pack_sf(s.view(torch.uint8)), g


def dequant_nvfp4_rows(data: torch.Tensor, sf: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    """Inverse of quant_nvfp4_rows / quant_nvfp4_ref (g per row or scalar)."""
    R = data.shape[0]
    K = data.shape[1] * 2
    lo = _e2m1_decode(data & 0xF)
    hi = _e2m1_decode(data >> 4)
    v = torch.stack([lo, hi], -1).view(R, K)
    s = unpack_sf(sf, R, K * 2).view(torch.float8_e4m3fn).float()       # [R, K/16] (K/16 = 2K/32 columns)
    gg = g.float().reshape(-1, 1) if g.dim() > 0 else g.float()
    return (v.view(R, K // 16, 16) * s.unsqueeze(-1)).view(R, K) * gg


def dequant_nvfp4(data: torch.Tensor, sf: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    if data.dim() == 3:
        return torch.stack([dequant_nvfp4(data[e], sf[e], g[e]) for e in range(data.shape[0])])
    return dequant_nvfp4_rows(data, sf, g)
