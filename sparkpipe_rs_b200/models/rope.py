"""Rotary tables (plain and YaRN) shared by the kernels and the fp32 oracle.

Convention: adjacent pairs (x[2i], x[2i+1]) rotate by angle pos * inv_freq[i];
the table row for position p holds rope/2 cosines followed by rope/2 sines
(fp32), which is what the sm_100a kernels read.

YaRN frequency blending follows Peng et al., "YaRN: Efficient Context Window
Extension of Large Language Models" (2023): wavelengths below the beta_fast
boundary keep the base frequency, those above beta_slow are interpolated by
`factor`, with a linear ramp in between; the attention-logit scale is handled
by ``MLAMoEConfig.softmax_scale``.
"""
from __future__ import annotations

import math

import torch

from .config import MLAMoEConfig, yarn_mscale


def _yarn_correction_dim(num_rot: float, dim: int, base: float, max_pos: int) -> float:
    return (dim * math.log(max_pos / (num_rot * 2 * math.pi))) / (2 * math.log(base))


def inv_frequencies(cfg: MLAMoEConfig) -> torch.Tensor:
    dim = cfg.qk_rope_head_dim
    base = cfg.rope_theta
    freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    rs = cfg.rope_scaling
    if not rs or rs.get("type", "yarn") != "yarn" or rs.get("factor", 1.0) <= 1.0:
        return freq
    factor = rs["factor"]
    orig = rs.get("original_max_position_embeddings", 4096)
    lo = math.floor(_yarn_correction_dim(rs.get("beta_fast", 32.0), dim, base, orig))
    hi = math.ceil(_yarn_correction_dim(rs.get("beta_slow", 1.0), dim, base, orig))
    lo, hi = max(lo, 0), min(hi, dim - 1)
    if lo == hi:
        hi += 0.001
    ramp = ((torch.arange(dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0, 1)
    extrapolate = 1.0 - ramp  # 1 -> keep the base frequency
    return freq / factor * (1 - extrapolate) + freq * extrapolate


def cos_sin_table(cfg: MLAMoEConfig, max_pos: int, device=None) -> torch.Tensor:
    """[max_pos, rope] fp32: cos then sin of pos * inv_freq (times the YaRN cos/sin mscale)."""
    inv = inv_frequencies(cfg)
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(pos, inv)
    m = 1.0
    rs = cfg.rope_scaling
    if rs and rs.get("factor", 1.0) > 1.0:
        # yarn_mscale(f, 0) == 1, so a missing mscale_all_dim leaves the plain mscale
        m = yarn_mscale(rs["factor"], rs.get("mscale", 1.0)) / yarn_mscale(rs["factor"], rs.get("mscale_all_dim", 0.0))
    tab = torch.cat([ang.cos() * m, ang.sin() * m], dim=1).to(torch.float32)
    return tab.to(device) if device is not None else tab


def apply_rope(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor) -> torch.Tensor:
    """Reference rotation of the last dim of x ([..., rope]) at positions pos ([T]) — fp32."""
    half = x.shape[-1] // 2
    cs = table[pos.long()]
    cos, sin = cs[:, :half], cs[:, half:]
    while cos.dim() < x.dim():
        cos = cos.unsqueeze(-2)
        sin = sin.unsqueeze(-2)
    x0 = x[..., 0::2].float()
    x1 = x[..., 1::2].float()
    y0 = x0 * cos - x1 * sin
    y1 = x0 * sin + x1 * cos
    return torch.stack([y0, y1], dim=-1).flatten(-2)
