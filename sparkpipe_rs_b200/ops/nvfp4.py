"""NVFP4 weights: 4-bit E2M1 values in 16-element blocks with one FP8 E4M3 scale per
block and one FP32 scale per tensor (x = e2m1 x block_scale x tensor_scale).

``quant_nvfp4`` packs a bf16 / fp32 weight (rows of K, K a multiple of 16; runs on
any device with torch), ``dequant_nvfp4_ref`` expands it in plain torch (the oracle)
and ``dequant_nvfp4`` expands it with the sm_100a kernel (one thread per block, copy
bandwidth). ``linear_nvfp4`` expands a weight into a reusable bf16 buffer and runs
the GEMM: the storage format for NVFP4 expert checkpoints, whose compute path on
this engine is the bf16 / fp8 tcgen05 GEMMs.

Rounding to E2M1 is to the nearest grid value, ties toward zero; a block's scale is
its absolute maximum over 6 rounded to E4M3; the tensor scale maps the largest block
scale to 448 (the E4M3 maximum).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

_GRID = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
_MIDS = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0])


@dataclass
class Nvfp4Weight:
    packed: torch.Tensor   # uint8 [..., K/2], element 2i in the low nibble
    scales: torch.Tensor   # uint8 (E4M3 bits) [..., K/16]
    tensor_scale: float
    shape: tuple

    @property
    def nbytes(self) -> int:
        return self.packed.numel() + self.scales.numel() + 4


def quant_nvfp4(w: torch.Tensor) -> Nvfp4Weight:
    if w.shape[-1] % 16:
        raise ValueError("quant_nvfp4: the last dimension must be a multiple of 16")
    x = w.float().reshape(-1, 16)
    amax = x.abs().amax(-1)
    tensor_scale = float(amax.max()) / (6.0 * 448.0) if float(amax.max()) > 0 else 1.0
    bscale = (amax / 6.0 / tensor_scale).to(torch.float8_e4m3fn)
    s = bscale.float() * tensor_scale
    v = torch.where(s[:, None] > 0, x / s.clamp_min(1e-30)[:, None], torch.zeros_like(x))
    mag = v.abs().clamp(max=6.0)
    code = torch.bucketize(mag, _MIDS.to(mag.device), right=False).to(torch.uint8)  # ties toward zero
    code = code | ((v < 0) & (code > 0)).to(torch.uint8) << 3
    code = code.reshape(-1, 8, 2)
    packed = (code[..., 0] | (code[..., 1] << 4)).reshape(*w.shape[:-1], w.shape[-1] // 2)
    return Nvfp4Weight(packed.contiguous(), bscale.view(torch.uint8).reshape(*w.shape[:-1], w.shape[-1] // 16).contiguous(),
                       tensor_scale, tuple(w.shape))


def dequant_nvfp4_ref(q: Nvfp4Weight, dtype=torch.float32) -> torch.Tensor:
    p = q.packed.reshape(-1)
    codes = torch.stack([p & 0xF, p >> 4], -1).reshape(-1).long()
    mag = _GRID.to(p.device)[codes & 7]
    val = torch.where(codes & 8 > 0, -mag, mag).reshape(-1, 16)
    s = q.scales.reshape(-1).view(torch.float8_e4m3fn).float() * q.tensor_scale
    return (val * s[:, None]).reshape(q.shape).to(dtype)


def dequant_nvfp4(q: Nvfp4Weight, out: torch.Tensor | None = None) -> torch.Tensor:
    from . import _count, kernels

    if out is None:
        out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.packed.device)
    kernels().dequant_nvfp4(q.packed, q.scales, float(q.tensor_scale), out)
    _count(1)
    return out


def linear_nvfp4(x: torch.Tensor, q: Nvfp4Weight, scratch: torch.Tensor | None = None) -> torch.Tensor:
    """x [T, K] bf16 @ W^T for an NVFP4 weight W [N, K]."""
    w = dequant_nvfp4(q, scratch)
    return x @ w.t()
