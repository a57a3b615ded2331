"""Quantizers and the int4 packing format of the A8W4 recipe (host-side torch code).

Mirrors the role of the reference's arc/testing/quant.py (per-token / per-group casts
returning (data, scale) pairs, `TensorPair`, quant.py:10) for the int8 x int4 recipe:

* activations: int8 in [-127, 127] with one fp32 scale per token (row);
* weights: int4 in [-8, 7] with one bf16 scale per (column, 128-wide K group), two
  codes per byte along K, the even k in the LOW nibble — the byte layout the
  reference's fp4 packer writes (quant.py:82-83:
  `(codes[..., 0] & 0x0F) | ((codes[..., 1] & 0x0F) << 4)`).

These run wherever the tensors live (CPU or GPU); the GEMM itself is GPU-only.
"""
from __future__ import annotations

from typing import TypeAlias

import torch

TensorPair: TypeAlias = tuple[torch.Tensor, torch.Tensor]

INT8_MAX = 127.0
INT4_MAX = 7.0


def pack_int4(codes: torch.Tensor) -> torch.Tensor:
    """[..., K] integer codes in [-8, 7] -> [..., K/2] uint8 (even k in the low nibble)."""
    if codes.shape[-1] % 2 != 0:
        raise ValueError("packing int4 needs an even K")
    c = codes.to(torch.int16)
    if bool(((c < -8) | (c > 7)).any()):
        raise ValueError("int4 codes must lie in [-8, 7]")
    nib = (c & 0x0F).to(torch.uint8)
    return nib[..., 0::2] | (nib[..., 1::2] << 4)


def unpack_int4(packed: torch.Tensor) -> torch.Tensor:
    """[..., K/2] uint8 -> [..., K] int8 codes in [-8, 7]."""
    p = packed.to(torch.uint8)
    lo = (p & 0x0F).to(torch.int16)
    hi = (p >> 4).to(torch.int16)
    codes = torch.stack((lo, hi), dim=-1).flatten(-2)
    return torch.where(codes >= 8, codes - 16, codes).to(torch.int8)


def per_token_cast_to_int8(x: torch.Tensor) -> TensorPair:
    """x [M, K] float -> (int8 [M, K], fp32 scale [M]); x ~= q * scale per row."""
    if x.dim() != 2:
        raise ValueError("per-token int8 casting expects a 2D tensor")
    amax = x.abs().float().amax(dim=1).clamp(min=1e-4)
    sa = amax / INT8_MAX
    q = torch.round(x.float() / sa.unsqueeze(1)).clamp(-INT8_MAX, INT8_MAX).to(torch.int8)
    return q.contiguous(), sa.contiguous()


def per_group_cast_to_int4(w: torch.Tensor, gran_k: int = 128) -> TensorPair:
    """w [N, K] float -> (packed uint8 [N, K/2], bf16 scale [N, K/gran_k]).

    The bf16 scale is chosen first (amax/7 rounded to bf16) and the codes are
    rounded against that stored scale, so dequantization uses exactly what the GEMM
    sees.
    """
    if w.dim() != 2:
        raise ValueError("per-group int4 casting expects a 2D tensor")
    n, k = w.shape
    if k % gran_k != 0:
        raise ValueError(f"K ({k}) must be a multiple of gran_k ({gran_k})")
    view = w.float().view(n, k // gran_k, gran_k)
    sb = (view.abs().amax(dim=2).clamp(min=1e-4) / INT4_MAX).to(torch.bfloat16)
    q = torch.round(view / sb.float().unsqueeze(2)).clamp(-8, 7).to(torch.int8).view(n, k)
    return pack_int4(q).contiguous(), sb.contiguous()


def dequantize_int4(packed: torch.Tensor, sb: torch.Tensor, gran_k: int = 128) -> torch.Tensor:
    """(packed [N, K/2], sb [N, K/gran_k]) -> fp32 [N, K]."""
    codes = unpack_int4(packed).float()
    n, k = codes.shape
    return (codes.view(n, k // gran_k, gran_k) * sb.float().unsqueeze(2)).view(n, k)


__all__ = [
    "TensorPair",
    "pack_int4",
    "unpack_int4",
    "per_token_cast_to_int8",
    "per_group_cast_to_int4",
    "dequantize_int4",
]
