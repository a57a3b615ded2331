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


# ------------------------------------------------------------------ FP8 x FP4 recipe
# The quantisation of the reference's A8W4 test (tests/a8w4.py:29-30): e4m3
# activations with one power-of-two (UE8M0) scale per token and 128-wide K block, e2m1
# weights with one per row and 32-wide K block. Restated from
# arc/testing/quant.py:16-19 (ceil_to_ue8m0), :30-48 (per_token_cast_to_fp8),
# :51-58 (e2m1 rounding), :61-84 (per_token_cast_to_fp4) and arc/math.py:148-170
# (the e2m1 decode used by cast_back_from_fp4).
FP8_E4M3_MAX = 448.0
FP4_E2M1_MAX = 6.0
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_E2M1_EDGES = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)  # rounding boundaries between values


def ceil_to_ue8m0(s: torch.Tensor) -> torch.Tensor:
    """Smallest power of two >= |s| (biased exponent clamped to [1, 254]), as fp32."""
    bits = s.abs().float().view(torch.int32)
    exp = ((bits >> 23) & 0xFF) + ((bits & 0x7FFFFF) != 0).to(torch.int32)
    return (exp.clamp(1, 254) << 23).view(torch.float32)


def _blocks(x: torch.Tensor, gran_k: int) -> torch.Tensor:
    """[M, K] -> zero-padded [M, ceil(K/gran_k), gran_k] view."""
    m, k = x.shape
    kp = -(-k // gran_k) * gran_k
    xp = torch.zeros((m, kp), dtype=x.dtype, device=x.device)
    xp[:, :k] = x
    return xp.view(m, kp // gran_k, gran_k)


def per_token_cast_to_fp8(x: torch.Tensor, *, use_ue8m0: bool = True, gran_k: int = 128) -> TensorPair:
    """x [M, K] -> (float8_e4m3fn [M, K], fp32 scale [M, ceil(K/gran_k)])."""
    if x.dim() != 2:
        raise ValueError("per-token fp8 casting expects a 2D tensor")
    view = _blocks(x, gran_k)
    sf = view.abs().float().amax(dim=2).clamp(1e-4) / FP8_E4M3_MAX
    if use_ue8m0:
        sf = ceil_to_ue8m0(sf)
    q = (view * (1.0 / sf.unsqueeze(2))).to(torch.float8_e4m3fn)
    return q.view(x.shape[0], -1)[:, : x.shape[1]].contiguous(), sf


def _round_to_e2m1(v: torch.Tensor) -> torch.Tensor:
    """fp32 -> e2m1 code (magnitude index 0..7, bit 3 = sign, no negative zero)."""
    edges = torch.tensor(_E2M1_EDGES, dtype=torch.float32, device=v.device)
    idx = torch.bucketize(v.abs().clamp_max(FP4_E2M1_MAX).float(), edges)
    neg = (v < 0) & (idx != 0)
    return idx.to(torch.uint8) | (neg.to(torch.uint8) << 3)


def per_token_cast_to_fp4(x: torch.Tensor, *, use_ue8m0: bool = True, gran_k: int = 32) -> TensorPair:
    """x [N, K] -> (packed e2m1 uint8 [N, K/2], fp32 scale [N, ceil(K/gran_k)])."""
    if x.dim() != 2:
        raise ValueError("per-token fp4 casting expects a 2D tensor")
    if x.shape[1] % 2 != 0:
        raise ValueError("packed fp4 casting expects an even K")
    view = _blocks(x, gran_k)
    sf = view.abs().float().amax(dim=2).clamp_min(1e-4) / FP4_E2M1_MAX
    if use_ue8m0:
        sf = ceil_to_ue8m0(sf)
    codes = _round_to_e2m1(view * (1.0 / sf.unsqueeze(2))).view(x.shape[0], -1)
    packed = codes[:, 0::2] | (codes[:, 1::2] << 4)
    return packed[:, : x.shape[1] // 2].contiguous(), sf


def dequantize_fp4(packed: torch.Tensor, sf: torch.Tensor, gran_k: int = 32) -> torch.Tensor:
    """(packed e2m1 [N, K/2], fp32 scale [N, K/gran_k]) -> fp32 [N, K]."""
    p = packed.to(torch.uint8)
    codes = torch.stack((p & 0x0F, p >> 4), dim=-1).flatten(-2)
    table = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=p.device)
    mag = table[(codes & 0x07).long()]
    val = torch.where((codes & 0x08) != 0, -mag, mag)
    return val * sf.float().repeat_interleave(gran_k, dim=1)[:, : val.shape[1]]
