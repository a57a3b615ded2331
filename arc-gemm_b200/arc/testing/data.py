"""Seeded synthetic inputs for the GEMM configurations.

Generated on the CPU with a private `torch.Generator`, so a CPU checker and the GPU
see byte-identical inputs, then moved to `device`. Distributions:

* bf16 GEMM: A, B ~ N(0, 1) (tests/matmul.py:14-24 draws the same with torch.randn);
* A8W4: activations uniform int8 in [-127, 127], per-token fp32 scales U(0.01, 0.05);
  weights uniform int4 in [-8, 7] packed two per byte along K (even k in the low
  nibble), per-(column, 128-wide K group) bf16 scales U(0.005, 0.02).
"""
from __future__ import annotations

import torch

from ..quant import pack_int4


def generate_bf16(m: int, n: int, k: int, seed: int = 0, device="cpu"):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn((m, k), generator=g, dtype=torch.float32).to(torch.bfloat16)
    b = torch.randn((n, k), generator=g, dtype=torch.float32).to(torch.bfloat16)
    return a.to(device), b.to(device)


def generate_a8w4(m: int, n: int, k: int, seed: int = 0, device="cpu", group: int = 128):
    """Returns ((x, sa), (wp, sb)) with x int8 [m,k], sa f32 [m], wp u8 [n,k/2], sb bf16."""
    if k % group != 0:
        raise ValueError(f"K ({k}) must be a multiple of {group}")
    g = torch.Generator().manual_seed(seed)
    x = torch.randint(-127, 128, (m, k), generator=g, dtype=torch.int16).to(torch.int8)
    sa = torch.empty(m, dtype=torch.float32).uniform_(0.01, 0.05, generator=g)
    w = torch.randint(-8, 8, (n, k), generator=g, dtype=torch.int16)
    sb = torch.empty((n, k // group), dtype=torch.float32).uniform_(0.005, 0.02,
                                                                    generator=g).to(torch.bfloat16)
    wp = pack_int4(w)
    return (x.to(device), sa.to(device)), (wp.to(device), sb.to(device))


__all__ = ["generate_bf16", "generate_a8w4"]
