"""Column (N) sharding of the GEMMs across the GPUs of one node.

The reference has no multi-GPU code. The weight matrix shards naturally along N:
columns and their scales are independent, so rank r of g owns
W[r*N/g:(r+1)*N/g, :] (and the matching rows of sb), the activations are
replicated, and rank r computes out[:, r*N/g:(r+1)*N/g] with no exchange inside the
GEMM. The only collective is the optional all-gather of the bf16 output
(`torch.distributed.all_gather_into_tensor` over NCCL, i.e. NVLink/NVSwitch),
which lands as [g, M, N/g] and is re-laid out to [M, N].

One process per GPU; the process group comes from `torch.distributed`.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

from .quant import TensorPair


def column_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of the columns rank `rank` owns. N must split into 8-aligned slices."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank/world ({rank}/{world})")
    if n % world != 0 or (n // world) % 8 != 0:
        raise ValueError(f"N={n} does not split into {world} slices of a multiple of 8 columns")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_weights(b: TensorPair, rank: int, world: int) -> TensorPair:
    """The (packed weights, scales) rows this rank owns (views, no copy)."""
    wp, sb = b
    lo, hi = column_range(wp.shape[0], rank, world)
    return wp[lo:hi], sb[lo:hi]


def shard_columns(b: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """The rows of a K-major bf16 weight [N, K] this rank owns (a view)."""
    lo, hi = column_range(b.shape[0], rank, world)
    return b[lo:hi]


def gather_columns(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather per-rank column blocks [M, N/g] into the full [M, N] output."""
    m, nl = local.shape
    if world == 1:
        return local
    # Rank blocks land one after another along dim 0 ([g*M, N/g], accepted by NCCL
    # and gloo alike), then are re-laid out so rank r's block becomes columns
    # [r*N/g, (r+1)*N/g).
    stacked = torch.empty((world * m, nl), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(stacked, local.contiguous(), group=group)
    return stacked.view(world, m, nl).permute(1, 0, 2).reshape(m, world * nl)


def sharded_gemm(local_gemm: Callable[..., torch.Tensor], a, b_local, *, world: int,
                 all_gather: bool = False, group=None) -> torch.Tensor:
    """Run this rank's column block and optionally all-gather the full output.

    `local_gemm(a, b_local)` is the per-GPU GEMM (arc.a8w4_matmul or arc.matmul).
    """
    out_local = local_gemm(a, b_local)
    if not all_gather:
        return out_local
    return gather_columns(out_local, world, group=group)


__all__ = ["column_range", "shard_weights", "shard_columns", "gather_columns", "sharded_gemm"]
