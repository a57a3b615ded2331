"""Column (N) sharding of the GEMMs across the GPUs of one node.

The reference has no multi-GPU code. The weight matrix shards naturally along N:
columns and their scales are independent, so rank r of g owns
W[r*N/g:(r+1)*N/g, :] (and the matching rows of sb), the activations are
replicated, and rank r computes out[:, r*N/g:(r+1)*N/g] with no exchange inside the
GEMM. The only collective is the optional all-gather of the bf16 output: either
`torch.distributed.all_gather_into_tensor` over NCCL (NVLink/NVSwitch), which lands as
[g, M, N/g] and is re-laid out to [M, N], or, for decode batches, fused into the GEMM's
epilogue (FusedGather: each rank's kernel stores its tiles straight into every rank's
output over peer memory, then a flag barrier).

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


# Peer mappings opened by this process, by handle: a process may open each exported
# allocation only once, so FusedGather objects that map the same peer segment share it.
_OPENED: dict[bytes, list] = {}  # handle -> [mapping base, users]


def _ipc_open(handle: bytes, offset: int) -> tuple[int, bytes]:
    import ctypes

    from ._lib import check, lib

    entry = _OPENED.get(handle)
    if entry is None:
        ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
        check(lib().arc_ipc_open(handle, 0, ctypes.byref(ptr), ctypes.byref(base)), "arc_ipc_open")
        entry = _OPENED[handle] = [base.value, 0]
    entry[1] += 1
    return entry[0] + offset, handle


def _ipc_close(handle: bytes) -> None:
    from ._lib import check, lib

    entry = _OPENED[handle]
    entry[1] -= 1
    if entry[1] == 0:
        del _OPENED[handle]
        check(lib().arc_ipc_close(entry[0]), "arc_ipc_close")


class FusedGather:
    """Every rank's gathered output, mapped into this process, for the A8W4 decode GEMM
    with the all-gather fused into its epilogue (`arc_a8w4_gemm_gather`).

    Collective: every rank of `group` (one process per GPU, all GPUs of one node, each
    process seeing every GPU with the same numbering) builds it with the same `m` and
    `n_total`. Each rank allocates one buffer holding its [m, n_total] bf16 output and a
    small flag array, exports it with CUDA IPC (`arc_ipc_export`, handles exchanged with
    `all_gather_object`) and maps the others' into its own GPU's context (`arc_ipc_open`,
    which enables peer access from this GPU), so its GEMM can store its column block into
    every rank's output over NVLink and a flag barrier (`arc_peer_barrier`, or folded into
    the GEMM's last CTA with `one_launch=True`, `arc_a8w4_gemm_gather_sync`) can tell when
    all blocks have landed. `out` is this rank's gathered output; each `matmul` call overwrites it (and
    the other ranks') with the next result. `close()` (collective) unmaps the peers.
    """

    def __init__(self, m: int, n_total: int, *, group=None, device: torch.device | None = None,
                 one_launch: bool = False):
        import ctypes

        from ._lib import check, lib

        self.group = group
        # The GEMM and a separate barrier kernel (default), or one kernel per step with the
        # barrier folded into the GEMM's last CTA; both give the same output. On 2 B200s
        # the separate barrier measured faster (10.3 vs 18.3 us per decode step): with the
        # fold every CTA must wait for its stores into peer memory to be performed and fence
        # at system scope before it can count itself done, which lengthens every CTA.
        self.one_launch = one_launch
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the fused all-gather spans at most 8 GPUs")
        column_range(n_total, self.rank, self.world)  # validates the split
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.m, self.n_total = m, n_total
        out_bytes = -(-m * n_total * 2 // 256) * 256
        self._buf = torch.zeros(out_bytes + 256, dtype=torch.uint8, device=self.device)
        self.out = self._buf[: m * n_total * 2].view(torch.bfloat16).view(m, n_total)
        # world epoch flags, this rank's barrier counter, then its count of GEMM CTAs done
        self.flags = self._buf[out_bytes: out_bytes + 4 * (self.world + 2)].view(torch.int32)
        torch.cuda.synchronize(self.device)
        handle = ctypes.create_string_buffer(64)
        offset = ctypes.c_uint64()
        with torch.cuda.device(self.device):
            check(lib().arc_ipc_export(self._buf.data_ptr(), handle, ctypes.byref(offset)), "arc_ipc_export")
        mine = (handle.raw, offset.value)
        handles = [None] * self.world
        dist.all_gather_object(handles, mine, group=group)
        self._held = []  # peer handles this object opened
        outs, flags = [], []
        with torch.cuda.device(self.device):
            for i, (h, off) in enumerate(handles):
                if i == self.rank:
                    base = self._buf.data_ptr()
                else:
                    base, key = _ipc_open(h, off)
                    self._held.append(key)
                outs.append(base)
                flags.append(base + out_bytes)
        self._outs = (ctypes.c_void_p * self.world)(*outs)
        self._flags = (ctypes.c_void_p * self.world)(*flags)
        dist.barrier(group=group)  # every mapping exists before any rank writes into it

    def matmul(self, a: TensorPair, b_local: TensorPair, static_weights: bool = False) -> torch.Tensor:
        """This rank's column block of the A8W4 decode GEMM, stored into every rank's
        output, then the barrier after which `out` holds all blocks.
        `static_weights` as in `arc.a8w4_matmul`."""
        from ._lib import A8W4_STATIC_WEIGHTS, check, lib

        x, sa = a
        wp, sb = b_local
        m, k = x.shape
        n = wp.shape[0]
        if m != self.m or n * self.world != self.n_total:
            raise ValueError(f"shape [{m}, {n} x {self.world}] does not match this gather "
                             f"[{self.m}, {self.n_total}]")
        for t in (x, sa, wp, sb):
            if t.device != self.device:
                raise ValueError(f"operand on {t.device}, expected {self.device}")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        gemm_flags = A8W4_STATIC_WEIGHTS if static_weights else 0
        with torch.cuda.device(self.device):
            if self.one_launch:
                # GEMM, peer stores and barrier in one kernel.
                check(lib().arc_a8w4_gemm_gather_sync(x.data_ptr(), sa.data_ptr(), wp.data_ptr(), sb.data_ptr(),
                                                      self._outs, self._flags, self.world, self.rank, m, n, k,
                                                      gemm_flags, stream),
                      "arc_a8w4_gemm_gather_sync")
            else:
                check(lib().arc_a8w4_gemm_gather_ex(x.data_ptr(), sa.data_ptr(), wp.data_ptr(), sb.data_ptr(),
                                                    self._outs, self.world, self.rank, m, n, k, gemm_flags, stream),
                      "arc_a8w4_gemm_gather")
                check(lib().arc_peer_barrier(self._flags, self.world, self.rank, stream), "arc_peer_barrier")
        return self.out

    def close(self) -> None:
        """Collective: wait for this GPU's work, unmap the peers' buffers, and let every
        rank pass only once all ranks have unmapped (so no buffer is freed while mapped)."""
        if self._held is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # no rank still writes into a peer buffer
        with torch.cuda.device(self.device):
            for key in self._held:
                _ipc_close(key)
        self._held = None
        dist.barrier(group=self.group)


__all__ = ["column_range", "shard_weights", "shard_columns", "gather_columns", "sharded_gemm",
           "FusedGather"]
