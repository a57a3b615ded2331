"""CPU: column sharding and the output all-gather over two gloo ranks.

The per-rank GEMM in these multi-process tests is the CPU oracle (the product GEMM is
GPU-only); what is under test is the host logic around it: which rows of the packed
weights and scales each rank owns, and that gathering the per-rank outputs
reproduces the single-device result exactly.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from arc import parallel


def test_column_range():
    assert parallel.column_range(4096, 0, 2) == (0, 2048)
    assert parallel.column_range(4096, 1, 2) == (2048, 4096)
    assert parallel.column_range(28672, 7, 8) == (25088, 28672)
    with pytest.raises(ValueError):
        parallel.column_range(100, 0, 3)
    with pytest.raises(ValueError):
        parallel.column_range(4096, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_gemm(a, b):
    from oracle import oracle

    (x, sa), (wp, sb) = a, b
    out = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.contiguous().numpy(),
                          sb.contiguous().view(torch.int16).numpy().view(np.uint16))
    return torch.from_numpy(out.astype(np.float32)).to(torch.bfloat16)


def _worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "arc-gemm_b200"), str(root)]
    from arc import parallel as par
    from arc.testing.data import generate_a8w4

    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        a, b = generate_a8w4(6, 64, 256, seed=3)
        b_local = par.shard_weights(b, rank, world)
        full = par.sharded_gemm(_oracle_gemm, a, b_local, world=world, all_gather=True)
        local = par.sharded_gemm(_oracle_gemm, a, b_local, world=world, all_gather=False)
        result_q.put((rank, full.view(torch.int16).numpy().copy(),
                      local.view(torch.int16).numpy().copy()))
    finally:
        dist.destroy_process_group()


def test_sharded_a8w4_all_gather_two_ranks():
    from arc.testing.data import generate_a8w4

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, full, local = q.get(timeout=120)
        results[r] = (full, local)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    a, b = generate_a8w4(6, 64, 256, seed=3)
    single = _oracle_gemm(a, b).view(torch.int16).numpy()
    for r in range(world):
        full, local = results[r]
        assert np.array_equal(full, single)
        lo, hi = parallel.column_range(64, r, world)
        assert np.array_equal(local, single[:, lo:hi])


def test_ipc_mappings_open_once_per_handle(monkeypatch):
    """FusedGather's peer mappings: a process opens each exported allocation once (CUDA
    allows one mapping per handle and process), shares it between users at their own
    offsets, and closes it when the last user goes. The library is a fake here."""
    from arc import _lib

    calls = []

    class FakeLib:
        def arc_ipc_open(self, handle, offset, ptr, base):
            calls.append(("open", bytes(handle), offset))
            ptr._obj.value = 0x10000 + offset
            base._obj.value = 0x10000
            return 0

        def arc_ipc_close(self, base):
            calls.append(("close", base))
            return 0

    monkeypatch.setattr(_lib, "lib", lambda: FakeLib())
    monkeypatch.setattr(parallel, "_OPENED", {})
    h = bytes(range(64))
    p1, k1 = parallel._ipc_open(h, 256)
    p2, k2 = parallel._ipc_open(h, 4096)
    assert (p1, p2) == (0x10000 + 256, 0x10000 + 4096)
    assert calls == [("open", h, 0)]
    parallel._ipc_close(k1)
    assert len(calls) == 1
    parallel._ipc_close(k2)
    assert calls[-1] == ("close", 0x10000)
    assert parallel._OPENED == {}
