"""Two GPUs: column-sharded A8W4 GEMM with the NCCL all-gather of the output.

Each rank owns half of the weight columns (arc.parallel.shard_weights), runs the CUDA
GEMM on its slice and all-gathers the bf16 output over NCCL. The gathered result must
equal the single-GPU GEMM of the whole weight matrix bit for bit (the columns are
independent, so sharding changes no arithmetic). Skipped with fewer than 2 GPUs.
"""
from __future__ import annotations

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, m, n, k, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "arc-gemm_b200"), str(root)]
    import numpy as np

    import arc
    from arc import parallel as par
    from arc.testing.data import generate_a8w4
    from oracle import oracle

    def oracle_ok(out, x, sa, wp, sb):
        cols = np.sort(np.random.default_rng(rank).choice(n, size=min(n, 192), replace=False))
        want = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy()[cols],
                               sb.view(torch.int16).numpy().view(np.uint16)[cols])
        ok, _ = oracle.check_bf16_close(out.float().cpu().numpy()[:, cols], want, max_ulp=2.0)
        return ok

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=5)
        a = (x.to(dev), sa.to(dev))
        b_local = par.shard_weights((wp.to(dev), sb.to(dev)), rank, world)
        full = par.sharded_gemm(arc.a8w4_matmul, a, b_local, world=world, all_gather=True)
        torch.cuda.synchronize()
        ref = arc.a8w4_matmul(a, (wp.to(dev), sb.to(dev))) if rank == 0 else None
        torch.cuda.synchronize()
        if rank == 0:
            result_q.put(bool(torch.equal(full, ref)) and oracle_ok(full, x, sa, wp, sb))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (200, 1024, 1024)])
def test_two_gpu_sharded_gemm_with_all_gather(m, n, k):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, n, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        ok = q.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert ok, "sharded + gathered output differs from the single-GPU GEMM or the oracle"
    assert all(p.exitcode == 0 for p in procs)


def _fused_worker(rank, world, port, m, n, k, result_q, one_launch=True):
    """Each rank: its column block through the GEMM with the fused all-gather, twice in a
    row (two barrier epochs). The gathered output must match the CPU oracle on sampled
    columns of every rank's block (within 2 bf16 ulps) and equal the NCCL all-gather of
    the same blocks bit for bit (same kernel, same plan per block)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "arc-gemm_b200"), str(root)]
    import numpy as np

    import arc
    from arc import parallel as par
    from arc.testing.data import generate_a8w4
    from oracle import oracle

    def oracle_ok(out, x, sa, wp, sb):
        cols = np.sort(np.random.default_rng(rank).choice(n, size=min(n, 192), replace=False))
        want = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy()[cols],
                               sb.view(torch.int16).numpy().view(np.uint16)[cols])
        ok, _ = oracle.check_bf16_close(out.float().cpu().numpy()[:, cols], want, max_ulp=2.0)
        return ok

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        fg = par.FusedGather(m, n, device=dev, one_launch=one_launch)
        ok = True
        for seed in (5, 6):
            (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=seed)
            a = (x.to(dev), sa.to(dev))
            b_local = par.shard_weights((wp.to(dev), sb.to(dev)), rank, world)
            ref = par.sharded_gemm(arc.a8w4_matmul, a, b_local, world=world, all_gather=True)
            got = fg.matmul(a, b_local)
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(got, ref)) and arc.device_status(rank) == 0
            ok = ok and oracle_ok(got, x, sa, wp, sb)
            dist.barrier()
        # The same call captured once in a CUDA graph and replayed on new inputs: the
        # barrier's epoch lives on the device, so every replay synchronises afresh.
        (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=7)
        xs, sas, wps, sbs = x.to(dev), sa.to(dev), wp.to(dev), sb.to(dev)
        b_static = par.shard_weights((wps, sbs), rank, world)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fg.matmul((xs, sas), b_static)
        for seed in (8, 9):
            (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=seed)
            for dst, src in ((xs, x), (sas, sa), (wps, wp), (sbs, sb)):
                dst.copy_(src)
            ref = par.sharded_gemm(arc.a8w4_matmul, (xs, sas), b_static, world=world, all_gather=True)
            graph.replay()
            torch.cuda.synchronize()
            ok = ok and bool(torch.equal(fg.out, ref)) and arc.device_status(rank) == 0
            ok = ok and oracle_ok(fg.out, x, sa, wp, sb)
            dist.barrier()
        del graph
        fg.close()
        result_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("one_launch", [True, False])
@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (5, 1040, 1024)])
def test_two_gpu_fused_all_gather(m, n, k, one_launch):
    """The barrier folded into the GEMM's last CTA (one launch per step) and the separate
    barrier kernel give the same, oracle-checked output."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, m, n, k, q, one_launch)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = dict(q.get(timeout=180) for _ in range(world))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(results.values()), f"fused all-gather differs from the oracle or the NCCL all-gather: {results}"
    assert all(p.exitcode == 0 for p in procs)
