"""The timeout path of the kernels' bounded waits, made to run out on purpose.

Every wait in the library is bounded; when one runs out the kernel records a bit in the
device status word (arc_device_status) and returns, instead of hanging the GPU or exiting
the process as the reference does on errors (arc/include/common.cuh:8-28). Here the
peer barrier of the fused all-gather waits for a peer that never announces: one process,
one GPU, rank 0 of a world of two whose second flag array nobody writes, with a 50 ms
limit. The kernel must return, report kStatusTimeoutPeer, and leave the GPU working (a
following GEMM matches the oracle).
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

import arc
from arc import _lib
from arc.testing.data import generate_a8w4
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_peer_barrier_times_out_and_reports(cuda_device):
    dev = cuda_device
    L = _lib.lib()
    arc.device_status(0)  # clear
    world = 2
    flags = [torch.zeros(world + 1, dtype=torch.int32, device=dev) for _ in range(world)]
    arr = (ctypes.c_void_p * world)(*[f.data_ptr() for f in flags])
    stream = torch.cuda.current_stream(dev).cuda_stream
    t0 = time.perf_counter()
    assert L.arc_peer_barrier_ex(arr, world, 0, 50_000_000, ctypes.c_void_p(stream)) == _lib.ARC_OK, \
        L.arc_last_error()
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    status = arc.device_status(0)
    assert status & _lib.STATUS_TIMEOUT_PEER, f"status {status:#x}"
    assert 0.04 < waited < 1.9, f"the barrier returned after {waited:.3f} s"
    # Rank 0 announced its epoch in both arrays and counted the barrier.
    assert flags[0][0].item() == 1 and flags[1][0].item() == 1 and flags[0][world].item() == 1
    # The GPU keeps working.
    (x, sa), (wp, sb) = generate_a8w4(16, 256, 512, seed=3)
    out = arc.a8w4_matmul((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)))
    torch.cuda.synchronize()
    assert arc.device_status(0) == 0
    ref = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy(), sb.view(torch.int16).numpy().view(np.uint16))
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref, max_ulp=2.0)
    assert ok, msg


def test_peer_barrier_rejects_bad_limits(cuda_device):
    L = _lib.lib()
    flags = [torch.zeros(3, dtype=torch.int32, device=cuda_device) for _ in range(2)]
    arr = (ctypes.c_void_p * 2)(*[f.data_ptr() for f in flags])
    assert L.arc_peer_barrier_ex(arr, 2, 0, 0, None) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_peer_barrier_ex(arr, 2, 0, 3_000_000_000, None) == _lib.ARC_ERR_INVALID_ARGUMENT
