"""The allocation-free FP8 x FP4 entry point, arc_fp8_fp4_gemm_noalloc, called through the C ABI.

Some callers cannot allocate device memory: operator plugins whose host framework budgets
all of it and passes the operator only its input and output tensors, and hosts that must
not call cudaMalloc on the request path. For them the library keeps the K-split scratch of
decode-sized FP8 x FP4 problems in a fixed 4 MiB device array of its own. These tests check
that entry point against the CPU oracle (oracle.fp8fp4_out) and against the existing entry
point (arc_fp8_fp4_gemm, which runs without a K split) on the same operands, twice in a row
(the scratch keeps the previous call's contents, so the second call shows that it starts
clean). A shape whose split would need more than the array holds runs unsplit and is
checked the same way. This file is collected last, so a run that stops at the first failure
has run every other test before it.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from arc import _lib, quant
from oracle import oracle


def _operands(m, n, k, seed, dev):
    g = torch.Generator().manual_seed(seed)
    a = quant.per_token_cast_to_fp8(torch.randn(m, k, generator=g).to(torch.bfloat16),
                                    use_ue8m0=True, gran_k=128)
    b = quant.per_token_cast_to_fp4(torch.randn(n, k, generator=g).to(torch.bfloat16),
                                    use_ue8m0=True, gran_k=32)
    return tuple(t.to(dev) for t in (a[0], a[1], b[0], b[1]))


def _call(fn, ops, out, m, n, k, dev):
    x, sfa, wp, sfw = ops
    return fn(x.data_ptr(), sfa.data_ptr(), wp.data_ptr(), sfw.data_ptr(), out.data_ptr(), m, n, k,
              ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))


def _oracle(ops, rows=None, cols=None):
    x, sfa, wp, sfw = (t.cpu() for t in ops)
    x8 = x.view(torch.uint8).numpy()
    sfa, wp, sfw = sfa.numpy(), wp.numpy(), sfw.numpy()
    if rows is not None:
        x8, sfa = x8[rows], sfa[rows]
    if cols is not None:
        wp, sfw = wp[cols], sfw[cols]
    return oracle.fp8fp4_out(x8, sfa, wp, sfw)


def _check_twice(dev, m, n, k, seed, rows=None, cols=None):
    L = _lib.lib()
    ops = _operands(m, n, k, seed=seed, dev=dev)
    ref = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
    assert _call(L.arc_fp8_fp4_gemm, ops, ref, m, n, k, dev) == _lib.ARC_OK, L.arc_last_error()
    want = _oracle(ops, rows, cols)
    sel = (slice(None) if rows is None else rows, slice(None) if cols is None else cols)
    for call in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        assert _call(L.arc_fp8_fp4_gemm_noalloc, ops, out, m, n, k, dev) == _lib.ARC_OK, \
            L.arc_last_error()
        torch.cuda.synchronize()
        assert _lib.device_status(dev.index) == 0, "kernel reported a wait timeout"
        got = out.double().cpu().numpy()
        ok, msg = oracle.check_bf16_close(got[np.ix_(*[np.arange(d)[s] for d, s in zip((m, n), sel)])],
                                          want, max_ulp=2.0, atol=oracle.tensor_core_atol(k, want))
        assert ok, f"{m}x{n}x{k} call {call} vs oracle: {msg}"
        ref64 = ref.double().cpu().numpy()
        ok, msg = oracle.check_bf16_close(got, ref64, max_ulp=2.0, atol=oracle.tensor_core_atol(k, ref64))
        assert ok, f"{m}x{n}x{k} call {call} vs arc_fp8_fp4_gemm: {msg}"


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (8, 520, 1024)])
def test_noalloc_matches_oracle_and_existing_entry_point(cuda_device, monkeypatch, m, n, k):
    monkeypatch.delenv("ARC_FP8FP4_KERNEL", raising=False)
    monkeypatch.delenv("ARC_FP8FP4_SPLIT", raising=False)
    cols = None if n <= 1024 else np.sort(np.random.default_rng(0).choice(n, size=512, replace=False))
    _check_twice(cuda_device, m, n, k, seed=m + n + k, cols=cols)


@pytest.mark.gpu
def test_noalloc_shape_beyond_its_scratch_runs_unsplit(cuda_device, monkeypatch):
    """128 x 9472 x 512 split in two needs 4096 + 2*128*9472*4 bytes, more than the 4 MiB
    array: the call runs the unsplit kernel instead (full-size operands, plan pinned)."""
    monkeypatch.setenv("ARC_FP8FP4_KERNEL", "128")
    monkeypatch.setenv("ARC_FP8FP4_SPLIT", "2")
    L = _lib.lib()
    need = ctypes.c_size_t(0)
    assert L.arc_fp8_fp4_workspace_bytes(128, 9472, 512, ctypes.byref(need)) == _lib.ARC_OK
    assert need.value > 4 << 20
    g = np.random.default_rng(1)
    _check_twice(cuda_device, 128, 9472, 512, seed=5,
                 rows=np.sort(g.choice(128, size=32, replace=False)),
                 cols=np.sort(g.choice(9472, size=256, replace=False)))


def test_noalloc_rejects_bad_arguments_without_a_device(native_lib):
    """Argument errors are reported before any device call or stream work."""
    L = native_lib
    p = ctypes.c_void_p(16)
    nul = ctypes.c_void_p(0)
    assert L.arc_fp8_fp4_gemm_noalloc(nul, p, p, p, p, 16, 64, 128, None) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_fp8_fp4_gemm_noalloc(p, p, p, p, p, 0, 64, 128, None) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_fp8_fp4_gemm_noalloc(p, p, p, p, p, 16, 64, 100, None) == _lib.ARC_ERR_UNSUPPORTED
    assert L.arc_fp8_fp4_gemm_noalloc(p, p, ctypes.c_void_p(48), p, p, 16, 64, 128, None) == \
        _lib.ARC_ERR_UNSUPPORTED
