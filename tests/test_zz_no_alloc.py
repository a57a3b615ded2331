"""The allocation-free FP8 x FP4 entry point, arc_fp8_fp4_gemm_noalloc, called through the C ABI.

Some callers cannot allocate device memory: operator plugins whose host framework budgets
all of it and passes the operator only its input and output tensors, and hosts that must
not call cudaMalloc on the request path. For them the library keeps the K-split scratch of
decode-sized FP8 x FP4 problems in a fixed 4 MiB device array of its own. This test checks
that entry point against the existing one (arc_fp8_fp4_gemm, which runs without a K
split) on the same operands, twice in a row (the scratch keeps the previous call's
contents, so the second call shows that it starts clean), and that a shape whose split
needs more scratch than the array holds is refused. It sits in a file that pytest
collects last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from arc import _lib, quant
from oracle import oracle

pytestmark = pytest.mark.gpu


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


@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (8, 520, 1024)])
def test_noalloc_matches_the_existing_entry_point(cuda_device, monkeypatch, m, n, k):
    monkeypatch.delenv("ARC_FP8FP4_KERNEL", raising=False)
    monkeypatch.delenv("ARC_FP8FP4_SPLIT", raising=False)
    dev = cuda_device
    L = _lib.lib()
    ops = _operands(m, n, k, seed=m + n + k, dev=dev)
    ref = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
    assert _call(L.arc_fp8_fp4_gemm, ops, ref, m, n, k, dev) == _lib.ARC_OK, L.arc_last_error()
    ref64 = ref.double().cpu().numpy()
    for call in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        assert _call(L.arc_fp8_fp4_gemm_noalloc, ops, out, m, n, k, dev) == _lib.ARC_OK, \
            L.arc_last_error()
        torch.cuda.synchronize()
        assert _lib.device_status(dev.index) == 0, "kernel reported a wait timeout"
        ok, msg = oracle.check_bf16_close(out.double().cpu().numpy(), ref64, max_ulp=2.0,
                                          atol=oracle.tensor_core_atol(k, ref64))
        assert ok, f"{m}x{n}x{k} call {call}: {msg}"


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda_device, monkeypatch):
    """128 x 9472 x 512 splits K in two: 4096 + 2*128*9472*4 bytes, more than 4 MiB."""
    monkeypatch.delenv("ARC_FP8FP4_KERNEL", raising=False)
    monkeypatch.delenv("ARC_FP8FP4_SPLIT", raising=False)
    dev = cuda_device
    L = _lib.lib()
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=dev)
    p = buf.data_ptr()
    st = L.arc_fp8_fp4_gemm_noalloc(p, p, p, p, p, 128, 9472, 512, None)
    assert st == _lib.ARC_ERR_UNSUPPORTED
    assert b"scratch" in L.arc_last_error()
