"""TVM-FFI typed exports (libarcb200_tvm_ffi.so): the binding shape of the reference's
GEMM module (arc/mm.py:30 typed `matmul(a, b, out)`, exported at arc/mm.py:48).

CPU: the module builds and loads, exports matmul / a8w4_matmul / fp8_fp4_gemm_nt, and
rejects arguments before any device work (CPU tensors, wrong dtypes, shape mismatches).
GPU: both GEMMs called through TVM-FFI with torch CUDA tensors match the CPU oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

tvm_ffi = pytest.importorskip("tvm_ffi")

from arc import build, tvm_module  # noqa: E402
from arc.testing.data import generate_a8w4, generate_bf16  # noqa: E402
from oracle import oracle  # noqa: E402


@pytest.fixture(scope="module")
def mod():
    build.build()
    assert build.build_tvm_ffi() is not None
    return tvm_module.load()


def test_module_exports_the_typed_functions(mod):
    for name in ("matmul", "a8w4_matmul", "fp8_fp4_gemm_nt"):
        assert callable(getattr(mod, name))


def test_rejects_bad_arguments_without_a_gpu(mod):
    a = torch.zeros(4, 128, dtype=torch.bfloat16)
    b = torch.zeros(8, 128, dtype=torch.bfloat16)
    out = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        mod.matmul(a, b, out)
    x = torch.zeros(4, 256, dtype=torch.int8)
    sa = torch.zeros(4, dtype=torch.float32)
    wp = torch.zeros(8, 128, dtype=torch.uint8)
    sb = torch.zeros(8, 2, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        mod.a8w4_matmul(x, sa, wp, sb, out)
    with pytest.raises(TypeError):
        mod.matmul(a, b)  # wrong arity


@pytest.mark.gpu
def test_matmul_through_tvm_ffi(mod, cuda_device):
    m, n, k = 200, 264, 320
    a, b = generate_bf16(m, n, k, seed=4)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    mod.matmul(a.to(cuda_device), b.to(cuda_device), out)
    torch.cuda.synchronize()
    ref = oracle.bf16_gemm(a.view(torch.int16).numpy().view(np.uint16), b.view(torch.int16).numpy().view(np.uint16))
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref)
    assert ok, msg
    with pytest.raises(ValueError, match="Inner"):
        mod.matmul(a.to(cuda_device), b[:, :256].contiguous().to(cuda_device), out)


@pytest.mark.gpu
@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (100, 264, 512)])
def test_a8w4_matmul_through_tvm_ffi(mod, cuda_device, m, n, k):
    (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=9)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=cuda_device)
    mod.a8w4_matmul(x.to(cuda_device), sa.to(cuda_device), wp.to(cuda_device), sb.to(cuda_device), out)
    torch.cuda.synchronize()
    cols = np.sort(np.random.default_rng(1).choice(n, size=min(n, 256), replace=False))
    ref = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy()[cols], sb.view(torch.int16).numpy().view(np.uint16)[cols])
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy()[:, cols], ref, max_ulp=2.0)
    assert ok, msg
