"""bf16 GEMM parity on the B200: CUDA path through the C ABI vs the oracle.

Small and ragged shapes are checked against the CPU oracle (float64 of the bf16
inputs); the BASELINE sizes against an fp32 GPU reference (TF32 off) of the same
inputs. The bar is 2 bf16 ulps (rtol ~1e-2). Both kernels run every small shape: the
one-CTA 128 x 256 tile kernel and the CTA-pair 256 x 256 kernel (ARC_BF16_CTAS forces
one; large problems pick the pair kernel on their own).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import arc
from arc.testing.data import generate_bf16
from oracle import oracle

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("ctas", [1, 2])
@pytest.mark.parametrize("m,n,k", [
    (128, 256, 64),     # exactly one tile, one K block (half a pair tile)
    (32, 128, 128),     # the reference's minimum legal shape
    (1, 8, 8),          # tiny and ragged everywhere
    (200, 264, 320),    # ragged M, N, K
    (384, 768, 1000),   # K tail inside a block
    (1024, 1024, 2048),
    (300, 520, 192),    # pair tiles whose second CTA holds no rows / columns
])
def test_bf16_vs_oracle(cuda_device, monkeypatch, m, n, k, ctas):
    monkeypatch.setenv("ARC_BF16_CTAS", str(ctas))
    a, b = generate_bf16(m, n, k, seed=m + n + k)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    arc.matmul(a.to(cuda_device), b.to(cuda_device), out=out)
    torch.cuda.synchronize()
    assert arc.device_status(0) == 0
    ref = oracle.bf16_gemm(_bits(a), _bits(b))
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref,
                                      atol=oracle.tensor_core_atol(k, ref))
    assert ok, msg


@pytest.mark.parametrize("m,n,k", [(2048, 2048, 2048), (8192, 8192, 8192)])
def test_bf16_baseline_sizes(cuda_device, m, n, k):
    dev = cuda_device
    a, b = generate_bf16(m, n, k, seed=0, device=dev)
    out = arc.matmul(a, b)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = (a.float() @ b.float().T).double().cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    assert arc.device_status(0) == 0
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref,
                                      atol=oracle.tensor_core_atol(k, ref))
    assert ok, msg
    # Same answer as the vendor GEMM to within the bf16 rounding of each.
    cub = torch.mm(a, b.T).float().cpu().numpy()
    assert oracle.symm_square_rel_L2_error(out.float().cpu().numpy(), cub) < 1e-5


@pytest.mark.parametrize("ctas", [1, 2])
def test_bf16_strided_operands(cuda_device, monkeypatch, ctas):
    """Row pitch larger than K (a column slice of a wider matrix)."""
    monkeypatch.setenv("ARC_BF16_CTAS", str(ctas))
    dev = cuda_device
    a_full, b_full = generate_bf16(256, 384, 512, seed=9, device=dev)
    a = a_full[:, :448]
    b = b_full[:, :448]
    out = arc.matmul(a, b)
    ref = oracle.bf16_gemm(_bits(a.contiguous().cpu()), _bits(b.contiguous().cpu()))
    torch.cuda.synchronize()
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref,
                                      atol=oracle.tensor_core_atol(448, ref))
    assert ok, msg


def test_bf16_out_preallocated_and_deterministic(cuda_device):
    dev = cuda_device
    a, b = generate_bf16(512, 512, 512, seed=4, device=dev)
    o1 = torch.empty((512, 512), dtype=torch.bfloat16, device=dev)
    r = arc.matmul(a, b, out=o1)
    o2 = arc.matmul(a, b)
    torch.cuda.synchronize()
    assert r.data_ptr() == o1.data_ptr()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))


def test_kernel_name_matches_the_shape_rules(cuda_device):
    """arc_kernel_name reports the kernel each operation launches (what ncu lists)."""
    from arc import _lib
    assert arc.kernel_name(_lib.OP_MATMUL_BF16, 8192, 8192, 8192) == "gemm_bf16_pair_kernel"
    assert arc.kernel_name(_lib.OP_MATMUL_BF16, 128, 256, 64) == "gemm_bf16_kernel"
    # decode instantiations: <token tile, stream mode, partials dump, cluster size, fused gather>
    assert arc.kernel_name(_lib.OP_A8W4, 16, 4096, 4096) == "gemm_a8w4_decode_kernel<16, 0, 0, 4, 0>"
    assert arc.kernel_name(_lib.OP_A8W4, 16, 28672, 8192) == "gemm_a8w4_decode_kernel<16, 1, 0, 1, 0>"
    assert arc.kernel_name(_lib.OP_A8W4, 4096, 14336, 4096) == "gemm_a8w4_kernel<128,2,3>"
    assert arc.kernel_name(_lib.OP_FP8_FP4, 4096, 14336, 4096) == "gemm_fp8fp4_pair_kernel"
    assert arc.kernel_name(_lib.OP_FP8_FP4, 16, 4096, 4096) == "gemm_fp8fp4_kernel<1>"
