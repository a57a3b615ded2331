"""GPU per-token int8 quantisation (arc.quantize_int8 / arc_quantize_int8).

The kernel must reproduce the host quantizer arc.quant.per_token_cast_to_int8 (the
int8 form of the reference's per-token cast, arc/testing/quant.py:30-48) bit for bit:
the same amax clamp, fp32 division and round-half-even. Covered: the vector path
(K, row strides multiples of 8), the scalar path (ragged K), strided rows, rows longer
than the register-resident part, tiny rows hitting the 1e-4 amax clamp, and the fused
bf16 -> A8W4 path against the GEMM on host-quantized operands.
"""
from __future__ import annotations

import pytest
import torch

import arc
from arc.quant import per_token_cast_to_int8
from arc.testing.data import generate_a8w4

pytestmark = pytest.mark.gpu


def _check(dev, x_cpu: torch.Tensor):
    q_ref, sa_ref = per_token_cast_to_int8(x_cpu)
    q, sa = arc.quantize_int8(x_cpu.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(sa.cpu(), sa_ref), "per-token scales differ"
    assert torch.equal(q.cpu(), q_ref), "int8 codes differ"


@pytest.mark.parametrize("m,k", [(1, 128), (16, 4096), (33, 1000), (7, 8), (130, 8192),
                                 (3, 20480), (2, 5)])
def test_quantize_matches_host_quantizer(cuda_device, m, k):
    g = torch.Generator().manual_seed(m * 131 + k)
    x = (torch.randn(m, k, generator=g) * 3.0).to(torch.bfloat16)
    _check(cuda_device, x)


def test_quantize_ties_and_tiny_rows(cuda_device):
    # A row whose values sit exactly on rounding ties, one below the amax clamp, one zero.
    k = 256
    x = torch.zeros(4, k)
    x[0] = torch.arange(k) % 5 - 2.0        # amax 2: x/sa = 63.5 * x, ties at odd x
    x[0, 7] = 2.0
    x[1] = 1e-6                              # amax clamps to 1e-4
    x[3] = torch.linspace(-1, 1, k)
    _check(cuda_device, x.to(torch.bfloat16))


def test_quantize_strided_rows(cuda_device):
    g = torch.Generator().manual_seed(7)
    base = (torch.randn(64, 4096 + 64, generator=g)).to(torch.bfloat16)
    x = base[:, 32:32 + 4096]                # row stride 4160, 64-byte offset
    q_ref, sa_ref = per_token_cast_to_int8(x.contiguous())
    q, sa = arc.quantize_int8(base.to(cuda_device)[:, 32:32 + 4096])
    torch.cuda.synchronize()
    assert torch.equal(sa.cpu(), sa_ref) and torch.equal(q.cpu(), q_ref)


def test_bf16_path_equals_gemm_on_host_quantized_operands(cuda_device):
    m, n, k = 16, 256, 1024
    _, (wp, sb) = generate_a8w4(m, n, k, seed=3)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wp, sb = wp.to(cuda_device), sb.to(cuda_device)
    fused = arc.a8w4_matmul_bf16(x.to(cuda_device), (wp, sb))
    q, sa = per_token_cast_to_int8(x)
    ref = arc.a8w4_matmul((q.to(cuda_device), sa.to(cuda_device)), (wp, sb))
    torch.cuda.synchronize()
    assert torch.equal(fused, ref)
