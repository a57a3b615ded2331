"""GPU per-token int8 quantisation (arc.quantize_int8 / arc_quantize_int8).

The kernel must reproduce the CPU oracle's quantizer, oracle.int8_per_token_quant (the
int8 form of the reference's per-token cast, arc/testing/quant.py:30-48, in numpy fp32)
bit for bit: the same amax clamp, fp32 division and round-half-even. The host quantizer
of the package (arc.quant.per_token_cast_to_int8) is checked against the same oracle. Covered: the vector path
(K, row strides multiples of 8), the scalar path (ragged K), strided rows, rows longer
than the register-resident part, tiny rows hitting the 1e-4 amax clamp, and the fused
bf16 -> A8W4 path against the GEMM on host-quantized operands.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import arc
from arc.quant import per_token_cast_to_int8
from arc.testing.data import generate_a8w4
from oracle import oracle



def _oracle_quant(x_cpu: torch.Tensor):
    q, sa = oracle.int8_per_token_quant(x_cpu.contiguous().view(torch.int16).numpy().view(np.uint16))
    return torch.from_numpy(q), torch.from_numpy(sa)


def _check(dev, x_cpu: torch.Tensor):
    q_ref, sa_ref = _oracle_quant(x_cpu)
    q, sa = arc.quantize_int8(x_cpu.to(dev))
    torch.cuda.synchronize()
    assert torch.equal(sa.cpu(), sa_ref), "per-token scales differ"
    assert torch.equal(q.cpu(), q_ref), "int8 codes differ"


@pytest.mark.gpu
@pytest.mark.parametrize("m,k", [(1, 128), (16, 4096), (33, 1000), (7, 8), (130, 8192),
                                 (3, 20480), (2, 5)])
def test_quantize_matches_oracle(cuda_device, m, k):
    g = torch.Generator().manual_seed(m * 131 + k)
    x = (torch.randn(m, k, generator=g) * 3.0).to(torch.bfloat16)
    _check(cuda_device, x)


@pytest.mark.gpu
def test_quantize_ties_and_tiny_rows(cuda_device):
    # A row whose values sit exactly on rounding ties, one below the amax clamp, one zero.
    k = 256
    x = torch.zeros(4, k)
    x[0] = torch.arange(k) % 5 - 2.0        # amax 2: x/sa = 63.5 * x, ties at odd x
    x[0, 7] = 2.0
    x[1] = 1e-6                              # amax clamps to 1e-4
    x[3] = torch.linspace(-1, 1, k)
    _check(cuda_device, x.to(torch.bfloat16))


@pytest.mark.gpu
def test_quantize_strided_rows(cuda_device):
    g = torch.Generator().manual_seed(7)
    base = (torch.randn(64, 4096 + 64, generator=g)).to(torch.bfloat16)
    x = base[:, 32:32 + 4096]                # row stride 4160, 64-byte offset
    q_ref, sa_ref = _oracle_quant(x)
    q, sa = arc.quantize_int8(base.to(cuda_device)[:, 32:32 + 4096])
    torch.cuda.synchronize()
    assert torch.equal(sa.cpu(), sa_ref) and torch.equal(q.cpu(), q_ref)


@pytest.mark.gpu
def test_bf16_path_equals_gemm_on_host_quantized_operands(cuda_device):
    m, n, k = 16, 256, 1024
    _, (wp, sb) = generate_a8w4(m, n, k, seed=3)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wp, sb = wp.to(cuda_device), sb.to(cuda_device)
    fused = arc.a8w4_matmul_bf16(x.to(cuda_device), (wp, sb))
    q, sa = _oracle_quant(x)
    ref = arc.a8w4_matmul((q.to(cuda_device), sa.to(cuda_device)), (wp, sb))
    torch.cuda.synchronize()
    assert torch.equal(fused, ref)
    want = oracle.a8w4_out(q.numpy(), sa.numpy(), wp.cpu().numpy(),
                           sb.cpu().view(torch.int16).numpy().view(np.uint16))
    ok, msg = oracle.check_bf16_close(fused.float().cpu().numpy(), want, max_ulp=2.0)
    assert ok, msg


def test_host_quantizer_matches_oracle():
    """The package's host quantizer and the oracle's agree bit for bit (CPU only)."""
    g = torch.Generator().manual_seed(3)
    for m, k in ((5, 300), (16, 4096)):
        x = (torch.randn(m, k, generator=g) * 2.0).to(torch.bfloat16)
        q, sa = per_token_cast_to_int8(x)
        q_ref, sa_ref = _oracle_quant(x)
        assert torch.equal(q, q_ref) and torch.equal(sa, sa_ref)
