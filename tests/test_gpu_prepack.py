"""Weight pre-pack on the B200: the pre-pack kernel against the CPU oracle byte for byte,
and the GEMM on pre-packed weights against the GEMM on the reference packing (bit for
bit: the same arithmetic) and against the oracle's exact result.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import arc
from arc.testing.data import generate_a8w4
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n,k", [(1, 32), (8, 128), (1040, 1024), (4096, 4096), (3, 96)])
def test_prepack_kernel_matches_oracle(cuda_device, n, k):
    rng = np.random.default_rng(n + k)
    wp = rng.integers(0, 256, size=(n, k // 2), dtype=np.uint8)
    got = arc.prepack_weights(torch.from_numpy(wp).to(cuda_device)).cpu().numpy()
    assert np.array_equal(got, oracle.np_prepack_int4(wp))


def test_prepack_in_place_and_round_trip(cuda_device):
    rng = np.random.default_rng(7)
    wp = rng.integers(0, 256, size=(300, 2048), dtype=np.uint8)
    t = torch.from_numpy(wp).to(cuda_device)
    arc.prepack_weights(t, out=t)
    torch.cuda.synchronize()
    q = t.cpu().numpy()
    assert np.array_equal(q, oracle.np_prepack_int4(wp))
    assert np.array_equal(oracle.np_unprepack_int4(q), wp)


SHAPES = [
    (1, 256, 128),
    (5, 24, 256),
    (16, 4096, 4096),   # the decode configuration (split-K clusters)
    (32, 512, 1024),
    (33, 136, 384),     # first persistent-tile shape
    (100, 264, 256),
    (256, 1024, 2048),
    (1, 28672, 1024),   # persistent kernel at M = 1
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_prepacked_gemm_bit_identical(cuda_device, m, n, k):
    (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=m + n + k)
    dev = cuda_device
    a = (x.to(dev), sa.to(dev))
    ref = arc.a8w4_matmul(a, (wp.to(dev), sb.to(dev)))
    wq = arc.prepack_weights(wp.to(dev))
    got = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
    arc.a8w4_matmul(a, (wq, sb.to(dev)), got, prepacked=True)
    torch.cuda.synchronize()
    assert arc.device_status(dev.index or 0) == 0
    assert torch.equal(got, ref)
    if m * n * k <= 16 * 4096 * 4096:
        exact = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy(),
                                sb.view(torch.int16).numpy().view(np.uint16))
        ok, msg = oracle.check_bf16_close(got.float().cpu().numpy(), exact, max_ulp=2.0)
        assert ok, msg


def test_prepacked_prefill_size(cuda_device):
    # The prefill configuration through the persistent kernel, checked against the
    # reference-packing GEMM over every element.
    m, n, k = 4096, 14336, 4096
    (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=3)
    dev = cuda_device
    a = (x.to(dev), sa.to(dev))
    ref = arc.a8w4_matmul(a, (wp.to(dev), sb.to(dev)))
    got = arc.a8w4_matmul(a, (arc.prepack_weights(wp.to(dev)), sb.to(dev)), prepacked=True)
    torch.cuda.synchronize()
    assert arc.device_status(dev.index or 0) == 0
    assert torch.equal(got, ref)


def test_prepacked_rejects_partials(cuda_device):
    (x, sa), (wp, sb) = generate_a8w4(4, 64, 256, seed=1)
    dev = cuda_device
    parts = torch.zeros((4, 64, 2), dtype=torch.int32, device=dev)
    with pytest.raises(ValueError):
        arc.a8w4_matmul((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)), partials=parts, prepacked=True)
