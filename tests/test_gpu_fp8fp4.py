"""FP8 x FP4 (UE8M0 block scales) GEMM on the B200: arc.fp8_fp4_gemm_nt / arc_fp8_fp4_gemm.

The recipe and call shape of the reference's A8W4 test (tests/a8w4.py:29-30, :48):
operands quantized with the reference's quantizers (arc.quant ports, pinned to the
reference by tests/test_fp8fp4_port.py). Checked two ways:
* against the float64 oracle of the quantized operands: within 2 bf16 ulps plus the
  tensor core's accumulation bound for the K length;
* the reference's own criterion: symm_square_rel_L2_error against the unquantized
  fp32 product below 1e-2 (tests/a8w4.py:52-53).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import arc
from arc import quant
from oracle import oracle

pytestmark = pytest.mark.gpu


def _data(m, n, k, seed):
    g = torch.Generator().manual_seed(seed)
    a_ref = torch.randn(m, k, generator=g).to(torch.bfloat16)
    b_ref = torch.randn(n, k, generator=g).to(torch.bfloat16)
    a = quant.per_token_cast_to_fp8(a_ref, use_ue8m0=True, gran_k=128)
    b = quant.per_token_cast_to_fp4(b_ref, use_ue8m0=True, gran_k=32)
    return a_ref, b_ref, a, b


@pytest.mark.parametrize("kernel", ["128", "256", "pair"])
@pytest.mark.parametrize("m,n,k", [(128, 128, 128), (16, 256, 512), (200, 136, 384),
                                   (1, 8, 128), (256, 1024, 4096), (300, 520, 1152),
                                   (300, 520, 1024), (520, 264, 2048)])
def test_fp8_fp4_gemm_matches_oracle(cuda_device, monkeypatch, m, n, k, kernel):
    """All three kernels, forced through ARC_FP8FP4_KERNEL: 128-row weight tiles
    (double-buffered accumulators, two K groups per stage), 256-row tiles (two UMMAs per
    K step), and CTA pairs on 256 x 256 tiles (K % 512 == 0 only). The shapes cover
    ragged M and N, N below one tile, pair tiles whose second CTA holds no rows, and odd
    group counts (K = 384, 1152)."""
    if kernel == "pair" and k % 512:
        pytest.skip("the pair kernel needs K % 512 == 0")
    monkeypatch.setenv("ARC_FP8FP4_KERNEL", kernel)
    a_ref, b_ref, (x, sfa), (wp, sfw) = _data(m, n, k, seed=m + n + k)
    dev = cuda_device
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
    arc.fp8_fp4_gemm_nt((x.to(dev), sfa.to(dev)), (wp.to(dev), sfw.to(dev)), out,
                        recipe_a=(1, 128), recipe_b=(1, 32))
    torch.cuda.synchronize()
    assert arc.device_status(0) == 0, "kernel reported a wait timeout"
    got = out.float().cpu().numpy()
    ref = oracle.fp8fp4_out(x.view(torch.uint8).numpy(), sfa.numpy(), wp.numpy(), sfw.numpy())
    ok, msg = oracle.check_bf16_close(got, ref, max_ulp=2.0, atol=oracle.tensor_core_atol(k, ref))
    assert ok, f"{m}x{n}x{k} kernel={kernel}: {msg}"
    # The reference's own acceptance test, against the unquantized product.
    full = (a_ref.double() @ b_ref.double().T).numpy()
    assert oracle.symm_square_rel_L2_error(got, full) < 1e-2


def test_fp8_fp4_gemm_rejects_other_recipes(cuda_device):
    _, _, (x, sfa), (wp, sfw) = _data(16, 16, 128, seed=1)
    out = torch.empty(16, 16, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        arc.fp8_fp4_gemm_nt((x.to(cuda_device), sfa.to(cuda_device)),
                            (wp.to(cuda_device), sfw.to(cuda_device)), out, recipe_b=(1, 128))


@pytest.mark.parametrize("split", [2, 3, 4])
@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (1, 264, 1152), (33, 520, 2048)])
def test_fp8_fp4_gemm_k_split(cuda_device, monkeypatch, m, n, k, split):
    """Decode-sized problems split K over several CTAs per tile (the workspace path of
    arc.fp8_fp4_gemm_nt): forced split counts, including a ragged last split and one
    of a single group (K = 1152 has 9 groups). The result equals the unsplit kernel's
    within the same tolerance, and two calls in a row give identical bits (the partials
    are summed in a fixed order, and the tile counters are left at zero)."""
    monkeypatch.setenv("ARC_FP8FP4_KERNEL", "128")
    monkeypatch.setenv("ARC_FP8FP4_SPLIT", str(split))
    a_ref, b_ref, (x, sfa), (wp, sfw) = _data(m, n, k, seed=7 * m + n + k)
    dev = cuda_device
    xs, sas, wps, sfws = x.to(dev), sfa.to(dev), wp.to(dev), sfw.to(dev)
    outs = []
    for _ in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
        arc.fp8_fp4_gemm_nt((xs, sas), (wps, sfws), out, recipe_a=(1, 128), recipe_b=(1, 32))
        outs.append(out)
    torch.cuda.synchronize()
    assert arc.device_status(0) == 0, "kernel reported a wait timeout"
    assert torch.equal(outs[0].view(torch.int16), outs[1].view(torch.int16))
    got = outs[0].float().cpu().numpy()
    ref = oracle.fp8fp4_out(x.view(torch.uint8).numpy(), sfa.numpy(), wp.numpy(), sfw.numpy())
    ok, msg = oracle.check_bf16_close(got, ref, max_ulp=2.0, atol=oracle.tensor_core_atol(k, ref))
    assert ok, f"{m}x{n}x{k} split={split}: {msg}"
