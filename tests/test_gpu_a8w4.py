"""A8W4 parity on the B200: CUDA path through the C ABI vs the CPU oracle.

* int32 group partials: bit-exact against the oracle (tests at sizes it finishes fast);
* bf16 outputs: within 2 bf16 ulps of the oracle's exact (float64) result;
* full BASELINE sizes: exact oracle on sampled rows/columns, an fp32 torch reference of
  the dequantized operands on the GPU for every element, plus size-independent
  properties (determinism, exact scaling by powers of two in sa).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import arc
from arc.quant import dequantize_int4
from arc.testing.data import generate_a8w4
from oracle import oracle

pytestmark = pytest.mark.gpu


def _bits(sb: torch.Tensor) -> np.ndarray:
    return sb.view(torch.int16).numpy().view(np.uint16)


def _run(dev, m, n, k, seed, with_partials=True):
    (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=seed)
    parts = (torch.full((m, n, k // 128), -12345, dtype=torch.int32, device=dev)
             if with_partials else None)
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
    arc.a8w4_matmul((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)), out, partials=parts)
    torch.cuda.synchronize()
    assert arc.device_status(dev.index or 0) == 0, "kernel reported a wait timeout"
    return (x, sa, wp, sb), out, parts


SHAPES = [
    (1, 256, 128),      # single token, a single K group
    (5, 24, 256),       # ragged M, N smaller than one weight tile
    (16, 4096, 4096),   # the BASELINE decode configuration
    (16, 1000, 512),    # N not a multiple of the tile height
    (32, 512, 1024),    # 32-token split-K tile
    (33, 136, 384),     # first persistent-tile shape (64-token tiles)
    (64, 264, 640),
    (100, 264, 256),    # ragged 128-token tiles
    (256, 1024, 2048),  # several token and weight tiles
]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_a8w4_partials_exact_and_outputs(cuda_device, m, n, k):
    (x, sa, wp, sb), out, parts = _run(cuda_device, m, n, k, seed=m * 7 + n + k)
    p_ref = oracle.a8w4_partials(x.numpy(), wp.numpy())
    p_got = parts.cpu().numpy()
    mism = np.argwhere(p_got != p_ref)
    assert mism.size == 0, f"{len(mism)} partials differ, first at {tuple(mism[0])}: " \
                           f"{p_got[tuple(mism[0])]} vs {p_ref[tuple(mism[0])]}"
    ref = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy(), _bits(sb))
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref, max_ulp=2.0)
    assert ok, msg


@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (4096, 14336, 4096)])
def test_a8w4_baseline_sizes(cuda_device, m, n, k):
    """Full BASELINE configs: every element vs an fp32 GPU reference, sampled exact oracle."""
    (x, sa, wp, sb), out, _ = _run(cuda_device, m, n, k, seed=0, with_partials=False)
    dev = cuda_device
    # fp32 reference of the dequantized operands (TF32 off: true fp32 products).
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        w_f = dequantize_int4(wp.to(dev), sb.to(dev))
        a_f = x.to(dev).float() * sa.to(dev).unsqueeze(1)
        ref32 = (a_f @ w_f.T).double().cpu().numpy()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref32, max_ulp=2.0)
    assert ok, msg
    # Exact oracle on a sample of rows and columns.
    g = np.random.default_rng(1)
    rows = np.sort(g.choice(m, size=min(m, 48), replace=False))
    cols = np.sort(g.choice(n, size=min(n, 256), replace=False))
    ref = oracle.a8w4_out(x.numpy()[rows], sa.numpy()[rows], wp.numpy()[cols],
                          _bits(sb)[cols])
    got = out.float().cpu().numpy()[np.ix_(rows, cols)]
    ok, msg = oracle.check_bf16_close(got, ref, max_ulp=2.0)
    assert ok, msg
    # Statistical criterion of the reference's A8W4 check (tests/a8w4.py:53-54).
    assert oracle.symm_square_rel_L2_error(out.float().cpu().numpy(), ref32) < 1e-4


def test_a8w4_deterministic_and_sa_scaling(cuda_device):
    """Two runs are bit-identical; doubling sa doubles every output exactly."""
    dev = cuda_device
    (x, sa), (wp, sb) = generate_a8w4(16, 4096, 4096, seed=5)
    args = ((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)))
    o1 = arc.a8w4_matmul(*args)
    o2 = arc.a8w4_matmul(*args)
    o3 = arc.a8w4_matmul((args[0][0], args[0][1] * 2), args[1])
    torch.cuda.synchronize()
    assert torch.equal(o1.view(torch.int16), o2.view(torch.int16))
    assert torch.equal((o1.float() * 2).to(torch.bfloat16).view(torch.int16), o3.view(torch.int16))
    assert arc.device_status(0) == 0


def test_a8w4_extreme_values_exact(cuda_device):
    """All-extreme operands (int8 -127/127, int4 -8/7): partials at their maximum size."""
    dev = cuda_device
    m, n, k = 16, 256, 512
    x = torch.where(torch.arange(m * k).view(m, k) % 3 == 0, -127, 127).to(torch.int8)
    w = torch.where(torch.arange(n * k).view(n, k) % 5 == 0, 7, -8).to(torch.int8)
    wp = arc.quant.pack_int4(w)
    sa = torch.full((m,), 0.03125)
    sb = torch.full((n, k // 128), 0.0078125, dtype=torch.bfloat16)
    parts = torch.empty((m, n, k // 128), dtype=torch.int32, device=dev)
    out = arc.a8w4_matmul((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)), partials=parts)
    torch.cuda.synchronize()
    assert np.array_equal(parts.cpu().numpy(), oracle.a8w4_partials(x.numpy(), wp.numpy()))
    ref = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy(), _bits(sb))
    ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref, max_ulp=2.0)
    assert ok, msg


def test_a8w4_gemm_nt_call_shape(cuda_device):
    dev = cuda_device
    (x, sa), (wp, sb) = generate_a8w4(16, 512, 1024, seed=3)
    out = torch.empty((16, 512), dtype=torch.bfloat16, device=dev)
    arc.a8w4_gemm_nt((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)), out,
                     recipe_a=(1, 1024), recipe_b=(1, 128))
    ref = arc.a8w4_matmul((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)))
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def _check_on_device(out: torch.Tensor, ref: torch.Tensor, max_ulp: float = 2.0):
    """check_bf16_close evaluated on the GPU (for outputs too large to copy out)."""
    ref = ref.double()
    got = out.double()
    ulp = torch.exp2(torch.floor(torch.log2(ref.abs().clamp_min(2.0 ** -126))) - 7)
    atol = float(ref.pow(2).mean().sqrt()) * 2.0 ** -12
    err = (got - ref).abs()
    bad = err > max_ulp * ulp + atol
    n_bad = int(bad.sum())
    assert n_bad == 0, f"{n_bad} of {ref.numel()} elements beyond {max_ulp} ulp + {atol:.3g}"


@pytest.mark.parametrize("m", [1, 16, 128, 1024, 8192])
def test_a8w4_large_weight_sweep(cuda_device, m):
    """N=28672, K=8192 at the sweep's token counts."""
    n, k = 28672, 8192
    dev = cuda_device
    (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=m)
    xd, sad, wpd, sbd = x.to(dev), sa.to(dev), wp.to(dev), sb.to(dev)
    out = arc.a8w4_matmul((xd, sad), (wpd, sbd))
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref32 = (xd.float() * sad.unsqueeze(1)) @ dequantize_int4(wpd, sbd).T
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    assert arc.device_status(0) == 0
    _check_on_device(out, ref32)
    g = np.random.default_rng(2)
    rows = np.sort(g.choice(m, size=min(m, 8), replace=False))
    cols = np.sort(g.choice(n, size=128, replace=False))
    ref = oracle.a8w4_out(x.numpy()[rows], sa.numpy()[rows], wp.numpy()[cols], _bits(sb)[cols])
    got = out.float().cpu().numpy()[np.ix_(rows, cols)]
    ok, msg = oracle.check_bf16_close(got, ref, max_ulp=2.0)
    assert ok, msg


@pytest.mark.parametrize("plan", ["128:4", "128:2", "128:1", "128:1:3", "128:1:1"])
def test_a8w4_decode_decompositions(cuda_device, monkeypatch, plan):
    """Every decode decomposition is exact; forced per test. K split over 4- and 2-CTA
    clusters, persistent unsplit tiles, and persistent CTAs capped at 3 and 1 so that each
    walks several tiles (the A slots, load stages and accumulators carry over between
    tiles). K = 384 and 640 give one-group load stages and uneven splits; K = 8192 and the
    capped grids give CTAs with more load stages than the ring holds (stream mode: both
    groups of a stage unpacked into TMEM, ring stages refilled ahead of the UMMAs), with 16
    and with 32 tokens per tile. A second call without the partials buffer runs the
    production instantiation of the same plan and must give the same output bit for bit."""
    monkeypatch.setenv("ARC_DECODE_PLAN", plan)
    S = int(plan.split(":")[1])
    for m, n, k in ((16, 1000, 1024), (3, 512, 2048), (32, 256, 512), (16, 1000, 384), (7, 264, 640),
                    (16, 384, 8192), (32, 256, 8192)):
        for static in (False, True):
            (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=S + m + k)
            dev = cuda_device
            parts = torch.full((m, n, k // 128), -12345, dtype=torch.int32, device=dev)
            out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
            arc.a8w4_matmul((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)), out, partials=parts,
                            static_weights=static)
            torch.cuda.synchronize()
            assert arc.device_status(0) == 0, "kernel reported a wait timeout"
            assert np.array_equal(parts.cpu().numpy(), oracle.a8w4_partials(x.numpy(), wp.numpy())), \
                f"plan {plan} {m}x{n}x{k} static={static}: partials differ"
            ref = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy(), _bits(sb))
            ok, msg = oracle.check_bf16_close(out.float().cpu().numpy(), ref, max_ulp=2.0)
            assert ok, f"plan {plan} {m}x{n}x{k} static={static}: {msg}"
            out2 = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev)
            arc.a8w4_matmul((x.to(dev), sa.to(dev)), (wp.to(dev), sb.to(dev)), out2, static_weights=static)
            torch.cuda.synchronize()
            assert arc.device_status(0) == 0, "kernel reported a wait timeout"
            assert torch.equal(out2, out), f"plan {plan} {m}x{n}x{k} static={static}: no-dump output differs"


@pytest.mark.parametrize("m,n,k", [(16, 4096, 4096), (32, 1000, 1024), (1, 28672, 8192)])
def test_a8w4_static_weights_back_to_back(cuda_device, m, n, k):
    """static_weights: consecutive decode GEMMs on one stream, each reading tokens that
    the kernel directly before it wrote (the GPU int8 quantizer). The GEMM streams its
    weights while the quantizer still runs, but must read the tokens only after it: every
    result equals the same GEMM run in isolation, bit for bit, and the oracle."""
    dev = cuda_device
    (_, _), (wp, sb) = generate_a8w4(m, n, k, seed=11)
    wpd, sbd = wp.to(dev), sb.to(dev)
    g = torch.Generator(device=dev).manual_seed(5)
    xs = [torch.randn(m, k, generator=g, device=dev, dtype=torch.bfloat16) for _ in range(6)]
    qs = [(torch.empty((m, k), dtype=torch.int8, device=dev), torch.empty((m,), dtype=torch.float32, device=dev))
          for _ in xs]
    outs = [torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=dev) for _ in xs]
    for x, q, o in zip(xs, qs, outs):  # quantize -> GEMM -> quantize -> GEMM ..., no syncs
        arc.quantize_int8(x, out=q)
        arc.a8w4_matmul(q, (wpd, sbd), o, static_weights=True)
    torch.cuda.synchronize()
    assert arc.device_status(0) == 0, "kernel reported a wait timeout"
    for i, (q, o) in enumerate(zip(qs, outs)):
        ref = arc.a8w4_matmul(q, (wpd, sbd))
        torch.cuda.synchronize()
        assert torch.equal(o.view(torch.int16), ref.view(torch.int16)), f"call {i} differs"
    cols = np.sort(np.random.default_rng(3).choice(n, size=min(n, 192), replace=False))
    q, sa = (t.cpu() for t in qs[-1])
    want = oracle.a8w4_out(q.numpy(), sa.numpy(), wp.numpy()[cols], _bits(sb)[cols])
    ok, msg = oracle.check_bf16_close(outs[-1].float().cpu().numpy()[:, cols], want, max_ulp=2.0)
    assert ok, msg
