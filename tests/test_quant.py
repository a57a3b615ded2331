"""CPU: int4 packing format, quantizers and synthetic data generators."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from arc import quant
from arc.testing.data import generate_a8w4, generate_bf16
from oracle import oracle


def test_pack_unpack_round_trip_all_codes():
    codes = torch.arange(-8, 8, dtype=torch.int8).repeat(4, 8)  # [4, 128]
    packed = quant.pack_int4(codes)
    assert packed.dtype == torch.uint8 and packed.shape == (4, 64)
    assert torch.equal(quant.unpack_int4(packed), codes)
    # byte 0 of each row holds k=0 (-8 -> 0x8) low and k=1 (-7 -> 0x9) high
    assert int(packed[0, 0]) == 0x98


def test_pack_rejects_out_of_range_and_odd_k():
    with pytest.raises(ValueError):
        quant.pack_int4(torch.tensor([[8, 0]]))
    with pytest.raises(ValueError):
        quant.pack_int4(torch.zeros((2, 3), dtype=torch.int8))


def test_per_group_int4_cast_dequant_error_and_format():
    g = torch.Generator().manual_seed(0)
    w = torch.randn((64, 512), generator=g)
    wp, sb = quant.per_group_cast_to_int4(w)
    assert wp.shape == (64, 256) and wp.dtype == torch.uint8
    assert sb.shape == (64, 4) and sb.dtype == torch.bfloat16
    deq = quant.dequantize_int4(wp, sb)
    # Rounding to the stored bf16 scale: error <= half a step (+ clamp at -8/+7 of amax/7).
    step = sb.float().repeat_interleave(128, dim=1)
    assert bool(((deq - w).abs() <= step * 0.5 + 1e-6).all())


def test_per_token_int8_cast():
    g = torch.Generator().manual_seed(1)
    x = torch.randn((9, 256), generator=g) * 3
    q, sa = quant.per_token_cast_to_int8(x)
    assert q.dtype == torch.int8 and sa.shape == (9,)
    assert int(q.abs().max()) == 127
    assert bool(((q.float() * sa[:, None] - x).abs() <= sa[:, None] * 0.5 + 1e-6).all())


def test_generate_a8w4_distributions_and_determinism():
    (x, sa), (wp, sb) = generate_a8w4(64, 256, 1024, seed=4)
    (x2, sa2), (wp2, sb2) = generate_a8w4(64, 256, 1024, seed=4)
    assert torch.equal(x, x2) and torch.equal(wp, wp2) and torch.equal(sa, sa2)
    assert torch.equal(sb.view(torch.int16), sb2.view(torch.int16))
    assert x.dtype == torch.int8 and int(x.min()) >= -127 and int(x.max()) <= 127
    w = quant.unpack_int4(wp)
    assert int(w.min()) == -8 and int(w.max()) == 7
    assert 0.01 <= float(sa.min()) and float(sa.max()) <= 0.05
    assert 0.005 <= float(sb.float().min()) and float(sb.float().max()) <= 0.0201
    assert sb.shape == (256, 8)


def test_generate_bf16():
    a, b = generate_bf16(16, 32, 64, seed=0)
    assert a.dtype == torch.bfloat16 and a.shape == (16, 64) and b.shape == (32, 64)
    assert abs(float(a.float().std()) - 1.0) < 0.2


def test_cpu_baseline_matches_oracle():
    """The timed CPU baseline (dequantize + fp32 matmul) agrees with the exact oracle."""
    (x, sa), (wp, sb) = generate_a8w4(8, 128, 512, seed=5)
    bits = sb.view(torch.int16).numpy().view(np.uint16)
    base = oracle.cpu_baseline_a8w4(x.numpy(), sa.numpy(), wp.numpy(), bits)
    ref = oracle.a8w4_out(x.numpy(), sa.numpy(), wp.numpy(), bits)
    ok, msg = oracle.check_bf16_close(base.float().numpy(), ref)
    assert ok, msg
