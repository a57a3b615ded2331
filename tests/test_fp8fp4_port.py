"""CPU: the FP8 / FP4 quantizer ports and the FP8 x FP4 oracle against the reference.

tests/golden/ref_fp8fp4_pin.npz holds the reference's own quantizer outputs
(arc/testing/quant.py:30-84 with the settings of tests/a8w4.py:29-30) and fp4 decode
(arc/math.py:159-170) on seeded inputs (see tests/golden/make_golden.py).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from arc import quant
from oracle import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "ref_fp8fp4_pin.npz"


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16)


def test_fp8_and_fp4_quantizers_match_the_reference():
    g = np.load(GOLDEN)
    a, b = _bf16(g["a"]), _bf16(g["b"])
    xq, sfa = quant.per_token_cast_to_fp8(a, use_ue8m0=True, gran_k=128)
    wq, sfw = quant.per_token_cast_to_fp4(b, use_ue8m0=True, gran_k=32)
    assert np.array_equal(xq.view(torch.uint8).numpy(), g["xq"])
    assert np.array_equal(sfa.numpy(), g["sfa"])
    assert np.array_equal(wq.numpy(), g["wq"])
    assert np.array_equal(sfw.numpy(), g["sfw"])
    assert np.array_equal(quant.dequantize_fp4(wq, sfw, 32).numpy(), g["dequant"])


def test_oracle_decoders_match_torch():
    bits = np.arange(256, dtype=np.uint8)
    ours = oracle.e4m3_to_f64(bits)
    theirs = torch.from_numpy(bits).view(torch.float8_e4m3fn).double().numpy()
    both_nan = np.isnan(ours) & np.isnan(theirs)
    assert np.array_equal(ours[~both_nan], theirs[~both_nan])
    g = np.load(GOLDEN)
    back = oracle.e2m1_unpack_f64(g["wq"]) * np.repeat(g["sfw"].astype(np.float64), 32, axis=1)
    assert np.array_equal(back.astype(np.float32), g["dequant"])


def test_oracle_fp8fp4_matches_dequantized_matmul():
    g = np.load(GOLDEN)
    a = torch.from_numpy(g["xq"]).view(torch.float8_e4m3fn).double()
    a = a * torch.from_numpy(g["sfa"]).double().repeat_interleave(128, dim=1)
    w = torch.from_numpy(g["dequant"]).double()
    ref = (a @ w.T).numpy()
    out = oracle.fp8fp4_out(g["xq"], g["sfa"], g["wq"], g["sfw"])
    assert np.allclose(out, ref, rtol=1e-12, atol=1e-12)
