"""Generate the committed golden fixtures in tests/golden/.

Run from the repository root in a container where the reference checkout is
available, with ARC_REFERENCE set to its path:

    ARC_REFERENCE=<path of the reference checkout> python tests/golden/make_golden.py

Fixtures:

* ref_nibble_pin.npz — pins the int4 byte layout to the reference's own code:
  4-bit codes are fed through the reference packer
  (arc/testing/quant.py:51-84 per_token_cast_to_fp4, packing at :82-83) and the
  resulting bytes through the reference unpacker (arc/math.py:159-170
  cast_back_from_fp4, unpacking at :144-146). Inputs are chosen so every 32-wide
  group contains a +-6.0, making the UE8M0 scale exactly 1.0 and each value an exact
  fp4 grid point, so the packer's codes are known in advance.
* ref_metric_pin.npz — the reference's symm_square_rel_L2_error (arc/math.py:14-23)
  and count_bytes (arc/math.py:26-33) on seeded inputs.
* ref_fp8fp4_pin.npz — the reference's FP8 / FP4 quantizers (arc/testing/quant.py:30-84,
  the recipe of tests/a8w4.py:29-30) on seeded bf16 inputs, and its fp4 decode
  (arc/math.py:159-170): pins arc.quant's ports of them bit for bit.
* a8w4_small.npz / bf16_small.npz — small seeded GEMM cases with the oracle's exact
  partials and float64 outputs; the partials are cross-checked here against an
  independent numpy formulation before being written.

The reference is only imported here, in this script; tests read the .npz files.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path[:0] = [str(ROOT / "arc-gemm_b200"), str(ROOT)]

FP4_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def _reference_path() -> str:
    ref = os.environ.get("ARC_REFERENCE")
    if not ref:
        raise SystemExit("set ARC_REFERENCE to the path of the reference checkout")
    return ref


def _reference():
    ref = _reference_path()
    if not Path(ref, "arc", "math.py").exists():
        raise SystemExit(f"reference checkout not found at {ref}")
    sys.path.insert(0, ref)
    import arc.math as ref_math  # the reference's module, not ours
    from arc.testing import quant as ref_quant

    return ref_math, ref_quant


def nibble_pin(ref_math, ref_quant):
    rng = np.random.default_rng(20240501)
    n, k = 16, 128
    # Codes 0..15 except 8 (the reference quantizer never emits a negative zero).
    choices = np.array([c for c in range(16) if c != 8], dtype=np.uint8)
    codes = rng.choice(choices, size=(n, k)).astype(np.uint8)
    codes[:, ::32] = 7  # +6.0 in every 32-wide group -> UE8M0 scale exactly 1.0
    mag = FP4_GRID[codes & 7]
    vals = np.where(codes & 8, -mag, mag).astype(np.float32)
    x = torch.from_numpy(vals).to(torch.bfloat16)
    packed_t, sf = ref_quant.per_token_cast_to_fp4(x, use_ue8m0=True, gran_k=32)
    assert torch.all(sf == 1.0), "scales must be exactly one"
    packed = packed_t.view(torch.uint8).numpy().copy()
    back = ref_math.cast_back_from_fp4(packed_t, torch.ones_like(sf), gran_k=32).numpy()
    np.savez_compressed(HERE / "ref_nibble_pin.npz", codes=codes, packed=packed,
                        dequant=back.astype(np.float32))


def metric_pin(ref_math):
    rng = np.random.default_rng(7)
    xs, ys, vals = [], [], []
    for scale in (1.0, 1e-3, 1e3):
        x = rng.standard_normal(512).astype(np.float32) * scale
        y = (x + rng.standard_normal(512).astype(np.float32) * 0.01 * scale).astype(np.float32)
        xs.append(x)
        ys.append(y)
        vals.append(float(ref_math.symm_square_rel_L2_error(torch.from_numpy(x),
                                                            torch.from_numpy(y))))
    z = np.zeros(8, np.float32)
    zero_val = float(ref_math.symm_square_rel_L2_error(torch.from_numpy(z), torch.from_numpy(z)))
    t = (torch.zeros(3, 5, dtype=torch.int8), (torch.zeros(7, dtype=torch.float32),
                                               torch.zeros(2, 2, dtype=torch.bfloat16)))
    nbytes = int(ref_math.count_bytes(*t))
    np.savez_compressed(HERE / "ref_metric_pin.npz", x=np.stack(xs), y=np.stack(ys),
                        symm=np.array(vals), zero=np.array(zero_val), count_bytes=np.array(nbytes))


def fp8fp4_pin(ref_math, ref_quant):
    g = torch.Generator().manual_seed(31)
    a = torch.randn(12, 384, generator=g).to(torch.bfloat16)
    b = torch.randn(20, 384, generator=g).to(torch.bfloat16)
    b[3, :40] = 0  # an all-zero block (scale clamp) and ties at block edges
    b[4, 5] = 3.0 * 2 ** -3
    xq, sfa = ref_quant.per_token_cast_to_fp8(a, use_ue8m0=True, gran_k=128)
    wq, sfw = ref_quant.per_token_cast_to_fp4(b, use_ue8m0=True, gran_k=32)
    back = ref_math.cast_back_from_fp4(wq, sfw, gran_k=32)
    np.savez_compressed(HERE / "ref_fp8fp4_pin.npz",
                        a=a.view(torch.int16).numpy().view(np.uint16),
                        b=b.view(torch.int16).numpy().view(np.uint16),
                        xq=xq.view(torch.uint8).numpy(), sfa=sfa.numpy(),
                        wq=wq.view(torch.uint8).numpy(), sfw=sfw.numpy(),
                        dequant=back.float().numpy())


def a8w4_small():
    from arc.testing.data import generate_a8w4
    from oracle import oracle

    cases = {}
    for tag, (m, n, k, seed) in {"a": (5, 24, 256, 11), "b": (3, 16, 128, 12),
                                 "c": (17, 40, 384, 13)}.items():
        (x, sa), (wp, sb) = generate_a8w4(m, n, k, seed=seed)
        xn, san, wpn = x.numpy(), sa.numpy(), wp.numpy()
        sbn = sb.view(torch.int16).numpy().view(np.uint16)
        P = oracle.a8w4_partials(xn, wpn)
        assert np.array_equal(P, oracle.np_a8w4_partials(xn, wpn)), "C and numpy partials differ"
        out = oracle.a8w4_out(xn, san, wpn, sbn)
        # Independent float64 restatement of the scale math.
        sbf = oracle.bf16_bits_to_f32(sbn).astype(np.float64)
        alt = san.astype(np.float64)[:, None] * np.einsum("mng,ng->mn", P.astype(np.float64), sbf)
        assert np.allclose(out, alt, rtol=1e-12, atol=0), "scale math differs"
        cases.update({f"{tag}_x": xn, f"{tag}_sa": san, f"{tag}_wp": wpn, f"{tag}_sb": sbn,
                      f"{tag}_P": P, f"{tag}_out": out})
    np.savez_compressed(HERE / "a8w4_small.npz", **cases)


def bf16_small():
    from arc.testing.data import generate_bf16
    from oracle import oracle

    a, b = generate_bf16(6, 10, 72, seed=21)
    ab = a.view(torch.int16).numpy().view(np.uint16)
    bb = b.view(torch.int16).numpy().view(np.uint16)
    c = oracle.bf16_gemm(ab, bb)
    alt = a.double().numpy() @ b.double().numpy().T
    assert np.allclose(c, alt, rtol=1e-12, atol=1e-12)
    np.savez_compressed(HERE / "bf16_small.npz", a=ab, b=bb, c=c)


def main():
    ref_math, ref_quant = _reference()
    nibble_pin(ref_math, ref_quant)
    metric_pin(ref_math)
    fp8fp4_pin(ref_math, ref_quant)
    # Drop the reference package from sys.modules so the local `arc` imports cleanly.
    for name in [m for m in sys.modules if m == "arc" or m.startswith("arc.")]:
        del sys.modules[name]
    sys.path.remove(_reference_path())
    a8w4_small()
    bf16_small()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
