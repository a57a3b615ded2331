"""CPU: the oracle of the int4 weight pre-pack (the layout arc_a8w4_prepack_weights writes).

The reference has no pre-pack step; its weights exist only in the packing of
arc/testing/quant.py:82-83. The layout is therefore pinned by a hand-built known answer
and by round trips through the reference-pinned unpack (oracle.np_unpack_int4).
"""
from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle


def _pack_reference(codes: np.ndarray) -> np.ndarray:
    """int4 codes [N, K] (-8..7) -> the reference packing, even k in the low nibble."""
    c = (np.asarray(codes, dtype=np.int16) & 0xF).astype(np.uint8)
    return (c[:, 0::2] | (c[:, 1::2] << 4)).astype(np.uint8)


def test_known_answer_one_piece():
    # Codes 0..31 as their 4-bit patterns (k mod 16), so each nibble names its position.
    k = np.arange(32)
    codes = np.where(k % 16 >= 8, k % 16 - 16, k % 16)[None, :]
    packed = _pack_reference(codes)
    assert packed[0, 0] == 0x10 and packed[0, 7] == 0xFE  # codes (0, 1) and (14, 15)
    q = oracle.np_prepack_int4(packed)
    # byte j = code j (bits 3:0) | code j+16 (bits 7:4); code j+16 has the pattern of j.
    assert q.tolist() == [[j | (j << 4) for j in range(16)]]


def test_known_answer_distinct_halves():
    codes = np.zeros((1, 32), dtype=np.int8)
    codes[0, 3] = -1      # pattern 0xF at k = 3
    codes[0, 16 + 5] = 7  # pattern 0x7 at k = 21
    q = oracle.np_prepack_int4(_pack_reference(codes))
    expect = np.zeros(16, dtype=np.uint8)
    expect[3] = 0x0F
    expect[5] = 0x70
    assert np.array_equal(q[0], expect)


@pytest.mark.parametrize("n,k", [(1, 32), (3, 128), (17, 4096), (128, 8192)])
def test_round_trip_and_code_preservation(n, k):
    rng = np.random.default_rng(n * 1000 + k)
    codes = rng.integers(-8, 8, size=(n, k), dtype=np.int8)
    packed = _pack_reference(codes)
    assert np.array_equal(oracle.np_unpack_int4(packed), codes)
    q = oracle.np_prepack_int4(packed)
    assert q.shape == packed.shape and q.dtype == np.uint8
    assert np.array_equal(oracle.np_unprepack_int4(q), packed)
    # Only nibbles inside each 16-byte piece move: the per-piece multiset of codes stays.
    pieces_in = np.sort(oracle.np_unpack_int4(packed).reshape(n, k // 32, 32), axis=-1)
    lo = (q & 0xF).reshape(n, k // 32, 16)
    hi = (q >> 4).reshape(n, k // 32, 16)
    nib = np.concatenate([lo, hi], axis=-1).astype(np.int16)
    pieces_out = np.sort(np.where(nib >= 8, nib - 16, nib), axis=-1)
    assert np.array_equal(pieces_in, pieces_out)


def test_rejects_k_not_multiple_of_32():
    with pytest.raises(AssertionError):
        oracle.np_prepack_int4(np.zeros((2, 8), dtype=np.uint8))
