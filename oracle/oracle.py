"""CPU oracle for the GEMM hot path. TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg and
its ``--impl reference`` arm) may import this module, and only as the checker or as
the timed CPU baseline. The product (``arc-gemm_b200/``) never imports it.

Two layers:

* ``liboracle.so`` (``a8w4_oracle.c``): the exact integer partials and the double
  precision outputs, restating the algorithm with plain loops.
* numpy/torch helpers in this file: independent re-statements used to cross-check
  the C code, the ulp metric used by the parity tests, and the CPU baseline
  "dequantize + fp32 matmul" that stands for the reference's CPU path.

Reference anchors: packing/unpacking order arc/testing/quant.py:82-83 and
arc/math.py:144-146; A8W4 data flow tests/a8w4.py:15-33; bf16 reference
tests/matmul.py:21-23; statistical metric arc/math.py:14-23.
"""
from __future__ import annotations

import ctypes
import os
import time
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "_build" / "liboracle.so"

_lib = None


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            from oracle.build import build_oracle

            build_oracle()
        lib = ctypes.CDLL(str(LIB_PATH))
        p = ctypes.c_void_p
        i = ctypes.c_int
        lib.oracle_unpack_int4.argtypes = [p, i, i, p]
        lib.oracle_a8w4_partials.argtypes = [p, p, i, i, i, i, p]
        lib.oracle_a8w4_out.argtypes = [p, p, p, p, i, i, i, i, p]
        lib.oracle_bf16_gemm.argtypes = [p, p, i, i, i, p]
        lib.oracle_f32_to_bf16.argtypes = [p, ctypes.c_long, p]
        for f in ("oracle_unpack_int4", "oracle_a8w4_partials", "oracle_a8w4_out",
                  "oracle_bf16_gemm", "oracle_f32_to_bf16"):
            getattr(lib, f).restype = None
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


# --------------------------------------------------------------------------- C oracle
def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """[rows, K/2] uint8 -> [rows, K] int8 in [-8, 7] (even k from the low nibble)."""
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    rows, half = packed.shape
    out = np.empty((rows, 2 * half), dtype=np.int8)
    _load().oracle_unpack_int4(_ptr(packed), rows, 2 * half, _ptr(out))
    return out


def a8w4_partials(a: np.ndarray, w_packed: np.ndarray, group: int = 128) -> np.ndarray:
    """Exact int32 partials P[m, n, g]."""
    a = np.ascontiguousarray(a, dtype=np.int8)
    w_packed = np.ascontiguousarray(w_packed, dtype=np.uint8)
    M, K = a.shape
    N = w_packed.shape[0]
    assert w_packed.shape[1] * 2 == K and K % group == 0
    P = np.empty((M, N, K // group), dtype=np.int32)
    _load().oracle_a8w4_partials(_ptr(a), _ptr(w_packed), M, N, K, group, _ptr(P))
    return P


def a8w4_out(a, sa, w_packed, sb_bits, group: int = 128) -> np.ndarray:
    """out[m, n] = sa[m] * sum_g sb[n, g] * P[m, n, g], in float64.

    ``sb_bits`` are the bf16 scale bits as uint16 ([N, K/group]).
    """
    a = np.ascontiguousarray(a, dtype=np.int8)
    sa = np.ascontiguousarray(sa, dtype=np.float32)
    w_packed = np.ascontiguousarray(w_packed, dtype=np.uint8)
    sb_bits = np.ascontiguousarray(sb_bits, dtype=np.uint16)
    M, K = a.shape
    N = w_packed.shape[0]
    out = np.empty((M, N), dtype=np.float64)
    _load().oracle_a8w4_out(_ptr(a), _ptr(sa), _ptr(w_packed), _ptr(sb_bits), M, N, K, group,
                            _ptr(out))
    return out


def bf16_gemm(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """C = A . B^T in float64 from bf16 bits ([M, K] and [N, K] uint16)."""
    a_bits = np.ascontiguousarray(a_bits, dtype=np.uint16)
    b_bits = np.ascontiguousarray(b_bits, dtype=np.uint16)
    M, K = a_bits.shape
    N = b_bits.shape[0]
    out = np.empty((M, N), dtype=np.float64)
    _load().oracle_bf16_gemm(_ptr(a_bits), _ptr(b_bits), M, N, K, _ptr(out))
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    _load().oracle_f32_to_bf16(_ptr(x), x.size, _ptr(out))
    return out


# ------------------------------------------------------------------ numpy restatements
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def np_unpack_int4(packed: np.ndarray) -> np.ndarray:
    """Independent numpy unpack: even k = low nibble, two's complement."""
    p = np.asarray(packed, dtype=np.uint8)
    lo = (p & 0x0F).astype(np.int16)
    hi = (p >> 4).astype(np.int16)
    codes = np.empty(p.shape[:-1] + (p.shape[-1] * 2,), dtype=np.int16)
    codes[..., 0::2] = lo
    codes[..., 1::2] = hi
    return np.where(codes >= 8, codes - 16, codes).astype(np.int8)


def np_prepack_int4(packed: np.ndarray) -> np.ndarray:
    """The reference's packing -> the pre-packed layout of arc_a8w4_prepack_weights.

    The reference has no pre-pack; this restates the layout that entry point defines on
    top of the reference's nibble order (arc/testing/quant.py:82-83): inside every
    16-byte piece of a row (32 codes, k = 32q .. 32q+31), byte j = code j in bits 3:0 and
    code j+16 in bits 7:4 (codes as raw 4-bit patterns).
    """
    p = np.asarray(packed, dtype=np.uint8)
    n, kb = p.shape
    assert kb % 16 == 0, "K must be a multiple of 32"
    nib = np.empty((n, 2 * kb), dtype=np.uint8)
    nib[:, 0::2] = p & 0x0F
    nib[:, 1::2] = p >> 4
    nib = nib.reshape(n, kb // 16, 32)
    return (nib[..., :16] | (nib[..., 16:] << 4)).reshape(n, kb)


def np_unprepack_int4(prepacked: np.ndarray) -> np.ndarray:
    """Inverse of np_prepack_int4: the pre-packed layout -> the reference's packing."""
    q = np.asarray(prepacked, dtype=np.uint8)
    n, kb = q.shape
    assert kb % 16 == 0, "K must be a multiple of 32"
    pieces = q.reshape(n, kb // 16, 16)
    nib = np.concatenate([pieces & 0x0F, pieces >> 4], axis=-1).reshape(n, 2 * kb)
    return (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)


def np_a8w4_partials(a: np.ndarray, w_packed: np.ndarray, group: int = 128) -> np.ndarray:
    """Independent numpy partials via int64 matmul per group."""
    w = np_unpack_int4(w_packed).astype(np.int64)
    a64 = np.asarray(a, dtype=np.int64)
    M, K = a64.shape
    G = K // group
    P = np.empty((M, w.shape[0], G), dtype=np.int64)
    for g in range(G):
        sl = slice(g * group, (g + 1) * group)
        P[:, :, g] = a64[:, sl] @ w[:, sl].T
    return P.astype(np.int32)


# ------------------------------------------------------------ FP8 x FP4 (UE8M0 blocks)
def e4m3_to_f64(bits: np.ndarray) -> np.ndarray:
    """float8 e4m3 (fn) bytes -> float64: sign bit 7, 4-bit exponent (bias 7), 3-bit
    mantissa, subnormals at exponent 0, 0x7F / 0xFF NaN (no infinities)."""
    b = np.asarray(bits, np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 0x7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * np.ldexp(1.0, e - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return sign * val


E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])


def e2m1_unpack_f64(packed: np.ndarray) -> np.ndarray:
    """[N, K/2] packed e2m1 (even k in the low nibble; code = magnitude | sign << 3,
    arc/testing/quant.py:51-84, decoded as arc/math.py:148-153) -> float64 [N, K]."""
    p = np.asarray(packed, np.uint8)
    codes = np.empty((p.shape[0], p.shape[1] * 2), np.uint8)
    codes[:, 0::2] = p & 0x0F
    codes[:, 1::2] = p >> 4
    mag = E2M1[codes & 7]
    return np.where(codes & 8, -mag, mag)


def fp8fp4_out(x_bits, sfa, w_packed, sfw) -> np.ndarray:
    """out[m,n] = sum_k x[m,k] sfa[m,k/128] * w[n,k] sfw[n,k/32] in float64 (every
    product of the scaled operands is exact; only the sum's order differs from the
    tensor core's)."""
    a = e4m3_to_f64(x_bits)
    k = a.shape[1]
    a = a * np.repeat(np.asarray(sfa, np.float64), 128, axis=1)[:, :k]
    w = e2m1_unpack_f64(w_packed) * np.repeat(np.asarray(sfw, np.float64), 32, axis=1)[:, :k]
    return a @ w.T


# ------------------------------------------------------------ activation quantizer
def int8_per_token_quant(x_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-token int8 quantisation of bf16 activations, in numpy float32 arithmetic.

    The shape of the reference's per-token activation cast
    (arc/testing/quant.py:30-48, per_token_cast_to_fp8: row amax over |x| in fp32,
    clamped below at 1e-4, scale = amax / format max, codes = x / scale cast to the
    format), restated for the int8 recipe: format max 127, the codes rounded half to
    even and clipped to [-127, 127].
      x_bits [M, K] uint16 (bf16 bits) -> (q [M, K] int8, sa [M] float32)
    """
    x = (np.ascontiguousarray(x_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    amax = np.maximum(np.abs(x).max(axis=1), np.float32(1e-4)).astype(np.float32)
    sa = (amax / np.float32(127.0)).astype(np.float32)
    q = np.rint(x / sa[:, None]).astype(np.float32)
    q = np.clip(q, -127, 127).astype(np.int8)
    return q, sa


# ----------------------------------------------------------------------- parity metric
def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers at |x| (normal range; subnormals get the min spacing)."""
    ax = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.maximum(ax, 2.0 ** -126)))
    return np.exp2(e - 7)


def ulp_distance(got_bf16_f32: np.ndarray, ref: np.ndarray) -> np.ndarray:
    """|got - ref| measured in bf16 ulps of the reference value."""
    return np.abs(np.asarray(got_bf16_f32, np.float64) - ref) / bf16_ulp(ref)


def tensor_core_atol(k: int, ref: np.ndarray) -> float:
    """Absolute error budget of an fp32 tensor-core accumulation over K.

    tcgen05 adds each K=16 (bf16) or K=32 (int8) slice of products into the fp32
    accumulator with truncating alignment, so the error can grow by about half an fp32
    ulp of the running sum per UMMA step: (K/16) * 2^-24 * 2^ceil(log2 max|ref|).
    """
    peak = float(np.max(np.abs(ref))) if ref.size else 0.0
    if peak == 0.0:
        return 0.0
    return (max(k, 16) / 16.0) * 2.0 ** -24 * 2.0 ** np.ceil(np.log2(peak))


def check_bf16_close(got_bf16_f32: np.ndarray, ref: np.ndarray, max_ulp: float = 2.0,
                     atol: float | None = None) -> tuple[bool, str]:
    """Parity rule for bf16 outputs: |got - ref| <= max_ulp bf16 ulps of ref + atol.

    `atol` covers elements that are small only through cancellation, where a bf16 ulp
    of ref says nothing about the arithmetic. Default: 2^-12 of the RMS of ref (well
    below one bf16 ulp of typical values). fp32 tensor-core accumulations over long K
    pass `tensor_core_atol(K, ref)` instead.
    """
    ref = np.asarray(ref, np.float64)
    got = np.asarray(got_bf16_f32, np.float64)
    if atol is None:
        rms = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
        atol = rms * 2.0 ** -12
    tol = max_ulp * bf16_ulp(ref) + atol
    err = np.abs(got - ref)
    bad = ~(err <= tol)
    if bad.any():
        idx = np.unravel_index(int(np.argmax(np.where(bad, err / tol, 0))), ref.shape)
        return False, (f"{int(bad.sum())} of {ref.size} elements beyond {max_ulp} ulp + "
                       f"{atol:.3g}; worst at {idx}: got {got[idx]!r} ref {ref[idx]!r}")
    return True, "ok"


def symm_square_rel_L2_error(x: np.ndarray, y: np.ndarray) -> float:
    """1 - 2<x,y>/(<x,x>+<y,y>) in float64 (the reference's metric, arc/math.py:14-23)."""
    x = np.asarray(x, np.float64)
    y = np.asarray(y, np.float64)
    den = float((x * x + y * y).sum())
    if den == 0.0:
        return 0.0
    return 1.0 - 2.0 * float((x * y).sum()) / den


# --------------------------------------------------------------------- CPU baseline
def cpu_baseline_a8w4(a, sa, w_packed, sb_bits, group: int = 128, threads: int | None = None):
    """The reference's CPU path for A8W4: dequantize both operands, fp32 matmul, bf16.

    W_f32[n,k] = int4[n,k] * sb[n, k/group], A_f32[m,k] = int8[m,k] * sa[m],
    out = bf16(A_f32 @ W_f32^T), on the host cores through torch (all threads by
    default). Returns the bf16 result as a torch tensor.
    """
    import torch

    if threads is not None:
        torch.set_num_threads(threads)
    a_t = torch.from_numpy(np.ascontiguousarray(a, np.int8))
    sa_t = torch.from_numpy(np.ascontiguousarray(sa, np.float32))
    p = torch.from_numpy(np.ascontiguousarray(w_packed, np.uint8))
    sb_t = torch.from_numpy(bf16_bits_to_f32(sb_bits))
    lo = (p & 0x0F).to(torch.int16)
    hi = (p >> 4).to(torch.int16)
    codes = torch.stack((lo, hi), dim=-1).reshape(p.shape[0], -1)
    w = torch.where(codes >= 8, codes - 16, codes).to(torch.float32)
    w = (w.view(w.shape[0], -1, group) * sb_t.unsqueeze(-1)).view(w.shape[0], -1)
    a_f = a_t.to(torch.float32) * sa_t.unsqueeze(1)
    return (a_f @ w.T).to(torch.bfloat16)


def time_cpu_baseline(fn, budget_s: float = 10.0, min_reps: int = 1):
    """Run fn repeatedly for about budget_s seconds; returns (seconds per call, reps)."""
    fn()
    reps = 0
    t0 = time.perf_counter()
    while True:
        fn()
        reps += 1
        el = time.perf_counter() - t0
        if reps >= min_reps and el >= budget_s:
            return el / reps, reps


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
