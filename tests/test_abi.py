"""CPU: the C-ABI library loads, exports every declared symbol, and validates input.

No compute call reaches a GPU here: every call below is rejected by host-side checks
that run before any CUDA call, or is a host-only entry point.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from arc import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "arc_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(arc_[a-z0-9_]+)\s*\(", text))


def test_header_declares_the_bound_symbols():
    assert declared_functions() == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(native_lib):
    for name in declared_functions():
        assert hasattr(native_lib, name), f"{name} missing from libarcb200.so"


def test_version_and_status_strings(native_lib):
    assert native_lib.arc_version() >= 100
    assert native_lib.arc_status_string(0) == b"ok"
    assert b"unsupported" in native_lib.arc_status_string(2)
    assert native_lib.arc_status_string(99) == b"unknown status"


def test_invalid_arguments_are_rejected_before_any_cuda_call(native_lib):
    L = native_lib
    nul = None
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.cast(buf, ctypes.c_void_p).value
    # null pointers
    assert L.arc_matmul_bf16(nul, p, p, 1, 1, 1, 8, 8, 8, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert b"null" in L.arc_last_error()
    # non-positive sizes
    assert L.arc_matmul_bf16(p, p, p, 0, 8, 8, 8, 8, 8, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    # leading dimension smaller than K
    assert L.arc_matmul_bf16(p, p, p, 8, 8, 16, 8, 16, 8, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    # leading dimension not a multiple of 8
    assert L.arc_matmul_bf16(p, p, p, 8, 8, 12, 12, 16, 8, nul) == _lib.ARC_ERR_UNSUPPORTED
    # A8W4: group other than 128, K not a multiple of 128, N not a multiple of 8
    assert L.arc_a8w4_gemm(p, p, p, p, p, 16, 64, 256, 64, nul, nul) == _lib.ARC_ERR_UNSUPPORTED
    assert L.arc_a8w4_gemm(p, p, p, p, p, 16, 64, 200, 128, nul, nul) == _lib.ARC_ERR_UNSUPPORTED
    assert L.arc_a8w4_gemm(p, p, p, p, p, 16, 60, 256, 128, nul, nul) == _lib.ARC_ERR_UNSUPPORTED
    assert L.arc_a8w4_gemm(p, nul, p, p, p, 16, 64, 256, 128, nul, nul) == \
        _lib.ARC_ERR_INVALID_ARGUMENT
    # misaligned operand
    assert L.arc_a8w4_gemm(p + 1, p, p, p, p, 16, 64, 256, 128, nul, nul) == _lib.ARC_ERR_UNSUPPORTED
    # quantizer: null output, leading dimension below K, misaligned input
    assert L.arc_quantize_int8(p, nul, p, 4, 64, 64, 64, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_quantize_int8(p, p, p, 4, 64, 32, 64, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_quantize_int8(p + 1, p, p, 4, 64, 64, 64, nul) == _lib.ARC_ERR_UNSUPPORTED
    # FP8 x FP4: K not a multiple of 128, misaligned packed weights (32 bytes needed)
    assert L.arc_fp8_fp4_gemm(p, p, p, p, p, 16, 64, 200, nul) == _lib.ARC_ERR_UNSUPPORTED
    a32 = (p + 31) // 32 * 32  # 32-byte aligned inside the buffer
    assert L.arc_fp8_fp4_gemm(a32, a32, a32 + 16, a32, a32, 16, 64, 256, nul) == \
        _lib.ARC_ERR_UNSUPPORTED
    # weight pre-pack: K not a multiple of 32, misaligned, partial overlap; prepacked GEMM group
    assert L.arc_a8w4_prepack_weights(p, p, 4, 48, nul) == _lib.ARC_ERR_UNSUPPORTED
    assert L.arc_a8w4_prepack_weights(p + 1, p + 1, 4, 64, nul) == _lib.ARC_ERR_UNSUPPORTED
    assert L.arc_a8w4_prepack_weights(a32, a32 + 16, 4, 64, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_a8w4_prepack_weights(nul, p, 4, 64, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_a8w4_gemm_prepacked(p, p, p, p, p, 16, 64, 256, 64, nul) == _lib.ARC_ERR_UNSUPPORTED
    # fused all-gather: world out of range, prefill-sized M; peer barrier: rank >= world
    outs = (ctypes.c_void_p * 2)(a32, a32)
    assert L.arc_a8w4_gemm_gather(p, p, p, p, outs, 9, 0, 16, 64, 256, nul) == \
        _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_a8w4_gemm_gather(p, p, p, p, outs, 2, 0, 64, 64, 256, nul) == _lib.ARC_ERR_UNSUPPORTED
    assert L.arc_peer_barrier(outs, 2, 2, nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    # CUDA IPC helpers: missing handle / output arguments
    off = ctypes.c_uint64()
    vp, vb = ctypes.c_void_p(), ctypes.c_void_p()
    assert L.arc_ipc_export(nul, p, ctypes.byref(off)) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_ipc_open(nul, 0, ctypes.byref(vp), ctypes.byref(vb)) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_ipc_close(nul) == _lib.ARC_ERR_INVALID_ARGUMENT
    # kernel-name query: no buffer / non-positive sizes
    assert L.arc_kernel_name(0, 8, 8, 8, nul, 16) == _lib.ARC_ERR_INVALID_ARGUMENT
    assert L.arc_kernel_name(0, 0, 8, 8, ctypes.cast(buf, ctypes.c_char_p), 16) == \
        _lib.ARC_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("m,n,k,expect", [
    # decode: 32 full-height tiles, K split four ways in 4-CTA clusters (one wave, at most
    # one CTA per SM so that the next launch in the stream fits beside it)
    (16, 4096, 4096, dict(split=1, token_tile=16, weight_rows=128, k_split=4, grid=128)),
    # 37 tiles x 4 = 148 CTAs still fit; 38 tiles drop to a split of two
    (16, 4736, 4096, dict(split=1, k_split=4, grid=148)),
    (16, 4864, 4096, dict(split=1, k_split=2, grid=76)),
    # large N: persistent unsplit 128-row tiles
    (1, 28672, 8192, dict(split=0, token_tile=16, weight_rows=128, grid=224)),
    (16, 14336, 4096, dict(split=0, k_split=1, grid=112)),
    # long K: splits use both CTA slots of an SM (two per SM, at most 296 CTAs)
    (16, 14336, 8192, dict(split=1, k_split=2, grid=224)),
    (16, 7168, 8192, dict(split=1, k_split=4, grid=224)),
    (32, 4096, 4096, dict(split=1, token_tile=32, k_split=4)),
    # K of one or two groups limits the split
    (16, 512, 128, dict(split=0, k_split=1, grid=4)),
    (16, 512, 256, dict(split=1, k_split=2, grid=8)),
    (33, 4096, 4096, dict(split=0, token_tile=64)),
    (4096, 14336, 4096, dict(split=0, token_tile=128, weight_rows=128, grid=148)),
])
def test_plans(native_lib, m, n, k, expect):
    plan = _lib.describe_plan(m, n, k, 148)
    for key, v in expect.items():
        assert plan[key] == v, (key, plan)
    if m <= 32:
        assert plan["weight_rows"] == 128
        assert plan["k_split"] in (1, 2, 4) and plan["k_split"] <= k // 128
        tiles = -(-n // 128)
        if plan["split"]:
            assert plan["grid"] == tiles * plan["k_split"] <= 148 * (2 if k // 128 >= 64 else 1)
        else:  # long tiles (>= 64 K-groups) run up to two CTAs per SM
            assert plan["grid"] == min(tiles, 148 * (2 if k // 128 >= 64 else 1))
        # weights stream in stages of two K-groups (a 128-byte box row) through 4 stages
        assert plan["groups_per_stage"] == 2 and plan["load_stages"] == 4


def test_decode_plans_cover_every_row(native_lib):
    """Every decode plan's tiles cover N and its K split never exceeds the group count."""
    for n in (8, 24, 256, 1000, 4096, 14336, 28672):
        for k in (128, 256, 4096, 8192):
            plan = _lib.describe_plan(16, n, k, 148)
            tiles = plan["grid"] // plan["k_split"] if plan["split"] else -(-n // plan["weight_rows"])
            assert tiles * plan["weight_rows"] >= n
            assert 1 <= plan["k_split"] <= max(1, k // 128)


def test_plan_rejects_bad_k(native_lib):
    with pytest.raises(_lib.ArcError):
        _lib.describe_plan(16, 64, 200, 148)
