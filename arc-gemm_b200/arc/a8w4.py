"""A8W4 matmul: int8 activations x packed int4 weights with K-group-128 scales.

In the reference this role is played by the third-party call
`deep_gemm.fp8_fp4_gemm_nt((a, sfa), (b, sfb), out, recipe_a=(1, 128), recipe_b=(1, 32))`
(tests/a8w4.py:48, :70): operands are (data, scale) pairs, `b` is K-major ("NT") and
`out` is preallocated by the caller. The same calling shape is kept here for the
int8 x int4 recipe:

    a = (x,  sa)   x  [M, K]   int8,   sa [M] float32 (one scale per token)
    b = (wp, sb)   wp [N, K/2] uint8 (two int4 per byte, even k in the low nibble),
                   sb [N, K/128] bfloat16 (one scale per column and 128-wide K group)
    out            [M, N] bfloat16

    out[m, n] = bf16( sa[m] * sum_g f32(sb[n, g]) * P[m, n, g] ),
    P[m, n, g] = sum_{k in group g} x[m, k] * w[n, k]   (int32, exact)

Everything runs in `arc_a8w4_gemm_ex` (include/arc_b200.h) on the caller's stream.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from ._lib import A8W4_PREPACKED, A8W4_STATIC_WEIGHTS, check, lib
from .quant import TensorPair

GROUP_K = 128


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _expect(t: torch.Tensor, name: str, dtype: torch.dtype, shape: tuple, device) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path), got {t.device}")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def a8w4_matmul(a: TensorPair, b: TensorPair, out: torch.Tensor | None = None, *,
                group: int = GROUP_K, partials: torch.Tensor | None = None,
                prepacked: bool = False, static_weights: bool = False) -> torch.Tensor:
    """out = A8W4 GEMM of (x, sa) and (wp, sb). See the module docstring.

    `partials`, if given, is an int32 [M, N, K/128] tensor that receives every exact
    group partial P[m, n, g] (a slow debugging mode).
    `prepacked=True` says wp is in the pre-packed layout of `prepack_weights` (same
    shape; results identical to the original packing).
    `static_weights=True` promises that wp and sb are not written by the kernel that
    directly precedes this call on the current stream (true of model weights loaded
    once). Decode-sized calls (M <= 32) then stream and unpack the weights while that
    kernel is still running, so back-to-back GEMMs overlap their weight traffic.
    Results are the same either way.
    """
    x, sa = a
    wp, sb = b
    m, k = x.shape
    n, k2 = wp.shape
    assert k == 2 * k2, f"Inner dimensions must match: {k} vs 2*{k2}"
    if group != GROUP_K:
        raise ValueError(f"only group={GROUP_K} is supported, got {group}")
    assert k % group == 0, f"K ({k}) must be a multiple of {group}"
    dev = x.device
    if sa.dim() == 2 and sa.shape[1] == 1:
        sa = sa.reshape(-1)
    _expect(x, "a[0]", torch.int8, (m, k), None)
    _expect(sa, "a[1]", torch.float32, (m,), dev)
    _expect(wp, "b[0]", torch.uint8, (n, k // 2), dev)
    _expect(sb, "b[1]", torch.bfloat16, (n, k // group), dev)
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    else:
        _expect(out, "out", torch.bfloat16, (m, n), dev)
    if prepacked and partials is not None:
        raise ValueError("partials are not available with prepacked weights")
    pptr = None
    if partials is not None:
        _expect(partials, "partials", torch.int32, (m, n, k // group), dev)
        pptr = partials.data_ptr()
    flags = (A8W4_PREPACKED if prepacked else 0) | (A8W4_STATIC_WEIGHTS if static_weights else 0)
    with torch.cuda.device(dev):
        check(lib().arc_a8w4_gemm_ex(x.data_ptr(), sa.data_ptr(), wp.data_ptr(), sb.data_ptr(),
                                     out.data_ptr(), m, n, k, group, flags, _stream_ptr(dev), pptr),
              "arc.a8w4_matmul")
    return out


def prepack_weights(wp: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Packed int4 weights [N, K/2] (the reference's packing, even k in the low nibble)
    -> the pre-packed layout, on the GPU: inside every 16-byte piece (32 codes of a row),
    byte j holds code j in its low nibble and code j+16 in its high nibble. `out` may be
    `wp` itself (in place). Use the result with `a8w4_matmul(..., prepacked=True)`.
    """
    if not isinstance(wp, torch.Tensor) or wp.dim() != 2:
        raise ValueError("wp must be a 2-D uint8 tensor [N, K/2]")
    n, k2 = wp.shape
    _expect(wp, "wp", torch.uint8, (n, k2), None)
    if out is None:
        out = torch.empty_like(wp)
    else:
        _expect(out, "out", torch.uint8, (n, k2), wp.device)
    with torch.cuda.device(wp.device):
        check(lib().arc_a8w4_prepack_weights(wp.data_ptr(), out.data_ptr(), n, 2 * k2, _stream_ptr(wp.device)),
              "arc.prepack_weights")
    return out


def a8w4_gemm_nt(a: TensorPair, b: TensorPair, out: torch.Tensor,
                 recipe_a: Sequence[int] | None = None,
                 recipe_b: Sequence[int] = (1, GROUP_K)) -> torch.Tensor:
    """deep_gemm-style entry (tests/a8w4.py:48): recipes name the scale granularity.

    recipe_a: None or (1, K) — one activation scale per token.
    recipe_b: (1, 128)       — one weight scale per column and 128-wide K group.
    """
    k = a[0].shape[1]
    if recipe_a is not None and tuple(recipe_a) != (1, k):
        raise ValueError(f"recipe_a must be per-token (1, {k}), got {tuple(recipe_a)}")
    if tuple(recipe_b) != (1, GROUP_K):
        raise ValueError(f"recipe_b must be (1, {GROUP_K}), got {tuple(recipe_b)}")
    return a8w4_matmul(a, b, out, group=GROUP_K)


def quantize_int8(x: torch.Tensor, out: TensorPair | None = None) -> TensorPair:
    """bf16 activations [M, K] -> (int8 [M, K], fp32 per-token scale [M]) on the GPU.

    The same numbers as arc.quant.per_token_cast_to_int8 (the host quantizer, which
    follows the reference's per-token cast, arc/testing/quant.py:30-48), computed by
    `arc_quantize_int8` on the caller's stream. `out` may supply the (q, sa) buffers.
    """
    if not isinstance(x, torch.Tensor) or x.dim() != 2:
        raise ValueError("quantize_int8 expects a 2D tensor")
    if x.device.type != "cuda":
        raise ValueError(f"x must be a CUDA tensor (there is no CPU path), got {x.device}")
    if x.dtype != torch.bfloat16:
        raise TypeError(f"x must be torch.bfloat16, got {x.dtype}")
    if x.stride(1) != 1:
        raise ValueError("x must have unit stride along K")
    m, k = x.shape
    dev = x.device
    if out is None:
        q = torch.empty((m, k), dtype=torch.int8, device=dev)
        sa = torch.empty((m,), dtype=torch.float32, device=dev)
    else:
        q, sa = out
        _expect(q, "out[0]", torch.int8, (m, k), dev)
        _expect(sa, "out[1]", torch.float32, (m,), dev)
    with torch.cuda.device(dev):
        check(lib().arc_quantize_int8(x.data_ptr(), q.data_ptr(), sa.data_ptr(), m, k, x.stride(0),
                                      q.stride(0), _stream_ptr(dev)),
              "arc.quantize_int8")
    return q, sa


def a8w4_matmul_bf16(x: torch.Tensor, b: TensorPair, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 activations through the whole A8W4 path: GPU quantisation, then the GEMM.

    Both kernels run on the caller's stream; the GEMM's prologue overlaps the
    quantizer (programmatic dependent launch) and reads (q, sa) only after it ends.
    """
    return a8w4_matmul(quantize_int8(x), b, out)


def fp8_fp4_gemm_nt(a: TensorPair, b: TensorPair, out: torch.Tensor,
                    recipe_a: Sequence[int] = (1, 128), recipe_b: Sequence[int] = (1, 32)) -> torch.Tensor:
    """FP8 x FP4 GEMM with UE8M0 block scales: the call shape of the reference's A8W4 test.

    The reference calls `deep_gemm.fp8_fp4_gemm_nt(a, b, out, recipe_a=(1, 128),
    recipe_b=(1, 32))` (tests/a8w4.py:48, :70) with
        a = (x  float8_e4m3fn [M, K], sfa float32 [M, K/128])  (powers of two)
        b = (wp uint8 [N, K/2] packed e2m1,  sfw float32 [N, K/32])
    and a preallocated bf16 `out` [M, N]; this runs `arc_fp8_fp4_gemm` on the same
    tensors (block-scaled tcgen05 MMA, fp32 accumulation).
    """
    if tuple(recipe_a) != (1, 128) or tuple(recipe_b) != (1, 32):
        raise ValueError(f"supported recipes: recipe_a=(1, 128), recipe_b=(1, 32); got "
                         f"{tuple(recipe_a)}, {tuple(recipe_b)}")
    x, sfa = a
    wp, sfw = b
    m, k = x.shape
    n, k2 = wp.shape
    assert k == 2 * k2, f"Inner dimensions must match: {k} vs 2*{k2}"
    assert k % 128 == 0, f"K ({k}) must be a multiple of 128"
    dev = x.device
    _expect(x, "a[0]", torch.float8_e4m3fn, (m, k), None)
    _expect(sfa, "a[1]", torch.float32, (m, k // 128), dev)
    _expect(wp, "b[0]", torch.uint8, (n, k // 2), dev)
    _expect(sfw, "b[1]", torch.float32, (n, k // 32), dev)
    _expect(out, "out", torch.bfloat16, (m, n), dev)
    with torch.cuda.device(dev):
        ws = _fp8_fp4_workspace(dev, m, n, k)
        check(lib().arc_fp8_fp4_gemm_ws(x.data_ptr(), sfa.data_ptr(), wp.data_ptr(), sfw.data_ptr(),
                                        out.data_ptr(), m, n, k,
                                        ws.data_ptr() if ws is not None else None,
                                        ws.numel() if ws is not None else 0, _stream_ptr(dev)),
              "arc.fp8_fp4_gemm_nt")
    return out


# One zeroed workspace per (device, stream), grown on demand: the K split of decode-sized
# problems keeps fp32 partials and per-tile counters in it, and every call leaves the
# counters at zero again. Keyed by stream so that calls that may run concurrently (on
# different streams) never share one.
_WORKSPACES: dict = {}


def _fp8_fp4_workspace(dev: torch.device, m: int, n: int, k: int):
    need = ctypes.c_size_t(0)
    check(lib().arc_fp8_fp4_workspace_bytes(m, n, k, ctypes.byref(need)), "arc_fp8_fp4_workspace_bytes")
    if need.value == 0:
        return None
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need.value:
        ws = torch.zeros(need.value + 256, dtype=torch.uint8, device=dev)
        off = (-ws.data_ptr()) % 256  # 256-byte aligned view
        ws = ws[off:off + need.value]
        _WORKSPACES[key] = ws
    return ws
