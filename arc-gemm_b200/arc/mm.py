"""bf16 matmul: the drop-in for the reference's `arc.matmul` (arc/mm.py:71-79).

`matmul(a, b, out=None)` computes out[M, N] = a[M, K] . b[N, K]^T in bf16 with fp32
accumulation, `b` being K-major ("NT"), exactly as the reference's entry point.
The reference JIT-compiles on first call and launches a 128x128 one-tile-per-CTA
kernel; this one calls the AOT-built persistent sm_100a kernel through the C ABI
(`arc_matmul_bf16`, include/arc_b200.h) on the caller's current stream.

Shapes: the reference asserts M % 32 == 0, N % 128 == 0, K % 128 == 0
(arc/mm.py:75). Every such shape is accepted here; so are other sizes as long as the
rows are 16-byte aligned (leading dimensions multiples of 8 elements).
"""
from __future__ import annotations

import torch

from ._lib import check, lib


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda_bf16(t: torch.Tensor, name: str) -> None:
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path), got {t.device}")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")


def _row_major(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(1) == 1 and t.stride(0) >= t.shape[1] else t.contiguous()


def matmul(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    m, k = a.shape
    n, _k = b.shape
    assert k == _k, f"Inner dimensions must match: {k} vs {_k}"
    _require_cuda_bf16(a, "a")
    _require_cuda_bf16(b, "b")
    if b.device != a.device:
        raise ValueError(f"a and b are on different devices ({a.device}, {b.device})")
    a = _row_major(a)
    b = _row_major(b)
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=a.device)
    else:
        _require_cuda_bf16(out, "out")
        if tuple(out.shape) != (m, n) or out.device != a.device or out.stride(1) != 1:
            raise ValueError(f"out must be a row-major bf16 [{m}, {n}] tensor on {a.device}")
    with torch.cuda.device(a.device):
        check(lib().arc_matmul_bf16(a.data_ptr(), b.data_ptr(), out.data_ptr(), m, n, k,
                                    a.stride(0), b.stride(0), out.stride(0),
                                    _stream_ptr(a.device)),
              "arc.matmul")
    return out
