"""arc — B200-native GEMMs behind the reference's `arc` Python entry points.

Public API (the reference exports `arc.matmul` and `arc.vecadd`, arc/__init__.py:1-7;
the GEMM path is what this package covers):

* `matmul(a, b, out=None)`            bf16 NT GEMM (drop-in for arc/mm.py:71)
* `a8w4_matmul((x, sa), (wp, sb), out=None)`  int8 x int4 GEMM with group-128 scales
* `a8w4_gemm_nt(a, b, out, recipe_a, recipe_b)`  the same with deep_gemm's call shape
* `prepack_weights(wp)`               packed int4 weights -> the kernels' expand layout
  (`a8w4_matmul(..., prepacked=True)`)
* `quantize_int8(x)`                  bf16 activations -> (int8, per-token fp32 scale) on the GPU
* `a8w4_matmul_bf16(x, (wp, sb))`     quantize_int8 followed by the A8W4 GEMM
* `fp8_fp4_gemm_nt(a, b, out, recipe_a, recipe_b)`  FP8 x FP4 with UE8M0 block scales, the
  recipe and call shape of the reference's own A8W4 test
* `quant`, `math`, `parallel`, `testing` helpers

The kernels are AOT-built into libarcb200.so for sm_100a (`python -m arc.build`).
"""
from . import math, parallel, quant
from ._lib import ArcError, describe_plan, device_status, kernel_name, version
from .a8w4 import (a8w4_gemm_nt, a8w4_matmul, a8w4_matmul_bf16, fp8_fp4_gemm_nt, prepack_weights,
                   quantize_int8)
from .mm import matmul

__all__ = [
    "matmul",
    "a8w4_matmul",
    "a8w4_gemm_nt",
    "a8w4_matmul_bf16",
    "fp8_fp4_gemm_nt",
    "quantize_int8",
    "prepack_weights",
    "ArcError",
    "describe_plan",
    "device_status",
    "kernel_name",
    "version",
    "math",
    "parallel",
    "quant",
]
