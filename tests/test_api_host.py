"""CPU: argument checking of the Python entry points (nothing reaches a kernel).

The reference raises AssertionError for inner-dimension mismatches (arc/mm.py:74);
the same holds here. There is no CPU path: CPU tensors are rejected loudly.
"""
from __future__ import annotations

import pytest
import torch

import arc
from arc.testing.data import generate_a8w4


def test_matmul_inner_dim_mismatch_asserts():
    with pytest.raises(AssertionError, match="Inner dimensions must match"):
        arc.matmul(torch.zeros(4, 8, dtype=torch.bfloat16), torch.zeros(4, 16, dtype=torch.bfloat16))


def test_matmul_rejects_cpu_tensors():
    a = torch.zeros(32, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        arc.matmul(a, a)


def test_a8w4_inner_dim_mismatch_asserts():
    (x, sa), (wp, sb) = generate_a8w4(4, 16, 256)
    with pytest.raises(AssertionError, match="Inner dimensions"):
        arc.a8w4_matmul((x, sa), (wp[:, :64], sb))


def test_a8w4_rejects_cpu_tensors_and_bad_group():
    (x, sa), (wp, sb) = generate_a8w4(4, 16, 256)
    with pytest.raises(ValueError, match="CUDA"):
        arc.a8w4_matmul((x, sa), (wp, sb))
    with pytest.raises(ValueError, match="group"):
        arc.a8w4_matmul((x, sa), (wp, sb), group=64)


def test_a8w4_gemm_nt_recipes():
    (x, sa), (wp, sb) = generate_a8w4(4, 16, 256)
    out = torch.empty(4, 16, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="recipe_b"):
        arc.a8w4_gemm_nt((x, sa), (wp, sb), out, recipe_b=(1, 32))
    with pytest.raises(ValueError, match="recipe_a"):
        arc.a8w4_gemm_nt((x, sa), (wp, sb), out, recipe_a=(1, 128))


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    """With the shared library absent the API raises instead of computing anything."""
    from arc import _lib

    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "libarcb200.so")
    with pytest.raises(RuntimeError, match="no fallback"):
        _lib.lib()
