"""Small numeric helpers with the reference's names and meaning (arc/math.py:14-41).

* `symm_square_rel_L2_error(x, y)` = 1 - 2<x,y>/(<x,x>+<y,y>) in float64, the pass
  criterion of the reference's A8W4 check (tests/a8w4.py:53-54);
* `count_bytes(*tensors)` sums element bytes, descending into (data, scale) pairs, as
  the reference's GB/s numbers do (tests/a8w4.py:77-83);
* `ceil_div`, `align`.
"""
from __future__ import annotations

import torch


def symm_square_rel_L2_error(x: torch.Tensor, y: torch.Tensor) -> float:
    x = x.double()
    y = y.double()
    den = (x * x + y * y).sum()
    if float(den) == 0.0:
        return 0.0
    return float(1.0 - 2.0 * (x * y).sum() / den)


def count_bytes(*tensors) -> int:
    total = 0
    for t in tensors:
        if isinstance(t, (tuple, list)):
            total += count_bytes(*t)
        elif t is not None:
            total += t.numel() * t.element_size()
    return total


def ceil_div(x: int, y: int) -> int:
    return (x + y - 1) // y


def align(x: int, y: int) -> int:
    return ceil_div(x, y) * y


__all__ = ["symm_square_rel_L2_error", "count_bytes", "ceil_div", "align"]
