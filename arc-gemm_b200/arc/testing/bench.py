"""Device timers with the semantics of the reference's arc/testing/bench.py.

* `do_bench(fn, warmup, rep)`: CUDA events around each call, an L2 flush (a buffer
  write larger than the 126 MB L2) before every timed call, mean milliseconds
  (reference: arc/testing/bench.py:227-276, with a 256 MB flush buffer);
* `do_bench_cudagraph(fn, n_calls)`: `n_calls` back-to-back calls captured in one CUDA
  graph and replayed; milliseconds per call (reference: bench.py:279-336).

All timings are taken on the stream the work is launched on.
"""
from __future__ import annotations

from typing import Callable

import torch

FLUSH_BYTES = 256 * 1024 * 1024


def _flush_buffer(device=None) -> torch.Tensor:
    return torch.empty(FLUSH_BYTES // 4, dtype=torch.int32, device=device or "cuda")


def do_bench(fn: Callable[[], object], warmup: int = 5, rep: int = 20,
             flush_l2: bool = True) -> float:
    """Mean milliseconds per call over `rep` timed calls (after `warmup` untimed ones)."""
    cache = _flush_buffer() if flush_l2 else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(rep)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(rep)]
    for i in range(rep):
        if cache is not None:
            cache.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    return sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / rep


def do_bench_cudagraph(fn: Callable[[], object], n_calls: int = 20, replays: int = 5) -> float:
    """Milliseconds per call, from replays of a graph holding `n_calls` calls."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(n_calls):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(replays):
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record(stream)
            graph.replay()
            e.record(stream)
            e.synchronize()
            times.append(s.elapsed_time(e) / n_calls)
    del graph
    return sum(times) / len(times)


__all__ = ["do_bench", "do_bench_cudagraph", "FLUSH_BYTES"]
