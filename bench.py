"""Benchmark of the arc A8W4 GEMM on B200 (the BASELINE metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME] [--no-extras] [--allgather nccl|fused|none]
                    [--prepacked]

Prints ONE JSON line on rank 0.

Headline (top-level fields): BASELINE configs[1], A8W4 decode M=16, N=4096, K=4096 -
int8 activations with per-token fp32 scales, int4 weights packed two per byte with bf16
per-(column, 128-group) scales, bf16 output; seeded synthetic data. A step is one GEMM
over one batch. With N GPUs each rank owns its own 4096-column slice of an N*4096-column
weight (weak scaling) and the step includes the all-gather of the output, fused into the
decode GEMM's epilogue (each rank's kernel stores its tiles into every rank's output over
NVLink, then a flag barrier).

Sub-objects of the same line (default; --no-extras drops them):
  N = 1:  "prefill"   A8W4 M=4096, N=14336, K=4096 (tensor-bound),
          "bf16_2048" and "bf16_8192" (configs[0], [3]) with torch.mm (cuBLAS) timed on the
          same inputs beside them, "sweep_m16" and "sweep_m1024".
  every N: "sweep_m16", "sweep_m1024": N=28672, K=8192, the weight columns split over the N
          GPUs (strong scaling) with the all-gather of the output in the step (fused for
          M=16, NCCL for M=1024); "bf16_8192" likewise (NCCL all-gather of the output).
Every sub-object carries value, ms_per_step, roofline, clocks, and (on rank 0) parity_ok: the
last step's output against the CPU oracle on sampled rows and columns.

Timing: W untimed warm-up steps, then exactly K steps between barrier + synchronize on both
sides, on the launching stream with CUDA events, max over ranks. Short steps are captured
K at a time in one CUDA graph and replayed; L2 reuse between steps is prevented by rotating
through enough copies of the inputs (at distinct addresses) to exceed twice the 126 MB L2,
or, when one input set alone exceeds that, by a 512 MB write before every timed step
(outside the step's events). `value` is whole-job throughput (2*M*N*K per step over all
ranks). `e2e` repeats the headline (and the prefill) through the public Python API with
host (pinned) buffers: every step copies its inputs host->device and the output
device->host. Model weights are never written by the kernel before a GEMM, so the A8W4
calls pass static_weights=True (the decode kernel streams its weights while the previous
launch finishes; see include/arc_b200.h, ARC_A8W4_STATIC_WEIGHTS).

`--impl reference` times the reference's CPU path for the same workload on rank 0
(dequantize + fp32 matmul on all host threads; the reference itself has no CPU
implementation of this op), and prints the same fields and the same `config`.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT / "arc-gemm_b200", ROOT):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
METRIC = "A8W4 GEMM TOPS & HBM GB/s vs roofline, M in {16,4096}, 1/2/4/8 B200"

# N is per GPU for weak scaling, in total (split over the GPUs) for strong scaling.
WORKLOADS = {
    "decode": dict(kind="a8w4", M=16, N=4096, K=4096, scaling="weak", gather="fused"),
    "prefill": dict(kind="a8w4", M=4096, N=14336, K=4096, scaling="weak", gather="none"),
    "bf16_2048": dict(kind="bf16", M=2048, N=2048, K=2048, scaling="weak", gather="none"),
    "bf16_8192": dict(kind="bf16", M=8192, N=8192, K=8192, scaling="strong", gather="nccl"),
    **{f"sweep_m{m}": dict(kind="a8w4", M=m, N=28672, K=8192, scaling="strong",
                           gather="fused" if m <= 32 else "nccl")
       for m in (1, 16, 128, 1024, 8192)},
    # The recipe of the reference's own A8W4 test: e4m3 x e2m1 with UE8M0 block scales.
    "fp8fp4_prefill": dict(kind="fp8fp4", M=4096, N=14336, K=4096, scaling="weak", gather="none"),
    "fp8fp4_decode": dict(kind="fp8fp4", M=16, N=4096, K=4096, scaling="weak", gather="none"),
}
EXTRAS_SINGLE = ("prefill", "bf16_2048", "bf16_8192", "sweep_m16", "sweep_m1024")
EXTRAS_MULTI = ("sweep_m16", "sweep_m1024", "bf16_8192")


def a8w4_bytes(M, N, K, group=128):
    return M * K + 4 * M + N * K // 2 + 2 * N * (K // group) + 2 * M * N


def bf16_bytes(M, N, K):
    return 2 * (M * K + N * K + M * N)


def fp8fp4_bytes(M, N, K):
    return M * K + 4 * M * (K // 128) + N * K // 2 + 4 * N * (K // 32) + 2 * M * N


def algorithmic_bytes(kind, M, N, K):
    return {"a8w4": a8w4_bytes, "bf16": bf16_bytes, "fp8fp4": fp8fp4_bytes}[kind](M, N, K)


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {
            "hbm_gbs": float(d["hbm_gbs"]),
            "bf16_tflops": float(d["bf16_tflops"]),
            "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
            "source": "measured",
        }
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
            "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def traffic_from_profiles(workload: str, kind: str = "a8w4", n_rank: int | None = None):
    """DRAM bytes per launch from a committed ncu summary, if one exists. A record taken
    at another number of weight columns (column sharding) is scaled to this rank's share
    for A8W4, whose traffic is the weights'; other kinds report none then."""
    f = ROOT / "profiles" / f"traffic_{workload}.json"
    if not f.exists():
        return None
    try:
        rec = json.loads(f.read_text())
    except (ValueError, OSError):
        return None
    val = rec.get("dram_bytes_per_launch")
    n_rec = rec.get("N")
    if val is None or n_rank is None or n_rec is None or n_rec == n_rank:
        return val
    return int(val * n_rank / n_rec) if kind == "a8w4" else None


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 200 ms while the benchmark runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"arc_clocks_{os.getpid()}_{time.monotonic_ns()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smmax=float(parts[2]),
                                 power=float(parts[3]), util=float(parts[4]),
                                 reasons=[n for n, v in zip(
                                     ("hw_slowdown", "hw_thermal_slowdown",
                                      "sw_thermal_slowdown", "sw_power_cap"),
                                     parts[5:9]) if v.lower() == "active"]))
            except ValueError:
                continue
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [r for r in rows if r["util"] > 0] or rows
        reasons = sorted({x for r in loaded for x in r["reasons"]})
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded),
                "sm_max_mhz": max(r["smmax"] for r in rows),
                "power_w_max": max(r["power"] for r in rows),
                "samples_under_load": len(loaded),
                "reasons": reasons}


# ------------------------------------------------------------------------ distributed
def dist_setup(args):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world > 1 and args.impl == "ours":
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    import torch

    if world > 1:
        import torch.distributed as dist

        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def all_ranks_ok(ok: bool, world: int) -> bool:
    if world == 1:
        return ok
    import torch
    import torch.distributed as dist

    t = torch.tensor([0 if ok else 1], dtype=torch.int32, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return int(t.item()) == 0


# ----------------------------------------------------------------------------- shapes
def shape_of(wl, world):
    """(M, N per rank, N in total) of a workload at this world size."""
    if wl["scaling"] == "weak":
        return wl["M"], wl["N"], wl["N"] * world
    return wl["M"], wl["N"] // world, wl["N"]


def gather_mode(args, wl, world):
    if world == 1:
        return "none"
    mode = args.allgather if args.allgather is not None else wl["gather"]
    if mode == "fused" and (wl["kind"] != "a8w4" or wl["M"] > 32 or args.prepacked):
        mode = "nccl"  # the fused gather covers the A8W4 decode kernel on the reference packing
    return mode


def config_of(name, wl, world, gather):
    """The workload description; both arms print exactly this dict."""
    M, n_rank, n_total = shape_of(wl, world)
    cfg = {"workload": f"{wl['kind']}_{name}_m{M}_n{n_total}_k{wl['K']}",
           "M": M, "N": n_total, "N_per_gpu": n_rank, "K": wl["K"],
           "parallelism": f"column-shard{world}" if world > 1 else "single",
           "allgather": {"none": None,
                         "nccl": "NCCL all_gather_into_tensor of the bf16 output, every step",
                         "fused": "fused into the GEMM epilogue: TMA stores of every tile into "
                                  "each rank's output over NVLink + a flag barrier, every step"}[gather]}
    if wl["kind"] == "a8w4":
        cfg.update(group=128, activations="int8 + fp32 per-token scale",
                   weights="int4 packed x2 + bf16 per-(column,128) scale")
    elif wl["kind"] == "fp8fp4":
        cfg.update(recipe_a="(1, 128)", recipe_b="(1, 32)",
                   activations="e4m3 + UE8M0 scale per (token, 128-K block)",
                   weights="e2m1 packed x2 + UE8M0 scale per (row, 32-K block)")
    else:
        cfg.update(dtype="bf16 x bf16, fp32 accumulate")
    return cfg


# ----------------------------------------------------------------------- reference arm
def cpu_reference_a8w4(M, N, K, steps, warmup, budget_s=None):
    """Reference CPU path on the host cores: (seconds per step, reps, threads)."""
    import numpy as np
    import torch

    from arc.testing.data import generate_a8w4
    from oracle import oracle

    threads = oracle.host_threads()
    torch.set_num_threads(threads)
    (x, sa), (wp, sb) = generate_a8w4(M, N, K, seed=0)
    xs, sas, wps = x.numpy(), sa.numpy(), wp.numpy()
    sbs = sb.view(torch.int16).numpy().view(np.uint16)

    def step():
        oracle.cpu_baseline_a8w4(xs, sas, wps, sbs)

    for _ in range(warmup):
        step()
    if budget_s is not None:
        sec, reps = oracle.time_cpu_baseline(step, budget_s=budget_s)
        return sec, reps, threads
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    return (time.perf_counter() - t0) / steps, steps, threads


def run_reference(args, name, wl, world, rank):
    if rank != 0:
        return
    if wl["kind"] != "a8w4":
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference arm covers the A8W4 workloads only"}))
        return
    M, _, n_total = shape_of(wl, world)
    K = wl["K"]
    sec, reps, threads = cpu_reference_a8w4(M, n_total, K, args.steps, args.warmup)
    ops = 2 * M * n_total * K
    tops = ops / sec / 1e12
    line = {
        "impl": "reference", "metric": METRIC,
        "value": tops, "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": wl["scaling"], "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(name, wl, world, gather_mode(args, wl, world)),
        "hbm_gbs": a8w4_bytes(M, n_total, K) / sec / 1e9,
        "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": f"the whole {M}x{n_total}x{K} problem x {reps} steps: dequantize "
                                   "int8/int4 with their scales + fp32 torch.matmul on the host cores"},
        "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


# ------------------------------------------------------------------------------ inputs
def make_inputs(wl, world, rank, device, seed):
    """Full-problem inputs on the host (every rank generates the same) and this rank's
    device copy: returns (host_full, device_local)."""
    import torch

    from arc import parallel as par
    from arc.testing.data import generate_a8w4, generate_bf16

    M, n_rank, n_total = shape_of(wl, world)
    K = wl["K"]
    lo, hi = (rank * n_rank, (rank + 1) * n_rank)
    if wl["kind"] == "a8w4":
        (x, sa), (wp, sb) = generate_a8w4(M, n_total, K, seed=seed)
        host = ((x, sa), (wp, sb))
        dev = ((x.to(device), sa.to(device)), (wp[lo:hi].to(device), sb[lo:hi].to(device)))
    elif wl["kind"] == "fp8fp4":
        from arc import quant

        g = torch.Generator().manual_seed(seed)
        a = torch.randn(M, K, generator=g).to(torch.bfloat16)
        b = torch.randn(n_total, K, generator=g).to(torch.bfloat16)
        qa = quant.per_token_cast_to_fp8(a, use_ue8m0=True, gran_k=128)
        qb = quant.per_token_cast_to_fp4(b, use_ue8m0=True, gran_k=32)
        host = (qa, qb)
        dev = ((qa[0].to(device), qa[1].to(device)), (qb[0][lo:hi].to(device), qb[1][lo:hi].to(device)))
    else:
        a, b = generate_bf16(M, n_total, K, seed=seed)
        host = (a, b)
        dev = (a.to(device), par.shard_columns(b, rank, world).to(device))
    return host, dev


def clone_set(dev_set):
    """A copy of a device input set at new addresses (same values)."""
    def c(x):
        return tuple(c(t) for t in x) if isinstance(x, tuple) else x.clone()

    return c(dev_set)


def input_bytes(dev_set):
    def b(x):
        return sum(b(t) for t in x) if isinstance(x, tuple) else x.numel() * x.element_size()

    return b(dev_set)


# ----------------------------------------------------------------------------- timing
def time_steps(call, n_sets, args, stream, world, use_graph, flush, collective):
    """W warm-up steps, then exactly K timed steps; returns (step_ms, kernel_ms).

    call(i) runs step i on input set i % n_sets. With a graph, the K steps are replayed
    between two events (step_ms == kernel_ms). Otherwise each step is bracketed by its
    own events and an L2 flush (if any) runs between steps, outside them.
    """
    import torch

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            if flush is not None:
                flush.zero_()
            call(i % n_sets)
        torch.cuda.synchronize()
        graph = None
        if use_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(args.steps):
                    call(i % n_sets)
            graph.replay()  # one untimed replay
            torch.cuda.synchronize()
        # Bring clocks to a steady state before the timed region (untimed). With a
        # collective in the step every rank runs the same number of steps.
        if collective:
            reps = max(1, int(args.settle_s * 2000) // args.steps) if graph is not None else 20
            for r in range(reps):
                if graph is not None:
                    graph.replay()
                else:
                    call(r % n_sets)
            torch.cuda.synchronize()
        else:
            t_end = time.time() + args.settle_s
            while time.time() < t_end:
                if graph is not None:
                    graph.replay()
                else:
                    for i in range(4):
                        if flush is not None:
                            flush.zero_()
                        call(i % n_sets)
                torch.cuda.synchronize()
        barrier(world)
        if graph is not None:
            ev0 = torch.cuda.Event(enable_timing=True)
            ev1 = torch.cuda.Event(enable_timing=True)
            ev0.record(stream)
            graph.replay()
            ev1.record(stream)
            barrier(world)
            step_ms = ev0.elapsed_time(ev1) / args.steps
            kernel_ms = step_ms
        else:
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            for i in range(args.steps):
                if flush is not None:
                    flush.zero_()  # L2 flush between timed steps (outside the step events)
                starts[i].record(stream)
                call(i % n_sets)
                ends[i].record(stream)
            barrier(world)
            kernel_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
            step_ms = kernel_ms  # flush time excluded
        del graph
    return step_ms, kernel_ms


def kernel_launched(kind, M, N, K):
    """The kernel the library launches for this shape (as ncu names it)."""
    import arc
    from arc import _lib

    op = {"a8w4": _lib.OP_A8W4, "fp8fp4": _lib.OP_FP8_FP4}.get(kind, _lib.OP_MATMUL_BF16)
    return arc.kernel_name(op, M, N, K)


def roofline(kind, M, n_rank, K, kernel_ms, peaks, name):
    """Roofline record of the dominant kernel of one rank (one launch per step)."""
    ops = 2 * M * n_rank * K
    by = algorithmic_bytes(kind, M, n_rank, K)
    bound = "hbm" if (kind in ("a8w4", "fp8fp4") and M <= 128) else "tensor"
    if bound == "hbm":
        achieved, peak, unit = by / (kernel_ms * 1e-3) / 1e9, peaks["hbm_gbs"], "GB/s"
        note = f"hbm_gbs ({peaks['source']})"
    else:
        achieved = ops / (kernel_ms * 1e-3) / 1e12
        if kind == "bf16":
            peak, unit, note = peaks["bf16_tflops"], "TFLOP/s", f"bf16_tflops ({peaks['source']})"
        else:
            peak = 2.0 * peaks["bf16_tflops"]  # kind::i8 / kind::mxf8f6f4 issue at twice kind::f16
            unit = "TOPS" if kind == "a8w4" else "TFLOP/s"
            note = f"2 x bf16_tflops ({peaks['source']}): dense int8/fp8 = 2x dense bf16"
    return {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": traffic_from_profiles(name, kind, n_rank), "peak_source": note,
            "algorithmic_per_launch": by if bound == "hbm" else ops,
            "algorithmic_unit": "bytes" if bound == "hbm" else "ops",
            "kernel": kernel_launched(kind, M, n_rank, K)}


# --------------------------------------------------------------------- one workload
class Runner:
    """Times one workload on this rank; builds its record (rank 0 prints)."""

    def __init__(self, args, name, world, rank, local, stream, peaks):
        import torch

        self.args, self.name, self.world, self.rank = args, name, world, rank
        self.wl = WORKLOADS[name]
        self.device = torch.device("cuda", local)
        self.local = local
        self.stream = stream
        self.peaks = peaks
        self.gather = gather_mode(args, self.wl, world)

    def run(self, with_e2e: bool, with_cpu: bool):
        import torch

        import arc
        from arc import parallel as par

        wl, world = self.wl, self.world
        kind = wl["kind"]
        M, n_rank, n_total = shape_of(wl, world)
        K = wl["K"]
        host, dev0 = make_inputs(wl, world, self.rank, self.device, seed=17)
        in_bytes = input_bytes(dev0)
        # Enough copies of the inputs that consecutive steps never find theirs in L2.
        n_sets = max(1, min(64, -(-2 * L2_BYTES // in_bytes)))
        sets = [dev0] + [clone_set(dev0) for _ in range(n_sets - 1)]
        outs = [torch.empty((M, n_rank), dtype=torch.bfloat16, device=self.device) for _ in range(n_sets)]
        flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.int32, device=self.device) if n_sets == 1 else None
        prepacked = self.args.prepacked and kind == "a8w4"
        if prepacked:
            for st in sets:
                arc.prepack_weights(st[1][0], out=st[1][0])
            torch.cuda.synchronize(self.device)

        def gemm(st, out):
            if kind == "a8w4":
                return arc.a8w4_matmul(st[0], st[1], out, prepacked=prepacked, static_weights=True)
            if kind == "fp8fp4":
                return arc.fp8_fp4_gemm_nt(st[0], st[1], out, recipe_a=(1, 128), recipe_b=(1, 32))
            return arc.matmul(st[0], st[1], out)

        fused = None
        gathered = None
        launches = 1
        if self.gather == "fused":
            fused = par.FusedGather(M, n_total, device=self.device)
            launches = 2

            def call(i):
                return fused.matmul(sets[i][0], sets[i][1], static_weights=True)
        elif self.gather == "nccl":
            import torch.distributed as dist

            gathered = torch.empty((world * M, n_rank), dtype=torch.bfloat16, device=self.device)

            def call(i):
                dist.all_gather_into_tensor(gathered, gemm(sets[i], outs[i]))
                return gathered
        else:
            def call(i):
                return gemm(sets[i], outs[i])

        use_graph = flush is None and not self.args.no_graph and self.gather != "nccl"
        with ClockSampler(self.local) as clocks:
            step_ms, kernel_ms = time_steps(call, n_sets, self.args, self.stream, world, use_graph,
                                            flush, collective=self.gather != "none")
            # The last timed step ran on set (K-1) % n_sets: check it against the oracle.
            last = (self.args.steps - 1) % n_sets
            if fused is not None:
                result = fused.out
            elif gathered is not None:  # [world, M, N/world] blocks -> [M, N]
                result = gathered.view(world, M, n_rank).permute(1, 0, 2).reshape(M, n_total)
            else:  # this rank's columns; rank 0's start at column 0
                result = outs[last]
            torch.cuda.synchronize(self.device)
            parity = self.parity(host, result, result.shape[1])
            parity = all_ranks_ok(parity, world)
            e2e = None
            if with_e2e:
                e2e = run_e2e(self.args, kind, sets[0], self.device, self.stream, world,
                              fused=fused, gather_nccl=self.gather == "nccl", prepacked=prepacked)
        if fused is not None:
            fused.close()
        clk = clocks.summary()
        step_ms = max_over_ranks(step_ms, world)
        kernel_ms = max_over_ranks(kernel_ms, world)
        e2e_ms = max_over_ranks(e2e["ms_per_step"], world) if e2e is not None else None
        ops_total = 2 * M * n_total * K
        unit = "TOPS" if kind == "a8w4" else "TFLOP/s"
        rec = {
            "value": ops_total / (step_ms * 1e-3) / 1e12, "unit": unit, "ms_per_step": step_ms,
            "scaling": wl["scaling"],
            "config": config_of(self.name, wl, world, self.gather),
            "timing": {
                "l2": (f"{n_sets} copies of the inputs at distinct addresses "
                       f"({n_sets * in_bytes / 1e6:.0f} MB) > L2") if flush is None
                      else f"L2 flushed ({2 * L2_BYTES >> 20} MiB write) before every timed step, outside its events",
                "launch": (f"K steps ({launches} launch(es) each) in one CUDA graph" if use_graph
                           else "eager launches"),
                "static_weights": kind == "a8w4",
                "weights_layout": "pre-packed (arc.prepack_weights, outside the timed region)"
                                  if prepacked else "reference packing"},
            "hbm_gbs": world * algorithmic_bytes(kind, M, n_rank, K) / (step_ms * 1e-3) / 1e9,
            "roofline": roofline(kind, M, n_rank, K, kernel_ms, self.peaks, self.name),
            "parity_ok": parity,
            "gpu_launches": self.args.steps * launches,
            "clocks": clk,
        }
        if self.gather != "none":
            rec["roofline"]["note"] = ("the step's time includes the all-gather; achieved counts "
                                       "this rank's GEMM work over the whole step")
        kname = rec["roofline"]["kernel"]
        if self.gather == "fused" and kname.startswith("gemm_a8w4_decode_kernel<") and kname.endswith(", 0>"):
            # the last template argument of the decode kernel is the fused-gather flag
            rec["roofline"]["kernel"] = kname[:-2] + "1>"
        if e2e is not None:
            rec["e2e"] = {"value": ops_total / (e2e_ms * 1e-3) / 1e12, "unit": unit,
                          "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                          "ms_per_step": e2e_ms}
        if with_cpu and world == 1 and kind == "a8w4" and self.rank == 0:
            sec, reps, threads = cpu_reference_a8w4(M, n_total, K, 0, 1, budget_s=self.args.cpu_budget_s)
            rec["cpu_baseline"] = {
                "value": ops_total / sec / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
                "sample": f"full {M}x{n_total}x{K} problem x {reps} reps (~{self.args.cpu_budget_s:.0f} s): "
                          "dequantize + fp32 torch.matmul on the host cores"}
        if kind == "bf16" and world == 1:
            rec["vs_cublas"] = self.torch_mm(sets, n_sets, flush, use_graph, step_ms)
        return rec

    def parity(self, host, result, n_cols) -> bool:
        """Sampled rows and columns of the (gathered) output against the CPU oracle."""
        if self.rank != 0:
            return True
        import numpy as np
        import torch

        from oracle import oracle

        kind = self.wl["kind"]
        M = result.shape[0]
        g = np.random.default_rng(7)
        rows = np.sort(g.choice(M, size=min(M, 16), replace=False))
        cols = np.sort(g.choice(n_cols, size=min(n_cols, 256), replace=False))
        got = result.float().cpu().numpy()[np.ix_(rows, cols)]
        if kind == "a8w4":
            (x, sa), (wp, sb) = host
            if self.args.prepacked:
                pass  # the GEMM ran on pre-packed copies of the same weights: same results
            ref = oracle.a8w4_out(x.numpy()[rows], sa.numpy()[rows], wp.numpy()[cols],
                                  sb.view(torch.int16).numpy().view(np.uint16)[cols])
            ok, _ = oracle.check_bf16_close(got, ref, max_ulp=2.0)
        elif kind == "fp8fp4":
            (x, sfa), (wp, sfw) = host
            ref = oracle.fp8fp4_out(x.view(torch.uint8).numpy()[rows], sfa.numpy()[rows], wp.numpy()[cols],
                                    sfw.numpy()[cols])
            ok, _ = oracle.check_bf16_close(got, ref, max_ulp=2.0, atol=oracle.tensor_core_atol(x.shape[1], ref))
        else:
            a, b = host
            ref = oracle.bf16_gemm(a.view(torch.int16).numpy().view(np.uint16)[rows],
                                   b.view(torch.int16).numpy().view(np.uint16)[cols])
            ok, _ = oracle.check_bf16_close(got, ref, max_ulp=2.0, atol=oracle.tensor_core_atol(a.shape[1], ref))
        return bool(ok)

    def torch_mm(self, sets, n_sets, flush, use_graph, our_ms):
        """torch.mm (cuBLAS) on the same inputs, timed the same way (the reference's own
        comparison point, tests/matmul.py:66-81)."""
        import torch

        M, n_rank = sets[0][0].shape[0], sets[0][1].shape[0]
        outs = [torch.empty((M, n_rank), dtype=torch.bfloat16, device=self.device) for _ in range(n_sets)]

        def call(i):
            return torch.mm(sets[i][0], sets[i][1].T, out=outs[i])

        ms, _ = time_steps(call, n_sets, self.args, self.stream, 1, use_graph, flush, collective=False)
        ops = 2 * M * n_rank * sets[0][0].shape[1]
        return {"torch_mm_ms": ms, "torch_mm_tflops": ops / (ms * 1e-3) / 1e12, "speedup": ms / our_ms}


def run_e2e(args, kind, s, device, stream, world, fused=None, gather_nccl=False, prepacked=False):
    """Host buffers in, host buffer out, through the public API, K steps.

    fused: the FusedGather whose matmul is the step (output: the gathered [M, N_total]);
    gather_nccl: follow the GEMM with the NCCL all-gather of its output, as the timed step
    does. The weights are copied in every step, so the call does not claim static weights.
    """
    import torch

    import arc

    if kind in ("a8w4", "fp8fp4"):
        (x, sa), (wp, sb) = s
        host = [t.cpu().pin_memory() for t in (x, sa, wp, sb)]
        dev_bufs = [torch.empty_like(t) for t in (x, sa, wp, sb)]
        m, n = x.shape[0], wp.shape[0]
    else:
        a, b = s
        host = [t.cpu().pin_memory() for t in (a, b)]
        dev_bufs = [torch.empty_like(t) for t in (a, b)]
        m, n = a.shape[0], b.shape[0]
    n_out = n * world if (fused is not None or gather_nccl) else n
    out_h = torch.empty((m, n_out), dtype=torch.bfloat16).pin_memory()
    out_d = torch.empty((m, n), dtype=torch.bfloat16, device=device)
    if gather_nccl:
        import torch.distributed as dist

        gathered = torch.empty((world * m, n), dtype=torch.bfloat16, device=device)

    def step():
        for h, d in zip(host, dev_bufs):
            d.copy_(h, non_blocking=True)
        if fused is not None:
            o = fused.matmul((dev_bufs[0], dev_bufs[1]), (dev_bufs[2], dev_bufs[3]))
        elif kind == "a8w4":
            o = arc.a8w4_matmul((dev_bufs[0], dev_bufs[1]), (dev_bufs[2], dev_bufs[3]), out_d,
                                prepacked=prepacked)
        elif kind == "fp8fp4":
            o = arc.fp8_fp4_gemm_nt((dev_bufs[0], dev_bufs[1]), (dev_bufs[2], dev_bufs[3]), out_d)
        else:
            o = arc.matmul(dev_bufs[0], dev_bufs[1], out_d)
        if gather_nccl:
            dist.all_gather_into_tensor(gathered, o)
            o = gathered.view(world, m, n).permute(1, 0, 2).reshape(m, world * n)
        out_h.copy_(o, non_blocking=True)

    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = out_h.numel() * out_h.element_size()
    with torch.cuda.stream(stream):
        for _ in range(max(args.warmup, 3)):
            step()
        barrier(world)
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        barrier(world)
    return {"ms_per_step": ev0.elapsed_time(ev1) / args.steps, "h2d": h2d, "d2h": d2h}


def run_ours(args, world, rank, local):
    import torch

    stream = torch.cuda.Stream(torch.device("cuda", local))
    peaks = load_peaks()
    head = Runner(args, args.workload, world, rank, local, stream, peaks)
    rec = head.run(with_e2e=True, with_cpu=not args.skip_cpu_baseline)
    extras = {}
    if not args.no_extras and args.workload == "decode":
        for name in (EXTRAS_SINGLE if world == 1 else EXTRAS_MULTI):
            sub = Runner(args, name, world, rank, local, stream, peaks)
            extras[name] = sub.run(with_e2e=(name == "prefill"),
                                   with_cpu=(name == "prefill" and not args.skip_cpu_baseline))
            torch.cuda.empty_cache()
    if rank != 0:
        return
    wl = WORKLOADS[args.workload]
    line = {
        "metric": {"a8w4": METRIC,
                   "fp8fp4": "FP8xFP4 (UE8M0 block scales) GEMM TFLOP/s vs roofline"}.get(
                       wl["kind"], "bf16 GEMM TFLOP/s vs roofline"),
        "value": rec["value"], "unit": rec["unit"], "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
        "scaling": rec["scaling"], "vs_baseline": None,
        "dtype": {"a8w4": "int8xint4->int32, fp32 scale, bf16 out",
                  "fp8fp4": "e4m3 x e2m1, UE8M0 block scales, fp32 accumulate, bf16 out"}.get(
                      wl["kind"], "bf16"),
        "data": "synthetic (seeded, BASELINE distributions)",
    }
    line.update({k: v for k, v in rec.items() if k not in ("value", "unit", "ms_per_step", "scaling")})
    line.update(extras)
    print(json.dumps(line))


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="decode")
    ap.add_argument("--no-extras", action="store_true", help="only the headline workload")
    ap.add_argument("--allgather", choices=("nccl", "fused", "none"), default=None,
                    help="gather mode of the headline for N > 1 (default: the workload's)")
    ap.add_argument("--prepacked", action="store_true",
                    help="A8W4: weights converted once by arc.prepack_weights before timing")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--settle-s", type=float, default=1.0)
    ap.add_argument("--cpu-budget-s", type=float, default=8.0)
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    wl = WORKLOADS[args.workload]
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, args.workload, wl, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
