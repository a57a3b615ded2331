"""Benchmark of the arc A8W4 GEMM on B200 (the BASELINE metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|prefill|bf16_2048|bf16_8192]
                    [--allgather [nccl|fused]] [--prepacked]

Prints ONE JSON line on rank 0.

Workload (default "decode"): BASELINE configs[1], A8W4 M=16, N=4096, K=4096 — int8
activations with per-token fp32 scales, int4 weights packed two per byte with bf16
per-(column, 128-group) scales, bf16 output; seeded synthetic data. A step is one
GEMM over one batch. With N GPUs each rank owns its own 4096-column slice of an
N*4096-column weight (weak scaling, no collective in the data path; `--allgather`
adds the NCCL all-gather of the output, `--allgather fused` the all-gather fused into
the decode GEMM's epilogue). `--prepacked` runs the A8W4 GEMM on weights converted once,
before timing, by arc.prepack_weights.

Timing: W untimed warm-up steps, then exactly K steps between barrier +
synchronize on both sides, on the launching stream with CUDA events, max over ranks.
The decode kernel is a few microseconds long, so the K launches are captured in one
CUDA graph and replayed; between steps L2 reuse is prevented by rotating through
enough distinct input sets to exceed the 126 MB L2. `value` is whole-job TOPS
(2*M*N*K per rank per step). `e2e` repeats the measurement through the public
Python API with host (pinned) buffers: every step copies all of its inputs
host->device and the output device->host.

`--impl reference` times the reference's CPU path for the same workload on rank 0
(dequantize + fp32 matmul on all host threads; the reference itself has no CPU
implementation of this op), and prints the same JSON fields.
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

WORKLOADS = {
    "decode": dict(kind="a8w4", M=16, N=4096, K=4096),
    "prefill": dict(kind="a8w4", M=4096, N=14336, K=4096),
    "bf16_2048": dict(kind="bf16", M=2048, N=2048, K=2048),
    "bf16_8192": dict(kind="bf16", M=8192, N=8192, K=8192),
    # The recipe of the reference's own A8W4 test: e4m3 x e2m1 with UE8M0 block scales.
    "fp8fp4_prefill": dict(kind="fp8fp4", M=4096, N=14336, K=4096),
    "fp8fp4_decode": dict(kind="fp8fp4", M=16, N=4096, K=4096),
}


def a8w4_bytes(M, N, K, group=128):
    return M * K + 4 * M + N * K // 2 + 2 * N * (K // group) + 2 * M * N


def bf16_bytes(M, N, K):
    return 2 * (M * K + N * K + M * N)


def fp8fp4_bytes(M, N, K):
    return M * K + 4 * M * (K // 128) + N * K // 2 + 4 * N * (K // 32) + 2 * M * N


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


def traffic_from_profiles(workload: str):
    """DRAM bytes per launch from a committed ncu summary, if one exists."""
    f = ROOT / "profiles" / f"traffic_{workload}.json"
    if f.exists():
        try:
            return json.loads(f.read_text()).get("dram_bytes_per_launch")
        except (ValueError, OSError):
            return None
    return None


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 200 ms while the benchmark runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"arc_clocks_{os.getpid()}.csv"

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


# ----------------------------------------------------------------------------- arms
def cpu_reference_value(wl, steps, warmup, budget_s=None):
    """Reference CPU path on the host cores: (seconds per step, reps, threads)."""
    import numpy as np
    import torch

    from arc.testing.data import generate_a8w4
    from oracle import oracle

    threads = oracle.host_threads()
    torch.set_num_threads(threads)
    M, N, K = wl["M"], wl["N"], wl["K"]
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


def run_reference(args, wl, world, rank):
    if rank != 0:
        return
    if wl["kind"] != "a8w4":
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference arm covers the A8W4 workloads only"}))
        return
    sec, reps, threads = cpu_reference_value(wl, args.steps, args.warmup)
    ops = 2 * wl["M"] * wl["N"] * wl["K"]
    tops = ops / sec / 1e12
    line = {
        "impl": "reference",
        "metric": "A8W4 GEMM TOPS & HBM GB/s vs roofline, M in {16,4096}, 1/2/4/8 B200",
        "value": tops, "unit": "TOPS", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(args, wl, world),
        "hbm_gbs": a8w4_bytes(wl["M"], wl["N"], wl["K"]) / sec / 1e9,
        "cpu_baseline": {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port",
                         "sample": f"full {wl['M']}x{wl['N']}x{wl['K']} problem x {reps} steps: "
                                   "dequantize int8/int4 with their scales + fp32 torch.matmul "
                                   "on the host cores"},
        "e2e": {"value": tops, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def config_of(args, wl, world):
    cfg = {"workload": f"{wl['kind']}_{args.workload}_m{wl['M']}_n{wl['N']}_k{wl['K']}",
           "M": wl["M"], "N_per_gpu": wl["N"], "K": wl["K"],
           "parallelism": f"column-shard{world}" if world > 1 else "single"}
    if wl["kind"] == "a8w4":
        cfg.update(group=128, activations="int8 + fp32 per-token scale",
                   weights="int4 packed x2 + bf16 per-(column,128) scale")
    elif wl["kind"] == "fp8fp4":
        cfg.update(recipe_a="(1, 128)", recipe_b="(1, 32)",
                   activations="e4m3 + UE8M0 scale per (token, 128-K block)",
                   weights="e2m1 packed x2 + UE8M0 scale per (row, 32-K block)")
    return cfg


def build_inputs(wl, rank, device, n_sets):
    import torch

    from arc.testing.data import generate_a8w4, generate_bf16

    sets = []
    for i in range(n_sets):
        seed = 1000 * rank + i
        if wl["kind"] == "a8w4":
            (x, sa), (wp, sb) = generate_a8w4(wl["M"], wl["N"], wl["K"], seed=seed)
            out = torch.empty((wl["M"], wl["N"]), dtype=torch.bfloat16, device=device)
            sets.append(((x.to(device), sa.to(device)), (wp.to(device), sb.to(device)), out))
        elif wl["kind"] == "fp8fp4":
            from arc import quant

            g = torch.Generator(device=device).manual_seed(seed)
            a = torch.randn(wl["M"], wl["K"], generator=g, device=device, dtype=torch.bfloat16)
            b = torch.randn(wl["N"], wl["K"], generator=g, device=device, dtype=torch.bfloat16)
            out = torch.empty((wl["M"], wl["N"]), dtype=torch.bfloat16, device=device)
            sets.append((quant.per_token_cast_to_fp8(a, use_ue8m0=True, gran_k=128),
                         quant.per_token_cast_to_fp4(b, use_ue8m0=True, gran_k=32), out))
        else:
            a, b = generate_bf16(wl["M"], wl["N"], wl["K"], seed=seed, device=device)
            out = torch.empty((wl["M"], wl["N"]), dtype=torch.bfloat16, device=device)
            sets.append((a, b, out))
    return sets


def kernel_launched(wl, M, N, K):
    """The kernel the library launches for this workload's shape (as ncu names it)."""
    import arc
    from arc import _lib
    op = {"a8w4": _lib.OP_A8W4, "fp8fp4": _lib.OP_FP8_FP4}.get(wl["kind"], _lib.OP_MATMUL_BF16)
    return arc.kernel_name(op, M, N, K)


def run_ours(args, wl, world, rank, local):
    import torch

    import arc

    device = torch.device("cuda", local)
    M, N, K = wl["M"], wl["N"], wl["K"]
    ops = 2 * M * N * K
    if wl["kind"] == "a8w4":
        step_bytes = a8w4_bytes(M, N, K)
        in_bytes = step_bytes - 2 * M * N

        def call(s):
            # Model weights are written once, never by the kernel before a GEMM.
            return arc.a8w4_matmul(s[0], s[1], s[2], prepacked=args.prepacked, static_weights=True)
    elif wl["kind"] == "fp8fp4":
        step_bytes = fp8fp4_bytes(M, N, K)
        in_bytes = step_bytes - 2 * M * N

        def call(s):
            return arc.fp8_fp4_gemm_nt(s[0], s[1], s[2], recipe_a=(1, 128), recipe_b=(1, 32))
    else:
        step_bytes = bf16_bytes(M, N, K)
        in_bytes = step_bytes - 2 * M * N

        def call(s):
            return arc.matmul(s[0], s[1], s[2])

    # Enough distinct input sets that consecutive steps never find theirs in L2.
    n_sets = max(1, min(64, -(-2 * L2_BYTES // in_bytes)))
    sets = build_inputs(wl, rank, device, n_sets)
    if args.prepacked:
        if wl["kind"] != "a8w4":
            raise SystemExit("--prepacked applies to the A8W4 workloads")
        # One-time weight format step, outside the timed region. Its own kernel time is
        # reported beside the line: out-of-place calls over every set's weights into one
        # scratch buffer, enqueued back to back behind a GPU sleep so that the events
        # bracket device work only (HBM-bound; the sets' weights exceed L2).
        scratch = torch.empty_like(sets[0][1][0])
        arc.prepack_weights(sets[0][1][0], out=scratch)  # untimed first call (library setup)
        torch.cuda.synchronize(device)
        pp0 = torch.cuda.Event(enable_timing=True)
        pp1 = torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(5_000_000)  # ~2.5 ms: the host enqueues every call meanwhile
        pp0.record()
        for st in sets:
            arc.prepack_weights(st[1][0], out=scratch)
        pp1.record()
        torch.cuda.synchronize(device)
        pp_us = pp0.elapsed_time(pp1) * 1e3 / len(sets)
        del scratch
        for st in sets:
            arc.prepack_weights(st[1][0], out=st[1][0])
        torch.cuda.synchronize(device)
        pp_bytes = 2 * N * K // 2  # every packed byte read once and written once
        prepack_info = {"us_per_call": pp_us, "bytes_per_call": pp_bytes,
                        "gbs": pp_bytes / (pp_us * 1e-6) / 1e9, "calls": len(sets)}
    flush = None
    if n_sets == 1:  # inputs alone exceed 2x L2 only for the large configs
        flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.int32, device=device)
    gather = args.allgather if world > 1 else None
    launches_per_step = 1
    if gather == "nccl":
        # Each step also all-gathers the bf16 output over NCCL into [world*M, N/world]
        # (arc.parallel.gather_columns' layout); eager launches, no graph.
        import torch.distributed as dist

        gathered = torch.empty((world * M, N), dtype=torch.bfloat16, device=device)
        local_call = call

        def call(s):
            out = local_call(s)
            dist.all_gather_into_tensor(gathered, out)
            return gathered
    elif gather == "fused":
        # The GEMM stores its tiles into every rank's [M, world*N] output over NVLink,
        # then a flag barrier (arc.parallel.FusedGather); eager launches, no graph.
        if wl["kind"] != "a8w4" or M > 32 or args.prepacked:
            raise SystemExit("--allgather fused covers the A8W4 decode workload (M <= 32, "
                             "reference packing)")
        from arc import parallel as par

        fused = par.FusedGather(M, world * N, device=device)
        launches_per_step = 2

        def call(s):
            return fused.matmul(s[0], s[1], static_weights=True)
    # The fused gather's barrier keeps its epoch on the device, so its steps capture into
    # a graph like the GEMM alone; the NCCL gather runs eagerly.
    use_graph = flush is None and not args.no_graph and gather != "nccl"
    stream = torch.cuda.Stream(device)
    peaks = load_peaks()

    with ClockSampler(local) as clocks:
        with torch.cuda.stream(stream):
            for i in range(max(args.warmup, 3)):
                call(sets[i % n_sets])
            torch.cuda.synchronize()
            graph = None
            if use_graph:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for i in range(args.steps):
                        call(sets[i % n_sets])
                graph.replay()  # one untimed replay
                torch.cuda.synchronize()
            # Bring clocks to a steady state before the timed region (untimed). With a
            # collective in the step every rank must run the same number of steps, so
            # that case settles for a fixed count instead of a wall-clock time.
            if gather:
                if graph is not None:
                    for _ in range(max(1, int(args.settle_s * 2000) // args.steps)):
                        graph.replay()
                else:
                    for i in range(int(args.settle_s * 2000)):
                        call(sets[i % n_sets])
                torch.cuda.synchronize()
            t_end = time.time() + (0.0 if gather else args.settle_s)
            while time.time() < t_end:
                if graph is not None:
                    graph.replay()
                else:
                    for i in range(4):
                        if flush is not None:
                            flush.zero_()
                        call(sets[i % n_sets])
                torch.cuda.synchronize()

            barrier(world)
            if graph is not None:
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record(stream)
                graph.replay()
                ev1.record(stream)
                barrier(world)
                elapsed_ms = ev0.elapsed_time(ev1)
                kernel_ms = elapsed_ms / args.steps
            else:
                starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
                ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
                ev0 = torch.cuda.Event(enable_timing=True)
                ev1 = torch.cuda.Event(enable_timing=True)
                ev0.record(stream)
                for i in range(args.steps):
                    if flush is not None:
                        flush.zero_()  # L2 flush between timed steps (outside the step events)
                    starts[i].record(stream)
                    call(sets[i % n_sets])
                    ends[i].record(stream)
                ev1.record(stream)
                barrier(world)
                kernel_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends)) / args.steps
                elapsed_ms = kernel_ms * args.steps  # flush time excluded
            del graph

            # e2e through the public API with pinned host buffers (untimed warm-up first).
            e2e = run_e2e(args, wl, sets[0], device, stream, world,
                          gemm=(fused.matmul if gather == "fused" else None),
                          gather_nccl=(gather == "nccl"))
            if gather == "fused":
                fused.close()

    clk = clocks.summary()
    step_ms = max_over_ranks(elapsed_ms / args.steps, world)
    kernel_ms = max_over_ranks(kernel_ms, world)
    e2e_ms = max_over_ranks(e2e["ms_per_step"], world)
    if rank != 0:
        return
    value = world * ops / (step_ms * 1e-3) / 1e12
    if wl["kind"] in ("a8w4", "fp8fp4"):
        bound = "hbm" if M <= 128 else "tensor"
    else:
        bound = "tensor"
    if bound == "hbm":
        achieved = step_bytes / (kernel_ms * 1e-3) / 1e9
        peak, unit = peaks["hbm_gbs"], "GB/s"
        peak_note = f"hbm_gbs ({peaks['source']})"
    else:
        achieved = ops / (kernel_ms * 1e-3) / 1e12
        if wl["kind"] == "a8w4":
            peak = 2.0 * peaks["bf16_tflops"]  # kind::i8 issues at twice the kind::f16 rate
            peak_note = f"2 x bf16_tflops ({peaks['source']}): dense int8 = 2x dense bf16"
        elif wl["kind"] == "fp8fp4":
            peak = 2.0 * peaks["bf16_tflops"]  # kind::mxf8f6f4 (e4m3 operands) = int8 rate
            peak_note = f"2 x bf16_tflops ({peaks['source']}): dense fp8 = 2x dense bf16"
        else:
            peak = peaks["bf16_tflops"]
            peak_note = f"bf16_tflops ({peaks['source']})"
        unit = "TOPS" if wl["kind"] == "a8w4" else "TFLOP/s"
    traffic = traffic_from_profiles(args.workload)
    line = {
        "metric": {"a8w4": "A8W4 GEMM TOPS & HBM GB/s vs roofline, M in {16,4096}, 1/2/4/8 B200",
                   "fp8fp4": "FP8xFP4 (UE8M0 block scales) GEMM TFLOP/s vs roofline"}.get(
                       wl["kind"], "bf16 GEMM TFLOP/s vs roofline"),
        "value": value, "unit": "TOPS" if wl["kind"] == "a8w4" else "TFLOP/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {"a8w4": "int8xint4->int32, fp32 scale, bf16 out",
                  "fp8fp4": "e4m3 x e2m1, UE8M0 block scales, fp32 accumulate, bf16 out"}.get(
                      wl["kind"], "bf16"),
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": dict(config_of(args, wl, world),
                       l2=("rotating %d distinct input sets (%.0f MB) > L2" %
                           (n_sets, n_sets * in_bytes / 1e6)) if flush is None
                       else "L2 flushed (512 MB write) before every timed step",
                       launch=(f"K steps ({launches_per_step} launch(es) each) in one CUDA graph"
                               if use_graph else "eager launches"),
                       allgather={"nccl": "NCCL all_gather_into_tensor of the bf16 output every step",
                                  "fused": "fused into the GEMM epilogue: TMA stores of every tile "
                                           "into each rank's output over NVLink + a flag barrier"
                                  }.get(gather, False),
                       weights_layout=("pre-packed (arc.prepack_weights, outside the timed region)"
                                       if args.prepacked else "reference packing")),
        "hbm_gbs": world * step_bytes / (step_ms * 1e-3) / 1e9,
        "roofline": {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": peak_note,
                     "algorithmic_per_launch": step_bytes if bound == "hbm" else ops,
                     "kernel": kernel_launched(wl, M, N, K)},
        "e2e": {"value": world * ops / (e2e_ms * 1e-3) / 1e12,
                "unit": "TOPS" if wl["kind"] == "a8w4" else "TFLOP/s",
                "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"],
                "ms_per_step": e2e_ms},
        "gpu_launches": args.steps * launches_per_step,
        **({"prepack": dict(prepack_info, frac=prepack_info["gbs"] / peaks["hbm_gbs"])}
           if args.prepacked else {}),
        "clocks": clk,
    }
    if world == 1 and wl["kind"] == "a8w4" and not args.skip_cpu_baseline:
        sec, reps, threads = cpu_reference_value(wl, 0, 1, budget_s=args.cpu_budget_s)
        line["cpu_baseline"] = {
            "value": ops / sec / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"full {M}x{N}x{K} problem x {reps} reps (~{args.cpu_budget_s:.0f} s): "
                      "dequantize + fp32 torch.matmul on the host cores"}
    print(json.dumps(line))


def run_e2e(args, wl, s, device, stream, world, gemm=None, gather_nccl=False):
    """Host buffers in, host buffer out, through the public API, K steps.

    gemm: the A8W4 call to time instead of arc.a8w4_matmul (FusedGather.matmul, whose
    output is the gathered [M, world*N]); gather_nccl: follow the GEMM with the NCCL
    all-gather of its output, as the timed step does.
    """
    import torch

    import arc

    if wl["kind"] in ("a8w4", "fp8fp4"):
        (x, sa), (wp, sb), _ = s
        host = [t.cpu().pin_memory() for t in (x, sa, wp, sb)]
        dev_bufs = [torch.empty_like(t) for t in (x, sa, wp, sb)]
        n_out = wl["N"] * world if gemm is not None else wl["N"]
        m_out = wl["M"] * world if gather_nccl else wl["M"]
        out_h = torch.empty((m_out, n_out), dtype=torch.bfloat16).pin_memory()
        out_d = torch.empty((wl["M"], wl["N"]), dtype=torch.bfloat16, device=device)
        if gather_nccl:
            import torch.distributed as dist

            gathered = torch.empty((m_out, n_out), dtype=torch.bfloat16, device=device)

        def step():
            for h, d in zip(host, dev_bufs):
                d.copy_(h, non_blocking=True)
            if gemm is not None:
                o = gemm((dev_bufs[0], dev_bufs[1]), (dev_bufs[2], dev_bufs[3]))
            elif wl["kind"] == "a8w4":
                o = arc.a8w4_matmul((dev_bufs[0], dev_bufs[1]), (dev_bufs[2], dev_bufs[3]),
                                    prepacked=args.prepacked)
                if gather_nccl:
                    dist.all_gather_into_tensor(gathered, o)
                    o = gathered
            else:
                o = arc.fp8_fp4_gemm_nt((dev_bufs[0], dev_bufs[1]), (dev_bufs[2], dev_bufs[3]), out_d)
            out_h.copy_(o, non_blocking=True)
    else:
        a, b, _ = s
        host = [t.cpu().pin_memory() for t in (a, b)]
        dev_bufs = [torch.empty_like(t) for t in (a, b)]
        out_h = torch.empty((wl["M"], wl["N"]), dtype=torch.bfloat16).pin_memory()

        def step():
            for h, d in zip(host, dev_bufs):
                d.copy_(h, non_blocking=True)
            o = arc.matmul(dev_bufs[0], dev_bufs[1])
            out_h.copy_(o, non_blocking=True)

    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = out_h.numel() * out_h.element_size()
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


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="decode")
    ap.add_argument("--allgather", nargs="?", const="nccl", choices=("nccl", "fused"), default=None)
    ap.add_argument("--prepacked", action="store_true",
                    help="A8W4: weights converted once by arc.prepack_weights before timing")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--settle-s", type=float, default=1.0)
    ap.add_argument("--cpu-budget-s", type=float, default=10.0)
    ap.add_argument("--skip-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    wl = WORKLOADS[args.workload]
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            run_reference(args, wl, world, rank)
        else:
            run_ours(args, wl, world, rank, local)
    finally:
        if world > 1 and args.impl == "ours":
            import torch.distributed as dist

            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
