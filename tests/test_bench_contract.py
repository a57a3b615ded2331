"""CPU: bench.py's command-line contract.

* `--impl reference` (the reference's CPU path, timed on the host) prints one JSON line
  with the keys the driver reads, `impl: reference`, a `cpu_baseline` describing the run
  and an `e2e` with no host<->device bytes;
* fewer than 3 warm-up steps are refused;
* our arm fails loudly without a GPU (there is no CPU fallback).
"""
from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def _bench(*args: str, timeout: int = 240) -> subprocess.CompletedProcess:
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_json_line():
    r = _bench("--impl", "reference", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["n_gpus"] == 1 and d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["config"]["workload"] == "a8w4_decode_m16_n4096_k4096"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_warmup_below_three_is_refused():
    r = _bench("--impl", "reference", "--steps", "3", "--warmup", "2", timeout=120)
    assert r.returncode != 0
    assert "warmup" in (r.stdout + r.stderr)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_our_arm_fails_without_a_gpu():
    r = _bench("--steps", "3", "--warmup", "3", timeout=180)
    assert r.returncode != 0
    assert not r.stdout.strip(), "no JSON line may be printed without a GPU"
