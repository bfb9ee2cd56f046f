"""bench.py's command line and its reference arm, on the CPU.

The reference arm (`--impl reference`) times the CPU oracle port of the
reference's path; it needs no GPU, so the JSON contract of its line is checked
here: the keys the driver reads, a positive value, and the end-to-end entry
with no host<->device bytes. Under torchrun only rank 0 prints it.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                          text=True, env=env, timeout=300, cwd=str(ROOT))


@pytest.mark.parametrize("workload", ["whisper-prefix", "whisper-encoder"])
def test_reference_arm_line_keeps_the_contract(workload):
    done = _run(["--impl", "reference", "--workload", workload, "--cpu-seconds", "0.2",
                 "--steps", "4", "--warmup", "3"])
    assert done.returncode == 0, done.stderr[-2000:]
    lines = [line for line in done.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["value"] > 0 and line["steps"] == 4 and line["warmup"] == 3
    assert line["scaling"] == "weak" and line["higher_is_better"] is True
    assert isinstance(line["config"], dict) and "workload" in line["config"]
    base = line["cpu_baseline"]
    assert base["value"] == line["value"] and base["unit"] == line["unit"]
    assert base["cores"] >= 1 and base["kind"] in ("port", "reference") and base["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": line["unit"],
                           "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_prints_on_rank_zero_only():
    done = _run(["--impl", "reference", "--workload", "whisper-prefix", "--cpu-seconds", "0.2"],
                {"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert done.returncode == 0, done.stderr[-2000:]
    assert not [line for line in done.stdout.splitlines() if line.startswith("{")]


def test_every_workload_is_on_the_command_line(monkeypatch):
    for name in bench.WORKLOADS:
        monkeypatch.setattr(sys, "argv", ["bench.py", "--workload", name, "--batch", "8",
                                          "--layers", "2", "--no-extras"])
        args = bench.parse_args()
        assert args.workload == name and args.batch == 8 and args.layers == 2
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    args = bench.parse_args()
    assert args.workload == "whisper-decode" and args.gpus == 1 and args.warmup >= 3


def test_serving_trace_is_seeded_and_deals_rows_evenly():
    """The config-5 trace: Poisson arrivals at 25 requests/s per GPU, prompts of
    13 audio positions per second of U[1, 30] s audio plus 20 text positions,
    the same on every rank, and an equal share of requests per replica."""
    import numpy as np

    work = bench.WORKLOADS["qwen3-serve"](None)
    for world in (1, 2, 8):
        trace = work.trace(world, 192 * world)
        again = work.trace(world, 192 * world)
        assert [(r.arrival, r.length) for r in trace] == [(r.arrival, r.length) for r in again]
        counts = np.bincount([r.replica for r in trace], minlength=world)
        assert counts.tolist() == [192] * world
        arrivals = np.array([r.arrival for r in trace])
        assert (np.diff(arrivals) > 0).all()
        rate = len(trace) / arrivals[-1]
        assert 0.8 * 25 * world < rate < 1.2 * 25 * world
        lengths = np.array([r.length for r in trace])
        assert lengths.min() >= 13 + 20 and lengths.max() <= 390 + 20
