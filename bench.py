"""Benchmark of asrback's decoder-step attention on B200 (one replica per GPU).

Workload: Whisper large-v3-turbo decoder attention in
bf16, 4 decoder layers, 20 heads x 64, batch 64 slots whose self-attention
lengths start uniform in [1, 448] and grow by one per step (rows that reach
position 447, the last the cache holds, stay computed as in the reference),
cross-attention over 1500 encoder frames whose keys/values come from N(0, 1)
encoder states through the decoder's own k/v projections (seeded weights).
One step = the attention of one greedy decoder step: per layer, the
self-attention with its key/value write, then the cross-attention; the 8
launches of a step replay from one CUDA graph. Unit: decoded tokens (64 per
step per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

``--impl reference`` times the reference's CPU path for the same workload (the
CPU oracle port of its attention, float32, all host threads) on a bounded
sample of rows. Under torchrun every rank runs its own replica (weak scaling,
no collective on the data path); rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "decoder tokens/s/GPU (batch 64, bf16) at 1/2/4/8 B200; attention HBM GB/s"
UNIT = "tokens/s"

BATCH, HEADS, HEAD_DIM, LAYERS = 64, 20, 64, 4
TARGET, SOURCE, WIDTH = 448, 1500, 1280
SEED = 1


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=128)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("native", "reference"), default="native")
    parser.add_argument("--cpu-sample-rows", type=int, default=16,
                        help="rows of the batch the CPU baseline times per step")
    parser.add_argument("--cpu-seconds", type=float, default=10.0,
                        help="time budget of the CPU baseline sample")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    return parser.parse_args()


def config_dict(n_gpus: int) -> dict:
    return {
        "workload": "whisper-large-v3-turbo decoder-step attention (BASELINE config 2)",
        "model": "whisper-large-v3-turbo decoder attention, random init seed 1",
        "layers": LAYERS, "heads": HEADS, "head_dim": HEAD_DIM, "batch_per_gpu": BATCH,
        "global_batch": BATCH * n_gpus, "self_lengths": "U[1,448] at step 0, +1 per step",
        "cross_frames": SOURCE, "step": "per layer: self-attn with KV append, then cross-attn",
        "parallelism": f"replicas x{n_gpus} (no collective)",
        "l2": "inputs larger than L2 (2.26 GB of K/V read per step)",
    }


def initial_lengths(rng: np.random.Generator) -> np.ndarray:
    return rng.integers(1, TARGET + 1, size=BATCH)


def positions_schedule(lengths: np.ndarray, steps: int) -> np.ndarray:
    """(steps, batch) positions: start at length-1, +1 per step, capped at 447."""
    start = lengths - 1
    return np.minimum(start[None, :] + np.arange(steps)[:, None], TARGET - 1).astype(np.int64)


def attention_bytes(positions: np.ndarray) -> tuple[float, float]:
    """Algorithmic K/V bytes of one step: (self, cross), bf16."""
    row = HEADS * HEAD_DIM * 2 * 2  # K and V, bf16
    self_bytes = float(LAYERS * (positions.astype(np.float64) + 1).sum() * row)
    cross_bytes = float(LAYERS * BATCH * SOURCE * row)
    return self_bytes, cross_bytes


# ---------------------------------------------------------------- clocks ----

class ClockSampler:
    """Samples this GPU's SM clock and clock-event (throttle) reasons through
    NVML every 5 ms while the timed region runs (read-only queries)."""

    REASONS = {  # NVML clocks-event reason bits
        0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
        0x4: "sw_power_cap",
    }

    def __init__(self, uuid: str | None) -> None:
        self.uuid = uuid
        self.samples: list[tuple[float, float, int]] = []
        self.error = None

    def _handle(self, nvml):
        count = nvml.nvmlDeviceGetCount()
        for i in range(count):
            handle = nvml.nvmlDeviceGetHandleByIndex(i)
            uuid = nvml.nvmlDeviceGetUUID(handle)
            uuid = uuid.decode() if isinstance(uuid, bytes) else uuid
            if self.uuid and self.uuid.lower().replace("gpu-", "") in uuid.lower():
                return handle
        return nvml.nvmlDeviceGetHandleByIndex(0) if count == 1 else None

    def _run(self):
        import threading  # noqa: F401

        try:
            import pynvml as nvml

            nvml.nvmlInit()
            handle = self._handle(nvml)
            if handle is None:
                self.error = "no NVML device matches this GPU"
                return
            max_sm = float(nvml.nvmlDeviceGetMaxClockInfo(handle, nvml.NVML_CLOCK_SM))
            while not self._stop.is_set():
                sm = float(nvml.nvmlDeviceGetClockInfo(handle, nvml.NVML_CLOCK_SM))
                reasons = int(nvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
                self.samples.append((sm, max_sm, reasons))
                self._stop.wait(0.005)
        except Exception as exc:  # pragma: no cover - depends on the driver
            self.error = repr(exc)

    def __enter__(self):
        import threading

        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=5)

    def summary(self) -> dict | None:
        if not self.samples:
            return {"error": self.error or "no samples"}
        # Samples taken while the GPU was busy (the timed region is all busy).
        reasons = sorted({name for _, _, bits in self.samples
                          for bit, name in self.REASONS.items() if bits & bit})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples), "reasons": reasons,
                "samples": len(self.samples)}


# ------------------------------------------------------------- CPU oracle ----

def cpu_oracle_rate(seed: int, rows: int, budget_s: float, threads: int) -> dict:
    """Tokens/s of the CPU oracle (float32, the reference's CPU dtype) over
    ``rows`` rows of the workload, stepping until ``budget_s`` seconds have
    passed (at least one step): per step and layer, the self-attention with its
    in-place cache write and the cross-attention, rows spread over ``threads``
    threads (numpy's BLAS kept to one thread each)."""
    steps = 64
    sys.path.insert(0, str(ROOT))
    from oracle import attention as oracle

    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    rng = np.random.default_rng(seed)
    lengths = initial_lengths(rng)[:rows]
    positions = np.minimum(lengths[None, :] - 1 + np.arange(steps)[:, None], TARGET - 1)
    self_k = rng.standard_normal((LAYERS, rows, HEADS, TARGET, HEAD_DIM), dtype=np.float32)
    self_v = rng.standard_normal((LAYERS, rows, HEADS, TARGET, HEAD_DIM), dtype=np.float32)
    cross_k = rng.standard_normal((LAYERS, rows, HEADS, SOURCE, HEAD_DIM), dtype=np.float32)
    cross_v = rng.standard_normal((LAYERS, rows, HEADS, SOURCE, HEAD_DIM), dtype=np.float32)
    q = rng.standard_normal((steps, LAYERS, 4, rows, HEADS, HEAD_DIM), dtype=np.float32)

    def one_row(args):
        t, layer, b = args
        pos = positions[t, b:b + 1]
        oracle.whisper_self_attention_step(
            q[t, layer, 0, b:b + 1], q[t, layer, 1, b:b + 1], q[t, layer, 2, b:b + 1],
            self_k[layer, b:b + 1], self_v[layer, b:b + 1], pos, compute=np.float32, copy=False)
        oracle.whisper_cross_attention(q[t, layer, 3, b:b + 1], cross_k[layer, b:b + 1],
                                       cross_v[layer, b:b + 1], compute=np.float32)

    limit = threadpool_limits(1) if threadpool_limits else None
    try:
        with ThreadPoolExecutor(max_workers=threads) as pool:
            start = time.perf_counter()
            done = 0
            while done < steps:
                for layer in range(LAYERS):
                    list(pool.map(one_row, [(done, layer, b) for b in range(rows)]))
                done += 1
                if time.perf_counter() - start >= budget_s:
                    break
            elapsed = time.perf_counter() - start
    finally:
        if limit is not None and hasattr(limit, "unregister"):
            limit.unregister()
    return {"value": rows * done / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{rows} of {BATCH} rows x {done} steps x {LAYERS} layers "
                      f"(self with in-place append + cross over {SOURCE}), float32 numpy "
                      f"oracle, {elapsed:.1f} s"}


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: rank 0 times the CPU path; other ranks exit."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    result = cpu_oracle_rate(SEED, args.cpu_sample_rows, args.cpu_seconds, threads)
    line = {
        "impl": "reference", "metric": METRIC, "value": result["value"], "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": BATCH / result["value"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args.gpus), "cpu_baseline": result,
        "e2e": {"value": result["value"], "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "reference CPU path = CPU oracle port of the reference's attention "
                "(the Python reference is not present on the GPU box)",
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- native ----

def measured_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def profiled_traffic() -> float | None:
    """DRAM bytes per cross-attention launch from the committed ncu summary."""
    path = ROOT / "profiles" / "whisper_cross_decode_b64_bf16.md"
    try:
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except (OSError, ValueError):
        pass
    return None


def run_native(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from asrback_b200 import attention, whisper
    from asrback_b200.synthetic import seeded_normal, seeded_parameters
    from asrback_b200.transcription import CapturedGraph

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    dtype = torch.bfloat16
    seed = SEED + 1000 * rank
    rng = np.random.default_rng(seed)
    lengths = initial_lengths(rng)
    total = args.warmup + args.steps
    schedule = positions_schedule(lengths, total)

    # Caches and cross K/V through the decoder's own projections (seeded).
    config = whisper.large_v3_turbo_config()
    model = whisper.WhisperForConditionalGeneration(config, encoder=False)
    seeded_parameters(model.model.decoder, SEED)
    model = model.to(device, dtype).eval()
    cache = model.allocate_cache(BATCH)
    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for start in range(0, BATCH, 16):
            states = torch.randn((16, SOURCE, WIDTH), generator=gen, device=device, dtype=dtype)
            part = cache.rows(start, start + 16)
            model.set_encoder_output(part, states)
        for layer in range(LAYERS):
            for b in range(BATCH):
                p = int(lengths[b]) - 1
                if p > 0:
                    cache.self_keys[layer, b, :, :p].normal_(generator=gen)
                    cache.self_values[layer, b, :, :p].normal_(generator=gen)
    del model
    inputs = torch.randn((total, LAYERS, 4, BATCH, HEADS, HEAD_DIM), generator=gen, device=device,
                         dtype=dtype)
    positions_all = torch.from_numpy(schedule).to(device)
    step_in = torch.empty((LAYERS, 4, BATCH, HEADS, HEAD_DIM), device=device, dtype=dtype)
    pos = torch.empty((BATCH,), device=device, dtype=torch.int64)
    outputs: dict[int, torch.Tensor] = {}

    def step():
        for layer in range(LAYERS):
            outputs[2 * layer] = attention.whisper_self_attention_step(
                step_in[layer, 0], step_in[layer, 1], step_in[layer, 2],
                cache.self_keys[layer], cache.self_values[layer], pos)
            outputs[2 * layer + 1] = attention.whisper_cross_attention_step(
                step_in[layer, 3], cache.cross_keys[layer], cache.cross_values[layer])

    # Warm-up (eager) and capture, like the reference's CapturedGraph; the
    # warm-up steps advance positions too (their share of the schedule).
    step_in.copy_(inputs[0])
    pos.copy_(positions_all[0])
    graph = CapturedGraph(step)
    for t in range(args.warmup):
        step_in.copy_(inputs[t])
        pos.copy_(positions_all[t])
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    stream = torch.cuda.current_stream()
    uuid = getattr(torch.cuda.get_device_properties(device), "uuid", None)
    uuid = f"GPU-{uuid}" if uuid and not str(uuid).startswith("GPU-") else (str(uuid) if uuid else None)

    # ---- timed region: device-resident inputs, graph replay per step ----
    start_ev, end_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(uuid) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.nvtx.range_push("timed")
        start_ev.record(stream)
        for t in range(args.warmup, total):
            step_in.copy_(inputs[t])
            pos.copy_(positions_all[t])
            graph.replay()
        end_ev.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = start_ev.elapsed_time(end_ev)
    if world > 1:
        t_max = torch.tensor([ms], device=device)
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        ms = float(t_max.item())
    ms_per_step = ms / args.steps
    value = BATCH * world * args.steps / (ms / 1e3)

    # ---- kernel timing: average launch duration of each kernel, launched
    # back to back from a captured graph (no host launch cost in the way) ----
    kernel_ms = {}
    launches = 4 * LAYERS
    t_kernel = args.warmup

    def cross_only():
        for i in range(launches):
            layer = i % LAYERS
            attention.whisper_cross_attention_step(
                inputs[t_kernel, layer, 3], cache.cross_keys[layer], cache.cross_values[layer])

    def self_only():
        for i in range(launches):
            layer = i % LAYERS
            attention.whisper_self_attention_step(
                inputs[t_kernel, layer, 0], inputs[t_kernel, layer, 1], inputs[t_kernel, layer, 2],
                cache.self_keys[layer], cache.self_values[layer], positions_all[t_kernel])

    for name, fn in (("cross", cross_only), ("self", self_only)):
        kgraph = CapturedGraph(fn, warmup=1)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        kgraph.replay()
        torch.cuda.synchronize()
        a.record(stream)
        for _ in range(4):
            kgraph.replay()
        b.record(stream)
        torch.cuda.synchronize()
        kernel_ms[name] = a.elapsed_time(b) / (4 * launches)
        del kgraph
    self_bytes, cross_bytes = attention_bytes(schedule[args.warmup:])
    self_bytes_kernel, _ = attention_bytes(schedule[t_kernel:t_kernel + 1])
    self_bytes_per_launch = self_bytes_kernel / LAYERS
    cross_bytes_per_launch = cross_bytes / LAYERS
    peak, peak_kind = measured_peak()
    achieved = cross_bytes_per_launch / (kernel_ms["cross"] * 1e-3) / 1e9
    step_bytes = (self_bytes / args.steps + cross_bytes)

    # ---- e2e: pinned host inputs in, outputs back, every step ----
    host_in = torch.empty((args.steps,) + tuple(step_in.shape), dtype=dtype, pin_memory=True)
    host_in.copy_(inputs[args.warmup:total].cpu())
    host_pos = torch.from_numpy(schedule[args.warmup:]).pin_memory()
    out_list = [outputs[i] for i in range(2 * LAYERS)]
    out_bytes = sum(o.numel() * o.element_size() for o in out_list)
    host_out = torch.empty((args.steps, out_bytes), dtype=torch.uint8, pin_memory=True)
    in_bytes = step_in.numel() * step_in.element_size() + BATCH * 8
    # Restore the warm-up state's positions so e2e decodes the same schedule.
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for i in range(args.steps):
        step_in.copy_(host_in[i], non_blocking=True)
        pos.copy_(host_pos[i], non_blocking=True)
        graph.replay()
        offset = 0
        for o in out_list:
            n = o.numel() * o.element_size()
            host_out[i, offset:offset + n].copy_(o.view(-1).view(torch.uint8), non_blocking=True)
            offset += n
    e_end.record(stream)
    torch.cuda.synchronize()
    e_ms = e_start.elapsed_time(e_end)
    if world > 1:
        t_max = torch.tensor([e_ms], device=device)
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
        e_ms = float(t_max.item())
    e2e = BATCH * world * args.steps / (e_ms / 1e3)

    status = attention.read_status(device)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        cpu = cpu_oracle_rate(SEED, args.cpu_sample_rows, args.cpu_seconds, threads)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config_dict(world),
            "e2e": {"value": e2e, "unit": UNIT, "h2d_bytes_per_step": in_bytes,
                    "d2h_bytes_per_step": out_bytes},
            "roofline": {"bound": "hbm", "kernel": "decode_attention_kernel (cross, Whisper)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": peak_kind,
                         "traffic": profiled_traffic(),
                         "algorithmic_bytes_per_launch": cross_bytes_per_launch,
                         "launch_ms": kernel_ms["cross"]},
            "kernels": {
                "self_attention_ms": kernel_ms["self"],
                "self_attention_gbs": self_bytes_per_launch / (kernel_ms["self"] * 1e-3) / 1e9,
                "cross_attention_ms": kernel_ms["cross"],
                "cross_attention_gbs": achieved,
                "step_attention_gbs": step_bytes / (ms_per_step * 1e-3) / 1e9,
            },
            "gpu_launches": 2 * LAYERS * args.steps,
            "clocks": clocks.summary(),
            "cpu_baseline": cpu,
            "device_status": status,
        }
        print(json.dumps(line), flush=True)


def main() -> None:
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3 and args.impl == "native":
        print("bench.py: --warmup below 3 is not allowed", file=sys.stderr)
        sys.exit(2)
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_native(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
