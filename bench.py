"""Benchmarks of asrback's attention hot path on B200 (one replica per GPU).

Default workload (the headline configuration): Whisper large-v3-turbo
decoder-step attention in bf16 -- 4 decoder layers, 20 heads x 64, batch 64
slots whose self-attention lengths start uniform in [1, 448] and grow by one
per step (rows that reach position 447, the last the cache holds, stay
computed, as in the reference), cross-attention over 1500 encoder frames whose
keys/values come from N(0, 1) encoder states through seeded k/v projections.
One step = per layer, the self-attention with its key/value write, then the
cross-attention. Unit: decoded tokens (64 per step per GPU).

Other workloads (``--workload``):
  whisper-encoder  encoder self-attention of 32 layers over
                   32 windows of 1500 frames (20 x 64, bf16), non-causal; unit:
                   windows (32 per step);
  qwen3-decode     Qwen3-1.7B-style decode attention, 28
                   layers, 16 query / 8 key-value heads x 128, RoPE theta 1e6,
                   QK-RMSNorm, batch 64 rows whose caches hold the 410-position
                   prompt (390 audio + 20 text positions), then one position
                   per step; unit: decoded tokens;
  qwen3-prefill    causal grouped-query attention within 64 packed 410-token
                   prompts, 28 layers; unit: prompt tokens;
  qwen3-audio      non-causal attention within 104-token audio-encoder
                   windows, 64 requests of 390 tokens, 24 layers;
  whisper-step,    the greedy step epilogue after the decoder (logits against
  qwen3-step       the 51866 x 1280 tied embedding / the 151936 x 2048 lm_head,
                   argmax, log-softmax, state update) for 64 rows; unit: tokens;
  whisper-cross-kv set_encoder_output for 32 windows: the 4 decoder layers'
                   cross-attention keys/values projected into the cache; unit:
                   windows;
  whisper-prefix   the prompt pass's attention for 32 windows of 4 prompt
                   tokens (decode with length=P): causal self-attention and
                   cross-attention over 1500 frames, 4 layers; unit: windows;
  qwen3-serve      continuous-batching serving: a
                   Qwen3-0.6B-style text model (28 layers, hidden 1024) per
                   GPU fed by seeded Poisson arrivals, rows joining with a
                   packed prefill and leaving after their tokens; unit:
                   generated tokens; also timed at the offered load.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
                    [--workload NAME] [--batch B]

Timing: W untimed warm-up steps run eagerly; the K timed steps are captured
as ONE CUDA graph (inputs already in HBM, the step's own inputs per step) and
the timed region is one replay of it, bracketed by a barrier and a
synchronize, timed with CUDA events on the launching stream; the value is the
slowest rank's. The same graph replayed for about ``--sustain-seconds`` gives
the ``sustained`` figure. ``e2e`` runs the same K steps through the public ops
with each step's inputs copied from pinned host memory and its outputs copied
back, double-buffered on two copy streams so the copies overlap the steps.

``--impl reference`` times the reference's CPU path for the same workload:
the reference's attention call written with torch's CPU operators (its
``F.scaled_dot_product_attention`` calls with the same masks and grouped
views), float32 on all host threads, over a bounded sample. Under torchrun
every rank runs its own replica (weak scaling, no collective on the data
path); rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
DECODE_METRIC = "decoder tokens/s/GPU (batch 64, bf16) at 1/2/4/8 B200; attention HBM GB/s"
SEED = 1


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=128)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("native", "reference"), default="native")
    parser.add_argument("--workload", choices=tuple(WORKLOADS), default="whisper-decode")
    parser.add_argument("--batch", type=int, default=None,
                        help="override the workload's batch (small profiling cases)")
    parser.add_argument("--layers", type=int, default=None,
                        help="override the workload's layer count (small profiling cases that "
                             "keep the batch; not a bench line)")
    parser.add_argument("--cpu-seconds", type=float, default=8.0,
                        help="time budget of the CPU baseline sample")
    parser.add_argument("--sustain-seconds", type=float, default=1.0,
                        help="device time of the sustained (repeated graph replay) figure")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-extras", action="store_true",
                        help="skip the short runs of the other workloads in the default line")
    return parser.parse_args()


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

    def _sample(self):
        nvml = self._nvml
        sm = float(nvml.nvmlDeviceGetClockInfo(self._h, nvml.NVML_CLOCK_SM))
        reasons = int(nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h))
        self.samples.append((sm, self._max_sm, reasons))

    def _run(self):
        try:
            while not self._stop.wait(0.005):
                self._sample()
        except Exception as exc:  # pragma: no cover - depends on the driver
            self.error = repr(exc)

    def __enter__(self):
        import threading

        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml as nvml

            nvml.nvmlInit()
            self._nvml = nvml
            self._h = self._handle(nvml)
            if self._h is None:
                self.error = "no NVML device matches this GPU"
                return self
            self._max_sm = float(nvml.nvmlDeviceGetMaxClockInfo(self._h, nvml.NVML_CLOCK_SM))
        except Exception as exc:  # pragma: no cover - depends on the driver
            self.error = repr(exc)
            return self
        # NVML is ready before the timed region starts; sampling runs beside it.
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def mark(self):
        """Takes one sample now (called inside the timed region)."""
        if self._thread is not None:
            try:
                self._sample()
            except Exception as exc:  # pragma: no cover
                self.error = repr(exc)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)

    def summary(self) -> dict:
        if not self.samples:
            return {"error": self.error or "no samples"}
        reasons = sorted({name for _, _, bits in self.samples
                          for bit, name in self.REASONS.items() if bits & bit})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples), "reasons": reasons,
                "samples": len(self.samples)}


def measured_peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def peak_for(bound: str) -> tuple[float, str]:
    peaks = measured_peaks()
    if bound == "hbm":
        if "hbm_gbs" in peaks:
            return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, copy)"
        return 6650.0, "fallback 6.65 TB/s"
    if "bf16_tflops" in peaks:
        return float(peaks["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    return 1590.0, "fallback 1.59 PFLOP/s"


def profiled_traffic(name: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel, from its committed ncu
    summary under profiles/ (a line ``traffic_bytes_per_launch: N``)."""
    path = ROOT / "profiles" / name
    try:
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return float(line.split(":", 1)[1])
    except (OSError, ValueError):
        pass
    return None


def rope_tables(torch, theta: float, dim: int, length: int, device=None, dtype=None):
    """RoPE ``cos``/``sin`` tables ``(length, dim)`` over ``cat(angles,
    angles)``, computed in float32 then cast (as the reference's engine builds
    them, qwen3_asr.py:795-803)."""
    inverse = 1.0 / (theta ** (torch.arange(0, dim, 2).float() / dim))
    angles = torch.arange(length).float()[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos().to(device, dtype), angles.sin().to(device, dtype)


def kv_bucket(length: int, buckets=(128, 256, 512, 768, 1024)) -> int:
    """The reference's Qwen3 key/value view for a step whose longest row holds
    ``length`` keys (qwen3_asr.py:62, :805-816, :1108-1109)."""
    return next(size for size in buckets if size >= length)


def time_cpu(fn, budget_s: float, limit: int = 4096) -> tuple[int, float]:
    """Calls fn(i) for i = 0, 1, ... until ``budget_s`` seconds have passed (at
    least once); returns (calls, seconds)."""
    start = time.perf_counter()
    done = 0
    while True:
        fn(done)
        done += 1
        elapsed = time.perf_counter() - start
        if elapsed >= budget_s or done >= limit:
            return done, elapsed


def cpu_torch(threads: int):
    """torch on the host cores for a CPU baseline (float32, all threads)."""
    import torch

    torch.set_num_threads(threads)
    return torch


def run_numpy_pool(fn, rows, budget_s: float, threads: int):
    """Runs fn(step, row) over rows per step on `threads` threads (numpy, one
    BLAS thread each) until `budget_s` seconds have passed; returns (steps, s)."""
    from concurrent.futures import ThreadPoolExecutor

    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    limit = threadpool_limits(1) if threadpool_limits else None
    try:
        with ThreadPoolExecutor(max_workers=threads) as pool:
            done, elapsed = time_cpu(lambda i: list(pool.map(lambda r: fn(i, r), rows)), budget_s)
    finally:
        if limit is not None and hasattr(limit, "unregister"):
            limit.unregister()
    return done, elapsed


# -------------------------------------------------------------- workloads ----

class Workload:
    """One pass of a hot-path call site over a batch of synthetic inputs.

    ``inputs_at(t)`` are step t's own device inputs (the tensors a caller
    hands the ops each step); ``launch(inputs)`` runs the step's kernels on
    them and returns its outputs. Everything else the step reads (caches,
    weights, later layers' activations) is set up once in HBM."""

    reference_in_graph = False
    episode = 1  # distinct per-step inputs kept in HBM

    def __init__(self, batch: int | None):
        self.batch = batch or self.default_batch

    def inputs_at(self, t: int) -> list:
        return self.inputs

    def step_at(self, t: int) -> list:
        return self.launch(self.inputs_at(t))

    def cpu_rate(self, budget_s: float, threads: int) -> dict:  # pragma: no cover - abstract
        raise NotImplementedError


class WhisperDecode(Workload):
    """The headline: Whisper large-v3-turbo decoder-step attention."""

    name = "whisper-decode"
    metric = DECODE_METRIC
    unit = "tokens/s"
    bound = "hbm"
    reference_in_graph = True
    default_batch = 64
    layers, heads, head_dim, target, source, width = 4, 20, 64, 448, 1500, 1280
    profile = "whisper_cross_decode_b64_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "whisper-large-v3-turbo decoder-step attention (BASELINE config 2)",
            "model": "whisper-large-v3-turbo decoder attention, seeded k/v projections (seed 1)",
            "layers": self.layers, "heads": self.heads, "head_dim": self.head_dim,
            "batch_per_gpu": self.batch, "global_batch": self.batch * world,
            "self_lengths": "U[1,448] at step 0, +1 per step (capped at 447)",
            "cross_frames": self.source,
            "step": "per layer: self-attn with KV append, then cross-attn",
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2 (about 2.26 GB of K/V read per step)",
        }

    def units_per_step(self) -> int:
        return self.batch

    def lengths(self, rng) -> np.ndarray:
        return rng.integers(1, self.target + 1, size=self.batch)

    def setup(self, torch, device, seed: int, steps: int) -> None:
        from asrback_b200 import attention
        from asrback_b200.synthetic import seeded_parameter

        dtype = torch.bfloat16
        rng = np.random.default_rng(seed)
        lengths = self.lengths(rng)
        start = lengths - 1
        self.schedule = np.minimum(start[None, :] + np.arange(steps)[:, None],
                                   self.target - 1).astype(np.int64)
        b, h, d, w = self.batch, self.heads, self.head_dim, self.width
        # The reference's DecoderCache layout: (layers, batch, heads, length, 64).
        self.self_keys = torch.zeros((self.layers, b, h, self.target, d), dtype=dtype,
                                     device=device)
        self.self_values = torch.zeros_like(self.self_keys)
        self.cross_keys = torch.zeros((self.layers, b, h, self.source, d), dtype=dtype,
                                      device=device)
        self.cross_values = torch.zeros_like(self.cross_keys)
        gen = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for layer in range(self.layers):
                prefix = f"layers.{layer}.encoder_attn."
                wk, wv, bv = (seeded_parameter(prefix + name, shape, SEED).to(device, dtype)
                              for name, shape in (("k_proj.weight", (w, w)),
                                                  ("v_proj.weight", (w, w)),
                                                  ("v_proj.bias", (w,))))
                for b0 in range(0, b, 16):
                    b1 = min(b, b0 + 16)
                    states = torch.randn((b1 - b0, self.source, w), generator=gen, device=device,
                                         dtype=dtype)
                    attention.whisper_cross_kv_projection(
                        states, wk, wv, bv, self.cross_keys[layer, b0:b1],
                        self.cross_values[layer, b0:b1])
                for row in range(b):
                    p = int(lengths[row]) - 1
                    if p > 0:
                        self.self_keys[layer, row, :, :p].normal_(generator=gen)
                        self.self_values[layer, row, :, :p].normal_(generator=gen)
        shape = (self.layers, 4, b, h, d)
        self.episode = min(steps, 128)
        self.queries = torch.randn((self.episode,) + shape, generator=gen, device=device,
                                   dtype=dtype)
        self.positions_all = torch.from_numpy(self.schedule).to(device)

    def inputs_at(self, t: int) -> list:
        return [self.queries[t % self.episode], self.positions_all[t]]

    def launch(self, inputs) -> list:
        from asrback_b200 import attention

        x, pos = inputs
        outputs = []
        for layer in range(self.layers):
            outputs.append(attention.whisper_self_attention_step(
                x[layer, 0], x[layer, 1], x[layer, 2], self.self_keys[layer],
                self.self_values[layer], pos))
            outputs.append(attention.whisper_cross_attention_step(
                x[layer, 3], self.cross_keys[layer], self.cross_values[layer]))
        return outputs

    def launches_per_step(self) -> int:
        return 2 * self.layers

    def row_bytes(self) -> int:
        return self.heads * self.head_dim * 2 * 2  # K and V, bf16

    def kernels(self, t: int):
        """(name, launch function of a layer index, algorithmic work of one launch)."""
        from asrback_b200 import attention

        x, pos = self.inputs_at(t)
        self_bytes = float((self.schedule[t] + 1).sum()) * self.row_bytes()
        cross_bytes = float(self.batch * self.source * self.row_bytes())
        return [
            ("cross", lambda layer: attention.whisper_cross_attention_step(
                x[layer, 3], self.cross_keys[layer], self.cross_values[layer]), cross_bytes),
            ("self", lambda layer: attention.whisper_self_attention_step(
                x[layer, 0], x[layer, 1], x[layer, 2], self.self_keys[layer],
                self.self_values[layer], pos), self_bytes),
        ]

    def step_work(self, first: int, count: int) -> float:
        """Algorithmic bytes of steps first..first+count."""
        sched = self.schedule[first:first + count]
        per_row = self.row_bytes() * self.layers
        return float(((sched + 1).sum() + count * self.batch * self.source) * per_row)

    def torch_reference_step(self, torch):
        """The reference's own GPU computation of step t's attention (torch SDPA
        with its bool step mask and cuDNN-first backend priority, as
        whisper.py:58-63 and :222-240 run it), for context."""
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        key_positions = torch.arange(self.target, device=self.queries.device)
        backends = [SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
                    SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]
        rows = torch.arange(self.batch, device=self.queries.device)

        def run(t):
            x, pos = self.inputs_at(t)
            mask = (key_positions[None, :] <= pos[:, None])[:, None, None, :]
            with sdpa_kernel(backends, set_priority=True):
                for layer in range(self.layers):
                    q, k, v, qc = (x[layer, i][:, :, None, :] for i in range(4))
                    self.self_keys[layer][rows, :, pos] = k[:, :, 0]
                    self.self_values[layer][rows, :, pos] = v[:, :, 0]
                    F.scaled_dot_product_attention(q, self.self_keys[layer],
                                                   self.self_values[layer], attn_mask=mask)
                    F.scaled_dot_product_attention(qc, self.cross_keys[layer],
                                                   self.cross_values[layer])
        return run

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The reference's step attention on the host: for each layer, the
        key/value write (``scatter_`` at each row's position) and SDPA with the
        step mask over the 448-position cache, then SDPA over the 1500 cross
        keys (whisper.py:222-240, :262-264), float32, a sample of the rows."""
        torch = cpu_torch(threads)
        import torch.nn.functional as F

        rows, steps = 16, 64
        rng = np.random.default_rng(SEED)
        lengths = self.lengths(rng)[:rows]
        positions = torch.from_numpy(np.minimum(lengths[None, :] - 1 + np.arange(steps)[:, None],
                                                self.target - 1))
        gen = torch.Generator().manual_seed(SEED)
        h, d = self.heads, self.head_dim
        sk = torch.randn((self.layers, rows, h, self.target, d), generator=gen)
        sv = torch.randn(sk.shape, generator=gen)
        ck = torch.randn((self.layers, rows, h, self.source, d), generator=gen)
        cv = torch.randn(ck.shape, generator=gen)
        q = torch.randn((steps, self.layers, 4, rows, h, 1, d), generator=gen)
        key_positions = torch.arange(self.target)

        def one(i):
            t = i % steps
            pos = positions[t]
            mask = (key_positions[None, :] <= pos[:, None])[:, None, None, :]
            index = pos[:, None, None, None].expand(rows, h, 1, d)
            for layer in range(self.layers):
                x = q[t, layer]
                sk[layer].scatter_(2, index, x[1])
                sv[layer].scatter_(2, index, x[2])
                F.scaled_dot_product_attention(x[0], sk[layer], sv[layer], attn_mask=mask)
                F.scaled_dot_product_attention(x[3], ck[layer], cv[layer])

        with torch.inference_mode():
            done, elapsed = time_cpu(one, budget_s)
        return {"value": rows * done / elapsed, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {self.batch} rows x {done} steps x {self.layers} layers "
                          f"(scatter_ append + masked SDPA over 448, SDPA over {self.source}), "
                          f"torch CPU float32, {elapsed:.1f} s"}

    def oracle_rate(self, budget_s: float, threads: int) -> dict:
        """Cross-check: the float64-capable numpy oracle in float32."""
        from oracle import attention as oracle

        rows, steps = 16, 64
        rng = np.random.default_rng(SEED)
        lengths = self.lengths(rng)[:rows]
        positions = np.minimum(lengths[None, :] - 1 + np.arange(steps)[:, None], self.target - 1)
        f32 = np.float32
        sk = rng.standard_normal((self.layers, rows, self.heads, self.target, self.head_dim),
                                 dtype=f32)
        sv = rng.standard_normal(sk.shape, dtype=f32)
        ck = rng.standard_normal((self.layers, rows, self.heads, self.source, self.head_dim),
                                 dtype=f32)
        cv = rng.standard_normal(ck.shape, dtype=f32)
        q = rng.standard_normal((steps, self.layers, 4, rows, self.heads, self.head_dim),
                                dtype=f32)

        def one(t, b):
            t %= steps
            for layer in range(self.layers):
                oracle.whisper_self_attention_step(
                    q[t, layer, 0, b:b + 1], q[t, layer, 1, b:b + 1], q[t, layer, 2, b:b + 1],
                    sk[layer, b:b + 1], sv[layer, b:b + 1], positions[t, b:b + 1],
                    compute=f32, copy=False)
                oracle.whisper_cross_attention(q[t, layer, 3, b:b + 1], ck[layer, b:b + 1],
                                               cv[layer, b:b + 1], compute=f32)

        done, elapsed = run_numpy_pool(one, list(range(rows)), budget_s, threads)
        return {"value": rows * done / elapsed, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{rows} rows x {done} steps, float32 numpy oracle, {elapsed:.1f} s"}


class WhisperEncoder(Workload):
    """Whisper large-v3-turbo encoder self-attention prefill."""

    name = "whisper-encoder"
    metric = "encoder windows/s/GPU (32 windows x 1500 frames, 32 layers, bf16); attention TFLOP/s"
    unit = "windows/s"
    bound = "tensor"
    default_batch = 32
    layers, heads, head_dim, length = 32, 20, 64, 1500
    profile = "whisper_encoder_attention_b32_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "whisper-large-v3-turbo encoder self-attention prefill (BASELINE config 3)",
            "layers": self.layers, "heads": self.heads, "head_dim": self.head_dim,
            "frames": self.length, "batch_per_gpu": self.batch, "global_batch": self.batch * world,
            "step": "32 layers of non-causal attention over the batch's windows",
            "inputs": "N(0,1) bf16 q/k/v per layer in the projections' (B, S, H*D) layout",
            "e2e": "layer 0's q/k/v copied in from the host and the last layer's output copied "
                   "out per step (the layers between keep their activations on the device)",
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2 (369 MB of q/k/v per layer)",
        }

    def units_per_step(self) -> int:
        return self.batch

    def flops_per_layer(self) -> float:
        return 4.0 * self.length ** 2 * self.head_dim * self.heads * self.batch

    def setup(self, torch, device, seed: int, steps: int) -> None:
        gen = torch.Generator(device=device).manual_seed(seed)
        shape = (self.batch, self.length, self.heads * self.head_dim)
        self.qkv = [[torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16)
                     for _ in range(3)] for _ in range(self.layers)]
        self.inputs = list(self.qkv[0])

    def views(self, tensors):
        b, s, h, d = self.batch, self.length, self.heads, self.head_dim
        return [t.view(b, s, h, d).transpose(1, 2) for t in tensors]

    def attend(self, layer: int, tensors=None):
        from asrback_b200 import attention

        return attention.whisper_encoder_attention(*self.views(tensors or self.qkv[layer]))

    def launch(self, inputs) -> list:
        out = self.attend(0, inputs)
        for layer in range(1, self.layers):
            out = self.attend(layer)
        return [out]

    def launches_per_step(self) -> int:
        return self.layers

    def kernels(self, t: int):
        return [("encoder", lambda layer: self.attend(layer), self.flops_per_layer())]

    def step_work(self, first: int, count: int) -> float:
        return self.flops_per_layer() * self.layers * count

    def torch_reference_step(self, torch):
        """The reference's encoder call on the same tensors, eager as the
        reference runs it: torch SDPA, which on B200 with torch 2.11 dispatches
        this shape to cuDNN's sm100 kernel (in a fresh process and after the
        decoder step's cuDNN-first priority context alike; probed with the
        torch profiler). cuDNN is named here so that the figure does not depend
        on what ran before in the bench's process."""
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        def run(_t):
            with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                for layer in range(self.layers):
                    F.scaled_dot_product_attention(*self.views(self.qkv[layer]))
        return run

    def torch_flash_step(self, torch):
        """The same with torch's flash-attention backend forced (SDPA's first
        choice by its priority list; slower than cuDNN for this shape)."""
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        def run(_t):
            with sdpa_kernel([SDPBackend.FLASH_ATTENTION]):
                for layer in range(self.layers):
                    F.scaled_dot_product_attention(*self.views(self.qkv[layer]))
        return run

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The reference's unmasked encoder SDPA (whisper.py:102-110) on the
        host, float32, one window-layer (20 heads x 1500 x 1500) per call."""
        torch = cpu_torch(threads)
        import torch.nn.functional as F

        gen = torch.Generator().manual_seed(SEED)
        q, k, v = (torch.randn((1, self.heads, self.length, self.head_dim), generator=gen)
                   for _ in range(3))
        with torch.inference_mode():
            done, elapsed = time_cpu(lambda i: F.scaled_dot_product_attention(q, k, v), budget_s)
        return {"value": done / elapsed / self.layers, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{done} window-layers (20 heads x 1500 x 1500), torch CPU SDPA "
                          f"float32, {elapsed:.1f} s, scaled by 1/32 layers"}


class Qwen3Decode(Workload):
    """Qwen3-1.7B-style decode attention."""

    name = "qwen3-decode"
    metric = "decoder tokens/s/GPU (Qwen3 1.7B-style, batch 64, bf16); attention HBM GB/s"
    unit = "tokens/s"
    bound = "hbm"
    reference_in_graph = True
    default_batch = 64
    layers, heads, kv_heads, head_dim, cache_length, prompt = 28, 16, 8, 128, 1024, 410
    profile = "qwen3_decode_b64_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "Qwen3-ASR-1.7B-style decode attention (BASELINE config 4)",
            "layers": self.layers, "heads": self.heads, "kv_heads": self.kv_heads,
            "head_dim": self.head_dim, "rope_theta": 1e6, "qk_rmsnorm": True,
            "batch_per_gpu": self.batch, "global_batch": self.batch * world,
            "cache": "(28, batch, 1024, 8, 128) bf16; 410 prompt positions filled with "
                     "N(0,1) keys/values, then one position per step",
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2 (about 3.5 GB of K/V read per step)",
        }

    def units_per_step(self) -> int:
        return self.batch

    def setup(self, torch, device, seed: int, steps: int) -> None:
        dtype = torch.bfloat16
        gen = torch.Generator(device=device).manual_seed(seed)
        shape = (self.layers, self.batch, self.cache_length, self.kv_heads, self.head_dim)
        self.keys = torch.zeros(shape, dtype=dtype, device=device)
        self.values = torch.zeros(shape, dtype=dtype, device=device)
        self.keys[:, :, :self.prompt].normal_(generator=gen)
        self.values[:, :, :self.prompt].normal_(generator=gen)
        self.cos, self.sin = rope_tables(torch, 1e6, self.head_dim, self.cache_length, device,
                                         dtype)
        self.norms = (1 + 0.1 * torch.randn((self.layers, 2, self.head_dim), generator=gen,
                                            device=device)).to(dtype)
        width = (self.heads + 2 * self.kv_heads) * self.head_dim
        self.episode = min(steps, 128)
        self.qkv = torch.randn((self.episode, self.layers, self.batch, width), generator=gen,
                               device=device, dtype=dtype)
        self.schedule = np.minimum(self.prompt + np.arange(steps)[:, None]
                                   + np.zeros((1, self.batch), np.int64),
                                   self.cache_length - 1).astype(np.int64)
        self.positions_all = torch.from_numpy(self.schedule).to(device)

    def inputs_at(self, t: int) -> list:
        return [self.qkv[t % self.episode], self.positions_all[t]]

    def attend(self, layer, qkv, pos):
        from asrback_b200 import attention

        return attention.qwen3_attention_step(
            qkv, self.norms[layer, 0], self.norms[layer, 1], 1e-6, self.cos, self.sin, pos,
            self.keys[layer], self.values[layer], self.heads, self.kv_heads)

    def launch(self, inputs) -> list:
        qkv, pos = inputs
        return [self.attend(layer, qkv[layer], pos) for layer in range(self.layers)]

    def launches_per_step(self) -> int:
        return self.layers

    def row_bytes(self) -> int:
        return self.kv_heads * self.head_dim * 2 * 2

    def kernels(self, t: int):
        qkv, pos = self.inputs_at(t)
        bytes_ = float((self.schedule[t] + 1).sum()) * self.row_bytes()
        return [("qwen3", lambda layer: self.attend(layer, qkv[layer], pos), bytes_)]

    def step_work(self, first: int, count: int) -> float:
        sched = self.schedule[first:first + count]
        return float((sched + 1).sum()) * self.row_bytes() * self.layers

    def torch_reference_step(self, torch):
        """The reference's GPU fallback on torch 2.11 (varlen_attn lacks the
        kwargs it passes): q/k RMSNorm + RoPE in bf16, cache write, SDPA with
        the step mask over the key/value bucket view that holds the longest
        row (qwen3_asr.py:366-372, 392-432, 508-515, 1108-1109)."""
        import torch.nn.functional as F

        h, kvh, d = self.heads, self.kv_heads, self.head_dim
        rows = torch.arange(self.batch, device=self.qkv.device)
        key_positions = torch.arange(self.cache_length, device=self.qkv.device)

        def rotate(x, cos, sin):
            first, second = x.chunk(2, dim=-1)
            return x * cos[:, None, :] + torch.cat((-second, first), dim=-1) * sin[:, None, :]

        def run(t):
            qkv_all, pos = self.inputs_at(t)
            bucket = kv_bucket(int(self.schedule[t].max()) + 1)
            cos, sin = self.cos[pos], self.sin[pos]
            mask = (key_positions[None, :bucket] <= pos[:, None])[:, None, None, :]
            for layer in range(self.layers):
                q, k, v = qkv_all[layer].split([h * d, kvh * d, kvh * d], dim=-1)
                q = rotate(F.rms_norm(q.reshape(-1, h, d), (d,), self.norms[layer, 0], 1e-6),
                           cos, sin)
                k = rotate(F.rms_norm(k.reshape(-1, kvh, d), (d,), self.norms[layer, 1], 1e-6),
                           cos, sin)
                keys = self.keys[layer][:, :bucket]
                values = self.values[layer][:, :bucket]
                keys[rows, pos] = k
                values[rows, pos] = v.reshape(-1, kvh, d)
                F.scaled_dot_product_attention(q.view(-1, kvh, h // kvh, d),
                                               keys.transpose(1, 2), values.transpose(1, 2),
                                               attn_mask=mask)
        return run

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The reference's ``TextAttention.step`` attention on the host
        (qwen3_asr.py:366-372, :392-432 with its torch 2.11 fallback): per
        layer, q/k RMSNorm and rotate-half RoPE, the cache write, SDPA of the
        grouped queries with the step mask over the bucket view; float32, a
        sample of the rows, every layer with its own cache."""
        torch = cpu_torch(threads)
        import torch.nn.functional as F

        rows, steps = 4, 128
        h, kvh, d = self.heads, self.kv_heads, self.head_dim
        gen = torch.Generator().manual_seed(SEED)
        keys = torch.randn((self.layers, rows, self.cache_length, kvh, d), generator=gen)
        values = torch.randn(keys.shape, generator=gen)
        qkv = torch.randn((self.layers, rows, (h + 2 * kvh) * d), generator=gen)
        weight = torch.ones(d)
        cos_t, sin_t = rope_tables(torch, 1e6, d, self.cache_length)
        index = torch.arange(rows)
        key_positions = torch.arange(self.cache_length)

        def rotate(x, cos, sin):
            first, second = x.chunk(2, dim=-1)
            return x * cos[:, None, :] + torch.cat((-second, first), dim=-1) * sin[:, None, :]

        def one(i):
            position = min(self.prompt + i % steps, self.cache_length - 1)
            pos = torch.full((rows,), position)
            bucket = kv_bucket(position + 1)
            cos, sin = cos_t[pos], sin_t[pos]
            mask = (key_positions[None, :bucket] <= pos[:, None])[:, None, None, :]
            for layer in range(self.layers):
                q, k, v = qkv[layer].split([h * d, kvh * d, kvh * d], dim=-1)
                q = rotate(F.rms_norm(q.reshape(rows, h, d), (d,), weight, 1e-6), cos, sin)
                k = rotate(F.rms_norm(k.reshape(rows, kvh, d), (d,), weight, 1e-6), cos, sin)
                kc, vc = keys[layer][:, :bucket], values[layer][:, :bucket]
                kc[index, pos] = k
                vc[index, pos] = v.reshape(rows, kvh, d)
                F.scaled_dot_product_attention(q.view(rows, kvh, h // kvh, d), kc.transpose(1, 2),
                                               vc.transpose(1, 2), attn_mask=mask)

        with torch.inference_mode():
            done, elapsed = time_cpu(one, budget_s)
        return {"value": rows * done / elapsed, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {self.batch} rows x {done} steps x {self.layers} layers "
                          f"(RMSNorm + RoPE + write + masked grouped SDPA over the bucket), "
                          f"torch CPU float32, {elapsed:.1f} s"}


class Qwen3Prefill(Workload):
    """Admission prefill of the Qwen3 decode workload's prompts: causal grouped-query
    attention within the packed prompts (TextAttention.prefill's `attend`)."""

    name = "qwen3-prefill"
    metric = ("prefill tokens/s/GPU (Qwen3 1.7B-style, 64 packed prompts x 410 tokens, 28 layers, "
              "bf16); attention TFLOP/s")
    unit = "tokens/s"
    bound = "tensor"
    default_batch = 64
    layers, heads, kv_heads, head_dim, prompt = 28, 16, 8, 128, 410
    causal = True
    profile = "qwen3_prefill_b64_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "Qwen3-ASR-1.7B-style packed prompt prefill attention (BASELINE config 4 "
                        "admission: 390 audio + 20 prompt positions per row)",
            "layers": self.layers, "heads": self.heads, "kv_heads": self.kv_heads,
            "head_dim": self.head_dim, "causal": True, "prompts_per_gpu": self.batch,
            "prompt_tokens": self.prompt, "global_batch": self.batch * world,
            "step": "28 layers of causal varlen attention over the packed prompts",
            "inputs": "N(0,1) bf16 q (tokens, 16, 128), k/v (tokens, 8, 128) per layer",
            "e2e": "layer 0's q/k/v in, the last layer's output out, per step",
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2 (215 MB of q/k/v per layer)",
        }

    def units_per_step(self) -> int:
        return self.batch * self.prompt

    def lengths(self) -> list[int]:
        return [self.prompt] * self.batch

    def window(self) -> int:
        return self.prompt

    def flops_per_layer(self) -> float:
        # Causal: query i reads i + 1 keys; 2 flops per multiply-add, QK and PV.
        pairs = sum(n * (n + 1) / 2 for n in self.lengths())
        return 4.0 * pairs * self.head_dim * self.heads

    def setup(self, torch, device, seed: int, steps: int) -> None:
        gen = torch.Generator(device=device).manual_seed(seed)
        tokens = sum(self.lengths())
        dtype = torch.bfloat16

        def rand(heads):
            return torch.randn((tokens, heads, self.head_dim), generator=gen, device=device,
                               dtype=dtype)

        self.qkv = [[rand(self.heads), rand(self.kv_heads), rand(self.kv_heads)]
                    for _ in range(self.layers)]
        lengths = torch.tensor(self.lengths())
        self.starts = torch.nn.functional.pad(lengths.cumsum(0), (1, 0)).to(torch.int32).to(device)
        self.inputs = list(self.qkv[0])

    def attend(self, layer, tensors=None):
        from asrback_b200 import attention

        q, k, v = tensors or self.qkv[layer]
        return attention.varlen_attention(q, k, v, self.starts, self.window(), self.causal)

    def launch(self, inputs) -> list:
        out = self.attend(0, inputs)
        for layer in range(1, self.layers):
            out = self.attend(layer)
        return [out]

    def launches_per_step(self) -> int:
        return self.layers

    def kernels(self, t: int):
        return [("varlen", lambda layer: self.attend(layer), self.flops_per_layer())]

    def step_work(self, first: int, count: int) -> float:
        return self.flops_per_layer() * self.layers * count

    def _padded(self, torch, starts, longest):
        """The reference's padded path indices (qwen3_asr.py:136-149)."""
        device = starts.device
        offsets = torch.arange(longest, device=device)
        sizes = starts[1:] - starts[:-1]
        valid = offsets[None, :] < sizes[:, None]
        last = (starts[1:] - 1)[:, None]
        gather = torch.minimum(starts[:-1, None] + offsets, last)
        mask = valid[:, None, None, :]
        if self.causal:
            mask = mask & torch.ones((longest, longest), dtype=torch.bool, device=device).tril()
        return gather, valid, mask

    def torch_reference_step(self, torch):
        """The reference's `attend` on its GPU path under torch 2.11 (varlen_attn
        lacks the kwargs it passes, so the padded batch): gather the segments,
        SDPA with the valid (and causal) mask and grouped heads, keep the valid
        rows (qwen3_asr.py:136-149, 166-181), on the same tensors."""
        import torch.nn.functional as F

        gather, valid, mask = self._padded(torch, self.starts, self.window())

        def run(_t):
            for layer in range(self.layers):
                out = F.scaled_dot_product_attention(
                    *(t[gather].transpose(1, 2) for t in self.qkv[layer]), attn_mask=mask,
                    enable_gqa=self.heads != self.kv_heads)
                out.transpose(1, 2)[valid]
        return run

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The reference's padded ``attend`` (qwen3_asr.py:152-181) on the host
        for one request's segments, float32."""
        torch = cpu_torch(threads)
        import torch.nn.functional as F

        per_request = len(self.lengths()) // self.batch
        lengths = self.lengths()[:per_request]
        tokens = sum(lengths)
        gen = torch.Generator().manual_seed(SEED)
        q = torch.randn((tokens, self.heads, self.head_dim), generator=gen)
        k = torch.randn((tokens, self.kv_heads, self.head_dim), generator=gen)
        v = torch.randn(k.shape, generator=gen)
        starts = F.pad(torch.tensor(lengths).cumsum(0), (1, 0))
        gather, valid, mask = self._padded(torch, starts, max(lengths))

        def one(_i):
            out = F.scaled_dot_product_attention(*(t[gather].transpose(1, 2) for t in (q, k, v)),
                                                 attn_mask=mask,
                                                 enable_gqa=self.heads != self.kv_heads)
            out.transpose(1, 2)[valid]

        with torch.inference_mode():
            done, elapsed = time_cpu(one, budget_s)
        rate = done / elapsed / self.layers * tokens
        return {"value": rate, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{done} request-layers ({per_request} segments, {tokens} tokens, "
                          f"padded SDPA), torch CPU float32, {elapsed:.1f} s, scaled by "
                          f"1/{self.layers} layers"}


class Qwen3AudioWindows(Qwen3Prefill):
    """Qwen3-ASR audio encoder attention: non-causal attention within 104-token
    windows of packed audio tokens (AudioAttention.forward's `attend`)."""

    name = "qwen3-audio"
    metric = ("audio tokens/s/GPU (Qwen3-ASR-style audio encoder attention, 64 x 30 s requests "
              "in 104-token windows, bf16); attention TFLOP/s")
    unit = "tokens/s"
    bound = "tensor"
    causal = False
    # 30 s of audio = 30 chunks of 13 tokens = 390 tokens per request: windows
    # of 104 tokens (8 chunks) and a last window of 78.
    layers, heads, kv_heads, head_dim, prompt = 24, 16, 16, 64, 390
    span = 104
    profile = "qwen3_audio_b64_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "Qwen3-ASR-style audio encoder window attention (admission of audio windows)",
            "layers": self.layers, "heads": self.heads, "head_dim": self.head_dim,
            "causal": False, "requests_per_gpu": self.batch, "tokens_per_request": self.prompt,
            "window_tokens": self.span, "global_batch": self.batch * world,
            "assumed": "24 layers, 16 heads of 64 (d_model 1024); the checkpoint's audio config "
                       "is not available here",
            "step": "24 layers of non-causal varlen attention over the packed windows",
            "inputs": "N(0,1) bf16 q/k/v (tokens, 16, 64) per layer",
            "parallelism": f"replicas x{world} (no collective)",
        }

    def lengths(self) -> list[int]:
        per = [self.span] * (self.prompt // self.span)
        if self.prompt % self.span:
            per.append(self.prompt % self.span)
        return per * self.batch

    def window(self) -> int:
        return self.span

    def flops_per_layer(self) -> float:
        return float(sum(4.0 * n * n * self.head_dim * self.heads for n in self.lengths()))


class WhisperCrossKV(Workload):
    """Admission of 32 encoded windows into the decoder:
    `set_encoder_output` (whisper.py:313-319), each of the 4 decoder
    layers' cross-attention keys/values projected from the encoder output and
    written into the cache."""

    name = "whisper-cross-kv"
    metric = ("cross-attention K/V fill windows/s/GPU (Whisper large-v3-turbo set_encoder_output: "
              "32 windows x 1500 frames, 4 decoder layers, bf16); projection TFLOP/s")
    unit = "windows/s"
    bound = "tensor"
    default_batch = 32
    layers, width, tokens, heads = 4, 1280, 1500, 20
    profile = "cross_kv_projection_b32_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "Whisper large-v3-turbo set_encoder_output: k_proj/v_proj of the encoder "
                        "output into the cross-attention cache (window admission)",
            "layers": self.layers, "width": self.width, "heads": self.heads,
            "frames": self.tokens, "windows_per_gpu": self.batch,
            "global_batch": self.batch * world,
            "step": "4 decoder layers' projections into the cache",
            "inputs": "encoder output N(0, 1) bf16, weights N(0, 1/width), v_proj bias N(0, 0.02)",
            "e2e": "the encoder output in; one cache row back as the completion read",
            "parallelism": f"replicas x{world} (no collective)",
        }

    def units_per_step(self) -> int:
        return self.batch

    def flops_per_layer(self) -> float:
        return 2.0 * self.batch * self.tokens * 2 * self.width * self.width

    def setup(self, torch, device, seed: int, steps: int) -> None:
        gen = torch.Generator(device=device).manual_seed(seed)
        w, dtype = self.width, torch.bfloat16
        self.x = torch.randn((self.batch, self.tokens, w), generator=gen, device=device).to(dtype)
        self.wk = [(torch.randn((w, w), generator=gen, device=device) / w ** 0.5).to(dtype)
                   for _ in range(self.layers)]
        self.wv = [(torch.randn((w, w), generator=gen, device=device) / w ** 0.5).to(dtype)
                   for _ in range(self.layers)]
        self.bv = [(torch.randn((w,), generator=gen, device=device) * 0.02).to(dtype)
                   for _ in range(self.layers)]
        shape = (self.layers, self.batch, self.heads, self.tokens, w // self.heads)
        self.keys = torch.zeros(shape, device=device, dtype=dtype)
        self.values = torch.zeros(shape, device=device, dtype=dtype)
        self.inputs = [self.x]

    def attend(self, layer: int, x=None) -> None:
        from asrback_b200 import attention

        attention.whisper_cross_kv_projection(self.x if x is None else x, self.wk[layer],
                                              self.wv[layer], self.bv[layer], self.keys[layer],
                                              self.values[layer])

    def launch(self, inputs) -> list:
        for layer in range(self.layers):
            self.attend(layer, inputs[0])
        return [self.keys[self.layers - 1, 0, 0, 0]]

    def launches_per_step(self) -> int:
        return self.layers

    def kernels(self, t: int):
        return [("cross_kv", self.attend, self.flops_per_layer())]

    def step_work(self, first: int, count: int) -> float:
        return self.flops_per_layer() * self.layers * count

    def torch_reference_step(self, torch):
        """The reference's set_encoder_output on the same tensors: per layer,
        project_key_value (two F.linear, _split_heads) and the copy into the
        cache rows (whisper.py:313-319, :85-91)."""
        import torch.nn.functional as F

        def split(t):
            b, s, w = t.shape
            return t.view(b, s, self.heads, w // self.heads).transpose(1, 2)

        def run(_t):
            for layer in range(self.layers):
                self.keys[layer, :self.batch] = split(F.linear(self.x, self.wk[layer]))
                self.values[layer, :self.batch] = split(
                    F.linear(self.x, self.wv[layer], self.bv[layer]))
        return run

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The reference's per-layer ``project_key_value`` and cache copy on
        the host for one window, float32."""
        torch = cpu_torch(threads)
        import torch.nn.functional as F

        w = self.width
        gen = torch.Generator().manual_seed(SEED)
        x = torch.randn((1, self.tokens, w), generator=gen)
        wk = torch.randn((w, w), generator=gen) / w ** 0.5
        wv = torch.randn((w, w), generator=gen) / w ** 0.5
        bv = torch.randn((w,), generator=gen) * 0.02
        keys = torch.zeros((1, self.heads, self.tokens, w // self.heads))
        values = torch.zeros_like(keys)

        def split(t):
            return t.view(1, self.tokens, self.heads, w // self.heads).transpose(1, 2)

        def one(_i):
            keys[:] = split(F.linear(x, wk))
            values[:] = split(F.linear(x, wv, bv))

        with torch.inference_mode():
            done, elapsed = time_cpu(one, budget_s)
        return {"value": done / elapsed / self.layers, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{done} window-layers (1500 x 1280 @ 1280 x 2560 + cache copy), torch "
                          f"CPU float32, {elapsed:.1f} s, scaled by 1/4 layers"}


class WhisperPrefix(Workload):
    """The prompt pass of 32 windows at admission:
    `decode(tokens, positions[:P], cache, length=P)`
    (whisper.py:847-849) for 32 windows sharing the 4-token start sequence
    (windows queued together share a prefix length), the attention of its 4
    decoder layers: causal self-attention over the P written keys
    (whisper.py:228-236) and cross-attention of every prompt token over the
    window's 1500 encoder keys (:239-240)."""

    name = "whisper-prefix"
    metric = ("prompt-pass attention windows/s/GPU (Whisper large-v3-turbo decoder, 32 windows x "
              "4 prompt tokens, self + cross over 1500 frames, 4 layers, bf16); cross-attention "
              "GB/s")
    unit = "windows/s"
    bound = "hbm"
    default_batch = 32
    layers, heads, dim, frames, bucket = 4, 20, 64, 1500, 448
    tokens = 4
    profile = "whisper_prefix_b32_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "Whisper large-v3-turbo prompt pass attention (decode with length=P, "
                        "window admission)",
            "layers": self.layers, "heads": self.heads, "head_dim": self.dim,
            "prompt_tokens": self.tokens, "frames": self.frames,
            "windows_per_gpu": self.batch, "global_batch": self.batch * world,
            "step": "per layer: causal self-attention of P tokens + cross-attention of P tokens",
            "inputs": "queries and caches N(0, 1) bf16; cross caches 4 x 246 MB (> L2)",
            "parallelism": f"replicas x{world} (no collective)",
        }

    def units_per_step(self) -> int:
        return self.batch

    def cross_bytes(self) -> float:
        kv = 2.0 * self.batch * self.heads * self.frames * self.dim * 2
        rows = 2.0 * self.batch * self.tokens * self.heads * self.dim * 2
        return kv + rows

    def self_bytes(self) -> float:
        return 4.0 * self.batch * self.tokens * self.heads * self.dim * 2

    def setup(self, torch, device, seed: int, steps: int) -> None:
        gen = torch.Generator(device=device).manual_seed(seed)
        dtype, b, h, p, d = torch.bfloat16, self.batch, self.heads, self.tokens, self.dim

        def rand(*shape):
            return torch.randn(shape, generator=gen, device=device).to(dtype)

        self.self_q = rand(b, p, h * d)
        self.cross_q = rand(b, p, h * d)
        self.self_k = rand(self.layers, b, h, self.bucket, d)
        self.self_v = rand(self.layers, b, h, self.bucket, d)
        self.cross_k = rand(self.layers, b, h, self.frames, d)
        self.cross_v = rand(self.layers, b, h, self.frames, d)
        self.inputs = [self.self_q, self.cross_q]

    def _query(self, x):
        b, p, _ = x.shape
        return x.view(b, p, self.heads, self.dim).transpose(1, 2)

    def attend_self(self, layer: int, q=None):
        from asrback_b200 import attention

        layer %= self.layers
        p = self.tokens
        return attention.whisper_self_attention_prefix(
            self._query(self.self_q if q is None else q), self.self_k[layer][:, :, :p],
            self.self_v[layer][:, :, :p])

    def attend_cross(self, layer: int, q=None):
        from asrback_b200 import attention

        layer %= self.layers
        return attention.whisper_cross_attention_prefix(
            self._query(self.cross_q if q is None else q), self.cross_k[layer],
            self.cross_v[layer])

    def launch(self, inputs) -> list:
        outputs = []
        for layer in range(self.layers):
            outputs.append(self.attend_self(layer, inputs[0]))
            outputs.append(self.attend_cross(layer, inputs[1]))
        return outputs

    def launches_per_step(self) -> int:
        return 2 * self.layers

    def kernels(self, t: int):
        return [("cross_prefix", self.attend_cross, self.cross_bytes()),
                ("self_prefix", self.attend_self, self.self_bytes())]

    def step_work(self, first: int, count: int) -> float:
        return (self.cross_bytes() + self.self_bytes()) * self.layers * count

    def torch_reference_step(self, torch):
        """The reference's eager branch calls on the same tensors:
        `attend`'s SDPA with is_causal over the first P cache positions, then
        SDPA over the cross cache (whisper.py:233-240, :102-104)."""
        import torch.nn.functional as F

        p = self.tokens

        def run(_t):
            for layer in range(self.layers):
                F.scaled_dot_product_attention(
                    self._query(self.self_q), self.self_k[layer][:, :, :p],
                    self.self_v[layer][:, :, :p], is_causal=p > 1)
                F.scaled_dot_product_attention(
                    self._query(self.cross_q), self.cross_k[layer], self.cross_v[layer])
        return run

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The same two SDPA calls per layer on the host for one window, float32."""
        torch = cpu_torch(threads)
        import torch.nn.functional as F

        h, p, d = self.heads, self.tokens, self.dim
        gen = torch.Generator().manual_seed(SEED)
        q = torch.randn((1, h, p, d), generator=gen)
        k = torch.randn((1, h, p, d), generator=gen)
        ck = torch.randn((1, h, self.frames, d), generator=gen)
        cv = torch.randn(ck.shape, generator=gen)

        def one(_i):
            F.scaled_dot_product_attention(q, k, k, is_causal=p > 1)
            F.scaled_dot_product_attention(q, ck, cv)

        with torch.inference_mode():
            done, elapsed = time_cpu(one, budget_s, limit=1 << 16)
        return {"value": done / elapsed / self.layers, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{done} window-layers (20 heads, {p} prompt tokens, self + cross over "
                          f"1500 frames), torch CPU SDPA float32, {elapsed:.1f} s, scaled by 1/4 "
                          f"layers"}


class WhisperGreedyStep(Workload):
    """The step epilogue after the decoder: logits against
    the tied embedding, greedy `_choose` with the suppress mask and the state
    update (whisper.py:949-975), Whisper large-v3-turbo widths, 64 rows."""

    name = "whisper-step"
    family = "whisper"
    metric = ("greedy step epilogue tokens/s/GPU (Whisper large-v3-turbo: logits 51866 x 1280 + "
              "argmax/log-softmax + state update, 64 rows, bf16); weight-read GB/s")
    unit = "tokens/s"
    bound = "hbm"
    reference_in_graph = True
    default_batch = 64
    vocab, width, length, eos = 51866, 1280, 448, (50257,)
    copies = 4  # weight copies, rotated so that no launch finds its weights in L2
    profile = "greedy_step_whisper_b64_bf16.md"

    def __init__(self, batch: int | None):
        super().__init__(batch)
        self.layers = self.copies

    def config(self, world: int) -> dict:
        return {
            "workload": f"{self.family} greedy step epilogue (logits GEMM + _choose + state "
                        "update after the decoder)",
            "vocab": self.vocab, "hidden": self.width, "rows_per_gpu": self.batch,
            "global_batch": self.batch * world, "suppress": self.family == "whisper",
            "eos_ids": list(self.eos), "steps_per_replay": self.copies,
            "step": f"{self.copies} greedy steps, each over its own weight copy",
            "inputs": "weight N(0, 0.02) bf16, hidden N(0, 1) bf16",
            "parallelism": f"replicas x{world} (no collective)",
            "l2": f"{self.copies} weight copies of {self.weight_bytes() / 1e6:.0f} MB rotate "
                  "(larger than L2)",
        }

    def weight_bytes(self) -> int:
        return self.vocab * self.width * 2

    def bytes_per_launch(self) -> float:
        # The weight once, the hidden rows, the suppress flags, the state.
        return float(self.weight_bytes() + self.batch * self.width * 2
                     + (self.vocab if self.family == "whisper" else 0) + self.batch * 40)

    def units_per_step(self) -> int:
        return self.batch * self.copies

    def setup(self, torch, device, seed: int, steps: int) -> None:
        gen = torch.Generator(device=device).manual_seed(seed)
        self.weights = [(torch.randn((self.vocab, self.width), generator=gen, device=device)
                         * 0.02).to(torch.bfloat16) for _ in range(self.copies)]
        self.hidden = [torch.randn((self.batch, self.width), generator=gen, device=device)
                       .to(torch.bfloat16) for _ in range(self.copies)]
        self.suppress = None
        if self.family == "whisper":
            self.suppress = torch.zeros(self.vocab, dtype=torch.bool, device=device)
            self.suppress[50364:] = True  # timestamp tokens
        b = self.batch
        self.tokens = torch.zeros(b, dtype=torch.int64, device=device)
        self.position = torch.randint(0, 100, (b,), generator=gen, device=device)
        self.end = torch.full((b,), self.length - 1, dtype=torch.int64, device=device)
        self.finished = torch.zeros(b, dtype=torch.bool, device=device)
        self.sum_logprobs = torch.zeros(b, device=device)
        self.generated = torch.zeros((b, self.length), dtype=torch.int64, device=device)
        self.inputs = list(self.hidden)

    def attend(self, i: int, hidden=None) -> None:
        from asrback_b200 import step

        step.greedy_step(self.hidden[i] if hidden is None else hidden, self.weights[i],
                         self.tokens, self.position, self.end, self.finished, self.sum_logprobs,
                         self.generated, self.eos, self.suppress)

    def launch(self, inputs) -> list:
        for i in range(self.copies):
            self.attend(i, inputs[i])
        return [self.tokens]

    def launches_per_step(self) -> int:
        return self.copies

    def kernels(self, t: int):
        return [("greedy_step", self.attend, self.bytes_per_launch())]

    def step_work(self, first: int, count: int) -> float:
        return self.bytes_per_launch() * self.copies * count

    def torch_reference_step(self, torch):
        """The reference's `_step` after `decode` on its GPU path (graph-captured
        by the reference): logits, `_choose` without sampling, the state update
        (whisper.py:949-975 / qwen3_asr.py:1189-1213), on the same tensors."""
        import torch.nn.functional as F

        eos = torch.tensor(self.eos, device=self.tokens.device)
        tokens = self.tokens.clone()
        position, finished = self.position.clone(), self.finished.clone()
        sums, generated = self.sum_logprobs.clone(), self.generated.clone()

        def run(_t):
            for i in range(self.copies):
                logits = (self.weights[i] @ self.hidden[i].T).T.float()
                if self.suppress is not None:
                    logits.masked_fill_(self.suppress, -float("inf"))
                token = logits.argmax(dim=-1)
                logprob = F.log_softmax(logits, dim=-1).gather(1, token[:, None]).squeeze(1)
                active = ~finished
                pos = position + active
                token = torch.where(active, token, tokens)
                sums.add_(logprob.masked_fill(finished, 0.0))
                generated.scatter_(1, pos[:, None], token[:, None])
                finished.logical_or_(torch.isin(token, eos) | (pos >= self.end))
                position.copy_(pos)
                tokens.copy_(token)
        return run

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The reference's `_step` after `decode` on the host: the logits
        matmul, `_choose` (suppress, argmax, log-softmax) and the state update
        for the 64 rows, float32."""
        torch = cpu_torch(threads)
        import torch.nn.functional as F

        gen = torch.Generator().manual_seed(SEED)
        weight = torch.randn((self.vocab, self.width), generator=gen) * 0.02
        hidden = torch.randn((self.batch, self.width), generator=gen)
        suppress = None
        if self.family == "whisper":
            suppress = torch.zeros(self.vocab, dtype=torch.bool)
            suppress[50364:] = True
        eos = torch.tensor(self.eos)
        tokens = torch.zeros(self.batch, dtype=torch.int64)
        position = torch.zeros(self.batch, dtype=torch.int64)
        finished = torch.zeros(self.batch, dtype=torch.bool)
        sums = torch.zeros(self.batch)
        generated = torch.zeros((self.batch, self.length), dtype=torch.int64)
        end = torch.full((self.batch,), self.length - 1)

        def one(_i):
            logits = (weight @ hidden.T).T
            if suppress is not None:
                logits.masked_fill_(suppress, -float("inf"))
            token = logits.argmax(dim=-1)
            logprob = F.log_softmax(logits, dim=-1).gather(1, token[:, None]).squeeze(1)
            active = ~finished
            pos = torch.minimum(position + active, end)
            sums.add_(logprob.masked_fill(finished, 0.0))
            generated.scatter_(1, pos[:, None], token[:, None])
            finished.logical_or_(torch.isin(token, eos))
            position.copy_(pos)
            tokens.copy_(token)

        with torch.inference_mode():
            done, elapsed = time_cpu(one, budget_s)
        return {"value": self.batch * done / elapsed, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{done} steps of {self.batch} rows (logits {self.vocab} x {self.width} "
                          f"+ _choose + state update), torch CPU float32, {elapsed:.1f} s"}


class Qwen3GreedyStep(WhisperGreedyStep):
    """The Qwen3-ASR-1.7B step epilogue: `lm_head` (151936 x 2048), `_choose`,
    the state update with two EOS ids (qwen3_asr.py:1189-1213), 64 rows."""

    name = "qwen3-step"
    family = "qwen3"
    metric = ("greedy step epilogue tokens/s/GPU (Qwen3-ASR-1.7B-style: lm_head 151936 x 2048 + "
              "argmax/log-softmax + state update, 64 rows, bf16); weight-read GB/s")
    vocab, width, length, eos = 151936, 2048, 1024, (151643, 151645)
    copies = 2
    profile = "greedy_step_qwen3_b64_bf16.md"


class _Request:
    """One synthetic request of the serving trace."""

    __slots__ = ("index", "arrival", "seconds", "audio", "length", "replica", "done_at")

    def __init__(self, index: int, arrival: float, seconds: float, audio: int, text: int):
        self.index, self.arrival, self.seconds = index, arrival, seconds
        self.audio = audio
        self.length = audio + text
        self.replica = 0
        self.done_at = None


class Qwen3Serve:
    """continuous-batching serving, one replica per GPU.

    Each GPU holds a Qwen3-ASR-0.6B-style text model (28 layers, hidden 1024,
    16 query / 8 key-value heads of 128, MLP 3072, vocabulary 151936 tied to
    the embedding; seeded weights, seed 4) and the reference engine's
    scheduling (qwen3_asr.py:950-982, :1018-1151): a pool of 64 rows over a
    ``(28, 64, 1024, 8, 128)`` cache; requests that find a free row join with
    one packed causal prefill of their prompts (audio positions injected as
    N(0, 0.02) embeddings -- the audio front end and tower are not on this
    path -- plus 20 text positions); the rows decode together, one CUDA graph
    per batch bucket (1, 2, ..., 64: the highest occupied row decides), four
    steps between host checks for finished rows, which then leave; each request
    generates 128 tokens.

    Requests come from one seeded trace: Poisson arrivals at 25 requests/s per
    GPU (200/s over 8 GPUs), 16 kHz audio of U[1, 30] s, 13 audio positions per
    second (``architecture.md:471``), so a prompt holds 33 to 410 positions.
    ``ReplicaDispatcher`` assigns each request to the replica with the fewest
    outstanding requests (each holds one row for its 128 steps); every rank
    builds the same trace and serves its own share.

    Two runs: ``capacity`` queues every request of the replica's share at
    once (the engine's throughput under join/leave churn, the line's value),
    and ``paced`` releases them at their arrival times (tokens/s at the offered
    load, and per-request latency)."""

    name = "qwen3-serve"
    metric = ("whole-box generated tokens/s (Qwen3-ASR-0.6B-style LM, continuous batching, "
              "max batch 64, Poisson arrivals 200 req/s over 8 GPUs, 128 new tokens)")
    unit = "tokens/s"
    bound = "hbm"
    hidden, layers, heads, kv_heads, head_dim, inter, vocab = 1024, 28, 16, 8, 128, 3072, 151936
    cache_length, max_new, interval, eps = 1024, 128, 4, 1e-6
    rate_per_gpu, audio_rate, text_tokens = 25.0, 13, 20
    eos = (151643, 151645)

    def __init__(self, batch: int | None):
        self.max_batch = batch or 64
        self.buckets = sorted({min(2 ** i, self.max_batch)
                               for i in range(self.max_batch.bit_length())} | {self.max_batch})

    def config(self, world: int) -> dict:
        return {
            "workload": "Qwen3-ASR-0.6B-style continuous-batching serving (BASELINE config 5)",
            "layers": self.layers, "hidden": self.hidden, "heads": self.heads,
            "kv_heads": self.kv_heads, "head_dim": self.head_dim, "intermediate": self.inter,
            "vocab": self.vocab, "seed": 4, "max_batch": self.max_batch,
            "max_new_tokens": self.max_new,
            "arrivals": f"Poisson, {self.rate_per_gpu * world:g} req/s over {world} GPUs "
                        f"({self.rate_per_gpu:g} per GPU; 200/s at 8)",
            "audio": "U[1,30] s per request, 13 audio positions per second, injected as "
                     "N(0, 0.02) embeddings, plus 20 text positions",
            "engine": "pool of rows over a (28, 64, 1024, 8, 128) cache; packed causal prefill on "
                      "join; one CUDA graph per batch bucket; finished rows checked every 4 steps",
            "parallelism": f"replicas x{world} (no collective), least-loaded dispatch",
        }

    def units_per_step(self) -> int:
        """Tokens of one decode step of a full pool."""
        return self.max_batch

    # ---- the trace ----
    def trace(self, world: int, count: int) -> list:
        from asrback_b200.replicas import ReplicaDispatcher

        rng = np.random.default_rng(4)
        rate = self.rate_per_gpu * world
        arrivals = np.cumsum(rng.exponential(1.0 / rate, size=count))
        seconds = rng.uniform(1.0, 30.0, size=count)
        requests = []
        for i in range(count):
            audio = int(math.ceil(seconds[i] * self.audio_rate))
            requests.append(_Request(i, float(arrivals[i]), float(seconds[i]), audio,
                                     self.text_tokens))
        # Every request costs one row of the pool for its 128 steps whatever
        # its prompt, so the dispatcher balances rows (least outstanding
        # requests; in arrival order this deals them out in turn).
        dispatcher = ReplicaDispatcher(world)
        for request in requests:
            request.replica = dispatcher.assign(1.0)
        return requests

    # ---- the engine ----
    def setup(self, torch, device, seed: int, native: bool = True) -> None:
        dtype = torch.bfloat16
        self.torch, self.device, self.native = torch, device, native
        gen = torch.Generator(device=device).manual_seed(4)
        h, L = self.hidden, self.layers
        q, kv, d = self.heads, self.kv_heads, self.head_dim

        def weight(rows, cols):
            return (torch.randn((rows, cols), generator=gen, device=device)
                    / math.sqrt(cols)).to(dtype)

        def norm(*shape):
            return (1 + 0.1 * torch.randn(shape, generator=gen, device=device)).to(dtype)

        self.embed = (torch.randn((self.vocab, h), generator=gen, device=device) * 0.02).to(dtype)
        self.w_qkv = [weight((q + 2 * kv) * d, h) for _ in range(L)]
        self.w_o = [weight(h, q * d) for _ in range(L)]
        self.w_gate_up = [weight(2 * self.inter, h) for _ in range(L)]
        self.w_down = [weight(h, self.inter) for _ in range(L)]
        self.n_in, self.n_post, self.n_q, self.n_k = (norm(L, h), norm(L, h), norm(L, d),
                                                      norm(L, d))
        self.n_final = norm(h)
        shape = (L, self.max_batch, self.cache_length, kv, d)
        self.keys = torch.zeros(shape, dtype=dtype, device=device)
        self.values = torch.zeros(shape, dtype=dtype, device=device)
        self.cos, self.sin = rope_tables(torch, 1e6, d, self.cache_length, device, dtype)
        b = self.max_batch
        self.tokens = torch.zeros(b, dtype=torch.int64, device=device)
        self.position = torch.zeros(b, dtype=torch.int64, device=device)
        self.end = torch.zeros(b, dtype=torch.int64, device=device)
        self.finished = torch.ones(b, dtype=torch.bool, device=device)
        self.sum_logprobs = torch.zeros(b, device=device)
        self.generated = torch.zeros((b, self.cache_length), dtype=torch.int64, device=device)
        self.eos_t = torch.tensor(self.eos, device=device)
        self.audio_gen = torch.Generator(device=device).manual_seed(seed)
        self.graphs = {}

    def _rotate(self, x, cos, sin):
        first, second = x.chunk(2, dim=-1)
        return x * cos[:, None, :] + self.torch.cat((-second, first), dim=-1) * sin[:, None, :]

    def _mlp(self, layer, x):
        F = self.torch.nn.functional
        h = F.rms_norm(x, (self.hidden,), self.n_post[layer], self.eps)
        gate, up = (h @ self.w_gate_up[layer].T).chunk(2, dim=-1)
        return x + (F.silu(gate) * up) @ self.w_down[layer].T

    def _decode(self, b: int, kv_len: int | None) -> None:
        """One decode step of rows 0..b-1 (the graph body)."""
        torch = self.torch
        F = torch.nn.functional
        from asrback_b200 import attention, step

        q, kvh, d = self.heads, self.kv_heads, self.head_dim
        tokens, position = self.tokens[:b], self.position[:b]
        x = self.embed[tokens]
        if not self.native:
            rows = torch.arange(b, device=self.device)
            cos, sin = self.cos[position], self.sin[position]
            key_positions = torch.arange(kv_len, device=self.device)
            mask = (key_positions[None, :] <= position[:, None])[:, None, None, :]
        for layer in range(self.layers):
            h = F.rms_norm(x, (self.hidden,), self.n_in[layer], self.eps)
            qkv = h @ self.w_qkv[layer].T
            keys, values = self.keys[layer][:b], self.values[layer][:b]
            if self.native:
                out = attention.qwen3_attention_step(
                    qkv, self.n_q[layer], self.n_k[layer], self.eps, self.cos, self.sin,
                    position, keys, values, q, kvh)
            else:
                # The reference's TextAttention.step on its torch 2.11 path.
                qq, kk, vv = qkv.split([q * d, kvh * d, kvh * d], dim=-1)
                qq = self._rotate(F.rms_norm(qq.reshape(b, q, d), (d,), self.n_q[layer], self.eps),
                                  cos, sin)
                kk = self._rotate(F.rms_norm(kk.reshape(b, kvh, d), (d,), self.n_k[layer],
                                             self.eps), cos, sin)
                keys, values = keys[:, :kv_len], values[:, :kv_len]
                keys[rows, position] = kk
                values[rows, position] = vv.reshape(b, kvh, d)
                out = F.scaled_dot_product_attention(
                    qq.view(b, kvh, q // kvh, d), keys.transpose(1, 2), values.transpose(1, 2),
                    attn_mask=mask).reshape(b, q * d)
            x = self._mlp(layer, x + out @ self.w_o[layer].T)
        x = F.rms_norm(x, (self.hidden,), self.n_final, self.eps)
        if self.native:
            step.greedy_step(x, self.embed, tokens, position, self.end[:b], self.finished[:b],
                             self.sum_logprobs[:b], self.generated[:b], self.eos)
        else:
            logits = (x @ self.embed.T).float()
            token = logits.argmax(dim=-1)
            logprob = F.log_softmax(logits, dim=-1).gather(1, token[:, None]).squeeze(1)
            finished = self.finished[:b]
            active = ~finished
            pos = position + active
            token = torch.where(active, token, tokens)
            self.sum_logprobs[:b].add_(logprob.masked_fill(finished, 0.0))
            self.generated[:b].scatter_(1, pos[:, None], token[:, None])
            finished.logical_or_(torch.isin(token, self.eos_t) | (pos >= self.end[:b]))
            position.copy_(pos)
            tokens.copy_(token)

    def capture(self) -> None:
        """One graph per batch bucket (per key/value bucket too on the torch
        path, which reads the whole bucket view), captured before serving."""
        from asrback_b200.transcription import CapturedGraph

        pool = self.torch.cuda.graph_pool_handle()
        kv_buckets = (None,) if self.native else (128, 256, 512, 768, 1024)
        for b in self.buckets:
            for kv_len in kv_buckets:
                self.finished.zero_()
                self.position.zero_()
                self.end.fill_(self.cache_length - 1)
                self.graphs[b, kv_len] = CapturedGraph(
                    lambda b=b, kv_len=kv_len: self._decode(b, kv_len), pool)
        self.finished.fill_(True)
        self.position.zero_()
        self.tokens.zero_()

    def _prefill(self, requests: list, slots: list[int]) -> None:
        """Packed causal prefill of the joining requests into their rows, and
        their first tokens (qwen3_asr.py:1018-1091)."""
        torch = self.torch
        F = torch.nn.functional
        from asrback_b200 import attention, step

        q, kvh, d = self.heads, self.kv_heads, self.head_dim
        lengths = [r.length for r in requests]
        total = sum(lengths)
        ids = np.empty(total, np.int64)
        audio_rows = []
        offset = 0
        for r in requests:
            # <system + user> text, the audio positions, <assistant> text.
            head = self.text_tokens // 2
            ids[offset:offset + r.length] = (np.arange(r.length) * 7919 + r.index * 104729) \
                % 150000
            audio_rows.append(np.arange(offset + head, offset + head + r.audio))
            offset += r.length
        positions = np.concatenate([np.arange(n) for n in lengths])
        rows = np.repeat(np.asarray(slots), lengths)
        starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
        first = np.asarray(lengths, np.int64)
        ends = first - 1 + np.minimum(self.max_new, self.cache_length - first)
        host = [torch.from_numpy(a).pin_memory() for a in
                (ids, positions, rows, starts, np.concatenate(audio_rows), np.asarray(slots),
                 first, ends)]
        ids, positions, rows, starts, audio, slot_rows, first, ends = (
            t.to(self.device, non_blocking=True) for t in host)
        x = self.embed[ids]
        x[audio] = (torch.randn((audio.shape[0], self.hidden), generator=self.audio_gen,
                                device=self.device) * 0.02).to(x.dtype)
        cos, sin = self.cos[positions], self.sin[positions]
        longest = max(lengths)
        if not self.native:
            sizes = starts[1:] - starts[:-1]
            offsets = torch.arange(longest, device=self.device)
            valid = offsets[None, :] < sizes[:, None]
            gather = torch.minimum(starts[:-1, None] + offsets, (starts[1:] - 1)[:, None])
            mask = valid[:, None, None, :] & torch.ones((longest, longest), dtype=torch.bool,
                                                        device=self.device).tril()
        for layer in range(self.layers):
            h = F.rms_norm(x, (self.hidden,), self.n_in[layer], self.eps)
            qq, kk, vv = (h @ self.w_qkv[layer].T).split([q * d, kvh * d, kvh * d], dim=-1)
            qq = self._rotate(F.rms_norm(qq.reshape(total, q, d), (d,), self.n_q[layer],
                                         self.eps), cos, sin)
            kk = self._rotate(F.rms_norm(kk.reshape(total, kvh, d), (d,), self.n_k[layer],
                                         self.eps), cos, sin)
            vv = vv.reshape(total, kvh, d)
            self.keys[layer][rows, positions] = kk
            self.values[layer][rows, positions] = vv
            if self.native:
                out = attention.varlen_attention(qq, kk, vv, starts, longest, True)
            else:
                out = F.scaled_dot_product_attention(
                    *(t[gather].transpose(1, 2) for t in (qq, kk, vv)), attn_mask=mask,
                    enable_gqa=True).transpose(1, 2)[valid]
            x = self._mlp(layer, x + out.reshape(total, q * d) @ self.w_o[layer].T)
        last = F.rms_norm(x[starts[1:].long() - 1], (self.hidden,), self.n_final, self.eps)
        if self.native:
            token, logprob = step.greedy_choose(last, self.embed)
        else:
            logits = (last @ self.embed.T).float()
            token = logits.argmax(dim=-1)
            logprob = F.log_softmax(logits, dim=-1).gather(1, token[:, None]).squeeze(1)
        self.tokens[slot_rows] = token
        self.position[slot_rows] = first
        self.end[slot_rows] = ends
        self.finished[slot_rows] = torch.isin(token, self.eos_t) | (first >= ends)
        self.sum_logprobs[slot_rows] = logprob
        self.generated[slot_rows, first] = token

    def serve(self, requests: list, paced: bool) -> dict:
        """Serves ``requests`` (sorted by arrival) to the end; returns counts
        and device/host times."""
        torch = self.torch
        import collections

        pending = collections.deque()
        queue = collections.deque(requests)
        rows: dict[int, _Request] = {}
        bounds: dict[int, int] = {}
        generated = steps = prefills = 0
        stream = torch.cuda.current_stream()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        start.record(stream)
        while queue or pending or rows:
            now = time.perf_counter() - t0
            while queue and (not paced or queue[0].arrival <= now):
                pending.append(queue.popleft())
            free = [slot for slot in range(self.max_batch) if slot not in rows]
            if pending and free:
                joining = [pending.popleft() for _ in range(min(len(free), len(pending)))]
                slots = free[:len(joining)]
                self._prefill(joining, slots)
                prefills += 1
                for slot, r in zip(slots, joining):
                    rows[slot] = r
                    bounds[slot] = r.length
            if not rows:
                if queue:
                    time.sleep(max(0.0, min(queue[0].arrival - now, 0.002)))
                continue
            bucket = next(size for size in self.buckets if size > max(rows))
            count = min(self.interval,
                        max(r.length - 1 + self.max_new - bounds[s] for s, r in rows.items()))
            count = max(count, 1)
            kv_len = None
            if not self.native:
                length = max(min(bounds[s] + count, rows[s].length - 1 + self.max_new)
                             for s in rows) + 1
                kv_len = kv_bucket(length)
            graph = self.graphs[bucket, kv_len]
            for _ in range(count):
                graph.replay()
            steps += count
            for slot in rows:
                bounds[slot] = min(bounds[slot] + count, rows[slot].length - 1 + self.max_new)
            finished = self.finished[:max(rows) + 1].tolist()
            done = [slot for slot in rows if finished[slot]]
            if done:
                index = torch.tensor(done, device=self.device)
                last = self.position[index].tolist()
                now = time.perf_counter() - t0
                for slot, position in zip(done, last):
                    r = rows.pop(slot)
                    generated += position - r.length + 1
                    r.done_at = now
                self.finished[index] = True
                self.position[index] = 0
                self.tokens[index] = 0
        end.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        return {"tokens": generated, "requests": len(requests), "device_ms": start.elapsed_time(end),
                "wall_s": wall, "decode_steps": steps, "prefills": prefills}

    def cpu_rate(self, budget_s: float, threads: int) -> dict:
        """The reference's decode step of this model on the host (float32):
        embedding, 28 layers of RMSNorm, qkv, q/k RMSNorm + RoPE, cache write,
        masked grouped SDPA over the 512-position bucket, o_proj and the MLP,
        then the logits and ``_choose`` for 64 rows at positions 400..."""
        torch = cpu_torch(threads)
        F = torch.nn.functional
        gen = torch.Generator().manual_seed(4)
        h, L, q, kvh, d, b = self.hidden, self.layers, self.heads, self.kv_heads, self.head_dim, 64
        w_qkv = [torch.randn(((q + 2 * kvh) * d, h), generator=gen) / 32 for _ in range(L)]
        w_o = [torch.randn((h, q * d), generator=gen) / 45 for _ in range(L)]
        w_gu = [torch.randn((2 * self.inter, h), generator=gen) / 32 for _ in range(L)]
        w_d = [torch.randn((h, self.inter), generator=gen) / 55 for _ in range(L)]
        embed = torch.randn((self.vocab, h), generator=gen) * 0.02
        keys = torch.randn((L, b, 512, kvh, d), generator=gen)
        values = torch.randn(keys.shape, generator=gen)
        ones_h, ones_d = torch.ones(h), torch.ones(d)
        cos_t, sin_t = rope_tables(torch, 1e6, d, self.cache_length)
        rows = torch.arange(b)
        key_positions = torch.arange(512)

        def one(i):
            pos = torch.full((b,), 400 + i % 100)
            cos, sin = cos_t[pos], sin_t[pos]
            mask = (key_positions[None, :] <= pos[:, None])[:, None, None, :]
            x = embed[torch.arange(b)]
            for layer in range(L):
                hh = F.rms_norm(x, (h,), ones_h, 1e-6)
                qq, kk, vv = (hh @ w_qkv[layer].T).split([q * d, kvh * d, kvh * d], dim=-1)
                qq = self._rotate(F.rms_norm(qq.reshape(b, q, d), (d,), ones_d, 1e-6), cos, sin)
                kk = self._rotate(F.rms_norm(kk.reshape(b, kvh, d), (d,), ones_d, 1e-6), cos, sin)
                keys[layer][rows, pos] = kk
                values[layer][rows, pos] = vv.reshape(b, kvh, d)
                out = F.scaled_dot_product_attention(
                    qq.view(b, kvh, q // kvh, d), keys[layer].transpose(1, 2),
                    values[layer].transpose(1, 2), attn_mask=mask).reshape(b, q * d)
                x = x + out @ w_o[layer].T
                hh = F.rms_norm(x, (h,), ones_h, 1e-6)
                gate, up = (hh @ w_gu[layer].T).chunk(2, dim=-1)
                x = x + (F.silu(gate) * up) @ w_d[layer].T
            logits = F.rms_norm(x, (h,), ones_h, 1e-6) @ embed.T
            token = logits.argmax(dim=-1)
            F.log_softmax(logits, dim=-1).gather(1, token[:, None])

        self.torch = torch
        with torch.inference_mode():
            done, elapsed = time_cpu(one, budget_s)
        return {"value": b * done / elapsed, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{done} decode steps of 64 rows through the 28-layer model (no churn), "
                          f"torch CPU float32, {elapsed:.1f} s"}


def measure_serve(args, work, torch, dist, device, rank: int, world: int, requests_per_gpu: int,
                  cpu: bool, paced: bool) -> dict:
    """The serving workload: capacity (every request of this replica's share
    queued at once), then the same engine on the reference's torch attention
    path, then (optionally) the arrival-paced run; the slowest rank's time."""
    trace = work.trace(world, requests_per_gpu * world)
    mine = [r for r in trace if r.replica == rank]
    total_tokens = len(trace) * work.max_new
    results = {}
    with torch.inference_mode():
        for native in (True, False):
            work.setup(torch, device, SEED + 1000 * rank, native=native)
            work.capture()
            warm = work.trace(1, 8)  # a short warm-up through every code path
            work.serve(warm, paced=False)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            uuid = getattr(torch.cuda.get_device_properties(device), "uuid", None)
            with ClockSampler(str(uuid) if uuid else None) as clocks:
                run = work.serve(mine, paced=False)
            ranks = rank_times(torch, dist, world, run["device_ms"])
            tokens = rank_times(torch, dist, world, float(run["tokens"]))
            results["native" if native else "torch"] = dict(
                run, rank_ms=ranks, value=sum(tokens) / (max(ranks) / 1e3),
                clocks=clocks.summary())
            if native and paced:
                for r in mine:
                    r.done_at = None
                work.serve(work.trace(1, 4), paced=False)
                if world > 1:
                    dist.barrier()
                paced_run = work.serve(mine, paced=True)
                latency = sorted(r.done_at - r.arrival for r in mine if r.done_at is not None)
                walls = rank_times(torch, dist, world, paced_run["wall_s"])
                tokens_paced = rank_times(torch, dist, world, float(paced_run["tokens"]))
                results["paced"] = {
                    "value": sum(tokens_paced) / max(walls), "unit": work.unit,
                    "offered_tokens_per_s": work.rate_per_gpu * world * work.max_new,
                    "wall_s": max(walls), "requests": paced_run["requests"],
                    "latency_s_p50": latency[len(latency) // 2] if latency else None,
                    "latency_s_p99": latency[min(len(latency) - 1, int(0.99 * len(latency)))]
                    if latency else None,
                    "how": "requests released at their Poisson arrival times (host clock); "
                           "tokens/s over the wall time from the first arrival to the last "
                           "finish"}
            del work.graphs
            work.graphs = {}
            torch.cuda.empty_cache()
    native, ref = results["native"], results["torch"]
    steps = native["decode_steps"]
    ms = max(native["rank_ms"])
    line = {
        "metric": work.metric, "value": native["value"], "unit": work.unit, "n_gpus": world,
        "steps": steps, "warmup": 8, "ms_per_step": ms / max(steps, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": dict(work.config(world), requests_per_gpu=len(mine),
                                            requests_total=len(trace),
                                            tokens_total=total_tokens),
        "rank_ms": native["rank_ms"], "rank_spread": max(native["rank_ms"]) / min(
            native["rank_ms"]),
        "serving": {"decode_steps": steps, "prefills": native["prefills"],
                    "tokens": native["tokens"], "requests": native["requests"]},
        "timing": "capacity run: this replica's whole share queued at once, device time from the "
                  "first prefill to the last finish (host checks every 4 steps included), "
                  "slowest rank",
        "torch_gpu_reference": {
            "value": ref["value"], "unit": work.unit, "ms_per_step": max(ref["rank_ms"]) / max(
                ref["decode_steps"], 1),
            "what": "the same engine with the reference's torch 2.11 attention path (padded SDPA "
                    "prefill, masked SDPA over key/value buckets, torch logits and _choose)"},
        "paced": results.get("paced"),
        "clocks": native["clocks"],
    }
    if cpu and rank == 0 and world == 1:
        line["cpu_baseline"] = work.cpu_rate(args.cpu_seconds, os.cpu_count() or 1)
    return line


WORKLOADS = {cls.name: cls for cls in (WhisperDecode, WhisperEncoder, Qwen3Decode, Qwen3Prefill,
                                       Qwen3AudioWindows, WhisperGreedyStep, Qwen3GreedyStep,
                                       WhisperCrossKV, WhisperPrefix, Qwen3Serve)}


# ------------------------------------------------------------------ arms ----

def run_reference(args, rank: int) -> None:
    """The reference arm: rank 0 times the reference's CPU path of the workload."""
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT))
    work = WORKLOADS[args.workload](args.batch)
    threads = os.cpu_count() or 1
    # The arm's budget covers the --warmup and --steps it was given: a bounded
    # sample, so the whole run ends within a few minutes.
    result = work.cpu_rate(args.cpu_seconds, threads)
    line = {
        "impl": "reference", "metric": work.metric, "value": result["value"], "unit": work.unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": work.units_per_step() / result["value"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": work.config(args.gpus), "cpu_baseline": result,
        "e2e": {"value": result["value"], "unit": work.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "reference CPU path = the reference's attention call (torch SDPA with its masks "
                "and grouped views) on the host cores in float32; the Python reference itself "
                "runs torch, so this is its CPU arithmetic",
    }
    print(json.dumps(line), flush=True)


def graph_time_ms(torch, fn, reps: int, replays: int = 4) -> float:
    """Average device time of fn(i) for i < reps, launched back to back from a
    CUDA graph, over `replays` replays (CUDA events on the current stream)."""
    from asrback_b200.transcription import CapturedGraph

    graph = CapturedGraph(lambda: [fn(i) for i in range(reps)], warmup=1)
    graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(replays):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) / (replays * reps)


def rank_times(torch, dist, world: int, ms: float) -> list[float]:
    """Every rank's device time of the same region (all-gather; the value
    alone without a process group)."""
    if world == 1:
        return [ms]
    tensor = torch.tensor([ms], dtype=torch.float64, device="cuda")
    out = [torch.zeros_like(tensor) for _ in range(world)]
    dist.all_gather(out, tensor)
    return [float(t.item()) for t in out]


def e2e_pipeline(torch, dist, work, world: int, first: int, steps: int) -> dict:
    """The K steps through the public ops with host buffers: step i's inputs
    are copied from pinned host memory into one of two device slots on a copy
    stream, the step runs on the compute stream once its copy has landed, and
    its outputs go back to pinned host memory on a second copy stream, so the
    copies of steps i+1 and i-1 overlap step i. The K steps, with their copies
    and the cross-stream dependencies (a slot is refilled only after the step
    two before has read it), are captured as one multi-stream CUDA graph and
    timed, like the device-resident steps, as one replay: from before the
    first copy in to after the last copy out, on the compute stream."""
    proto = work.inputs_at(first)
    slots = [[torch.empty_like(x) for x in proto] for _ in range(2)]
    for slot in slots:
        for dst, src in zip(slot, proto):
            dst.copy_(src)
    distinct = min(steps, 8)
    if work.name in ("whisper-encoder", "qwen3-prefill", "qwen3-audio"):
        distinct = 2  # hundreds of MB per step: two pinned copies alternate
    host = []
    for i in range(distinct):
        inputs = work.inputs_at(first + i)
        pinned = [torch.empty(x.shape, dtype=x.dtype, pin_memory=True) for x in inputs]
        for dst, src in zip(pinned, inputs):
            dst.copy_(src.cpu())
        host.append(pinned)
    in_bytes = sum(x.numel() * x.element_size() for x in proto)
    probe = work.launch(slots[0])
    out_bytes = sum(o.numel() * o.element_size() for o in probe)
    del probe
    host_out = [torch.empty((max(out_bytes, 1),), dtype=torch.uint8, pin_memory=True)
                for _ in range(2)]
    torch.cuda.synchronize()
    compute = torch.cuda.Stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    landed = [torch.cuda.Event() for _ in range(steps)]
    done = [torch.cuda.Event() for _ in range(steps)]
    outs = []
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(compute), torch.cuda.graph(graph, stream=compute):
        h2d.wait_stream(compute)
        d2h.wait_stream(compute)
        for i in range(steps):
            s = i % 2
            with torch.cuda.stream(h2d):
                if i >= 2:
                    h2d.wait_event(done[i - 2])  # step i-2 has read slot s
                for dst, src in zip(slots[s], host[i % distinct]):
                    dst.copy_(src, non_blocking=True)
                landed[i].record(h2d)
            compute.wait_event(landed[i])
            out = work.launch(slots[s])
            outs.append(out)
            done[i].record(compute)
            with torch.cuda.stream(d2h):
                d2h.wait_event(done[i])
                offset = 0
                for o in out:
                    n = o.numel() * o.element_size()
                    host_out[s][offset:offset + n].copy_(o.reshape(-1).view(torch.uint8),
                                                         non_blocking=True)
                    offset += n
        compute.wait_stream(h2d)
        compute.wait_stream(d2h)
    graph.replay()  # uploads the graph; untimed
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    # As for the device-resident replay: untimed replays keep the GPU's clocks
    # up to the synchronize (and barrier) that opens the timed one.
    for _ in range(2):
        graph.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    start.record(stream)
    graph.replay()
    end.record(stream)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    ranks = rank_times(torch, dist, world, ms)
    value = work.units_per_step() * world * steps / (max(ranks) / 1e3)
    return {"value": value, "unit": work.unit, "h2d_bytes_per_step": in_bytes,
            "d2h_bytes_per_step": out_bytes, "steps": steps,
            "how": "pinned host inputs in and outputs out every step, double-buffered on two "
                   "copy streams; the K steps with their copies captured as one multi-stream "
                   "graph, one replay, slowest rank",
            "rank_ms": ranks}


def reference_whisper_module():
    """The reference's ``asrback.models.whisper`` from ``$ASRBACK_REFERENCE`` (a
    checkout) or ``baseline/_ref`` (where a copy of its package is laid down),
    or None. Its audio front end ``asrfront`` is not installed and nothing
    timed here calls it, so a module with the constants read at import stands
    in for it."""
    import types

    roots = [Path(os.environ["ASRBACK_REFERENCE"]) if os.environ.get("ASRBACK_REFERENCE")
             else None, ROOT / "baseline" / "_ref"]
    found = None
    for root in roots:
        if root is None:
            continue
        for candidate in (root / "src", root):
            if (candidate / "asrback" / "__init__.py").is_file():
                found = candidate
                break
        if found:
            break
    if found is None:
        return None
    if "asrfront" not in sys.modules:
        stub = types.ModuleType("asrfront")
        constants = dict(SAMPLE_RATE=16000, N_SAMPLES=480000, HOP_LENGTH=160, MAX_SAMPLES=480000,
                         N_MELS=128)
        for name in ("whisper", "qwen3_asr", "sensevoice", "gemma4"):
            setattr(stub, name, types.SimpleNamespace(**constants))
        sys.modules["asrfront"] = stub
    if str(found) not in sys.path:
        sys.path.insert(0, str(found))
    from asrback.models import whisper

    return whisper


def measure_admission(torch, dist, device, world: int, batches: int = 4, rounds: int = 3) -> dict:
    """Window admission at the caller's boundary, through the reference's own
    modules: log-mel windows copied in from pinned host memory, the encoder
    (``WhisperEncoder.forward``, ``whisper.py:140-153``: convolution stem, 32
    layers, final norm) and ``set_encoder_output`` (``:313-319``) into the
    cross-attention cache of a 4-layer decoder, one cache row read back. Timed
    with ``asrback_b200.plugin`` installed (the encoder attention and the
    cross K/V projection on this package's kernels, the linears on cuBLAS),
    installed with ``encoder=False`` (the encoder attention left to the
    reference's SDPA, the cross K/V projection on this package's kernel) and
    without it (the reference's torch path: default SDPA, ``F.linear`` and the
    cache copy), eager as the reference runs ``_encode``; large-v3-turbo
    widths, 32 windows of N(0, 1) log-mel, seeded random weights."""
    whisper = reference_whisper_module()
    if whisper is None:
        return {"unavailable": "the reference's package is not present ($ASRBACK_REFERENCE or "
                               "baseline/_ref)"}
    from asrback_b200 import plugin

    config = dict(d_model=1280, encoder_attention_heads=20, decoder_attention_heads=20,
                  encoder_layers=32, decoder_layers=4, encoder_ffn_dim=5120, decoder_ffn_dim=5120,
                  num_mel_bins=128, max_source_positions=1500, max_target_positions=448,
                  vocab_size=51866)
    torch.manual_seed(2)
    with torch.device(device):  # nn's default initialisation, drawn on the GPU
        model = whisper.WhisperForConditionalGeneration(config)
    model = model.eval().to(torch.bfloat16)
    windows = 32
    gen = torch.Generator().manual_seed(2)
    host_mel = torch.randn((windows, 128, 3000), generator=gen).to(torch.bfloat16).pin_memory()
    cache = model.allocate_cache(windows)
    host_row = torch.empty(cache.cross_keys[3, 0, 0].shape, dtype=torch.bfloat16, pin_memory=True)
    stream = torch.cuda.current_stream()

    def admit():
        mel = host_mel.to(device, non_blocking=True)
        model.set_encoder_output(cache, model.model.encoder(mel))
        host_row.copy_(cache.cross_keys[3, windows - 1, 19], non_blocking=True)

    # The three legs alternate over `rounds` rounds and each keeps its best
    # round: a leg timed once, after the others, saw the GPU's clocks drop as
    # the power cap bit, whichever leg came last.
    best: dict[str, float] = {}
    legs = (("value", "all"), ("cross_only", "cross"), ("torch", None))
    with torch.inference_mode():
        for _ in range(rounds):
            for label, patched in legs:
                if patched:
                    plugin.install(whisper, None, encoder=patched == "all")
                try:
                    for _ in range(2):
                        admit()
                    torch.cuda.synchronize()
                    if world > 1:
                        dist.barrier()
                    start = torch.cuda.Event(enable_timing=True)
                    end = torch.cuda.Event(enable_timing=True)
                    start.record(stream)
                    for _ in range(batches):
                        admit()
                    end.record(stream)
                    torch.cuda.synchronize()
                finally:
                    if patched:
                        plugin.uninstall()
                ranks = rank_times(torch, dist, world, start.elapsed_time(end))
                best[label] = min(best.get(label, float("inf")), max(ranks))
    out = {}
    for label, _ in legs:
        out[label] = windows * batches * world / (best[label] / 1e3)
        out[f"{label}_ms_per_batch"] = best[label] / batches
    del model, cache
    torch.cuda.empty_cache()
    return {"value": out["value"], "unit": "windows/s", "ms_per_batch": out["value_ms_per_batch"],
            "cross_only": out["cross_only"],
            "cross_only_ms_per_batch": out["cross_only_ms_per_batch"],
            "torch": out["torch"], "torch_ms_per_batch": out["torch_ms_per_batch"],
            "what": "32 windows of host log-mel through the reference's encoder and "
                    "set_encoder_output (large-v3-turbo widths) into the cross cache, eager; "
                    "value with the plugin installed, cross_only with install(encoder=False), "
                    "torch without; the legs alternate over 3 rounds, best round each"}


def measure(args, work, torch, dist, device, rank: int, world: int, steps: int, warmup: int,
            cpu: bool, sustain: bool) -> dict:
    """Runs one workload: the timed graph of K steps, the sustained figure,
    per-kernel timing, e2e, the reference's torch path on the same GPU, and
    the CPU baseline."""
    from asrback_b200 import attention
    from asrback_b200.replicas import max_over_ranks
    from asrback_b200.transcription import CapturedGraph

    seed = SEED + 1000 * rank
    total = warmup + steps
    work.setup(torch, device, seed, total)
    stream = torch.cuda.current_stream()
    for t in range(warmup):
        work.step_at(t)
    timed = CapturedGraph(lambda: [work.step_at(t) for t in range(warmup, total)], warmup=1)
    timed.replay()  # uploads the graph; untimed
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()  # ranks finish their captures at different times

    uuid = getattr(torch.cuda.get_device_properties(device), "uuid", None)
    uuid = str(uuid) if uuid else None

    # ---- timed region: exactly K steps, one graph replay, inputs in HBM ----
    start_ev, end_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(uuid) as clocks:
        # A GPU left idle (a rank waiting for the others, the clock sampler
        # starting) drops its clocks, and a timed replay begun on it ran up to
        # 20 % slow. So untimed replays keep the GPU running up to the
        # synchronize (and, with several ranks, the barrier, whose collective
        # runs after them) that opens the timed region.
        for _ in range(3):
            timed.replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_push("timed")
        start_ev.record(stream)
        timed.replay()
        clocks.mark()
        end_ev.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        own_ms = start_ev.elapsed_time(end_ev)
        ranks = rank_times(torch, dist, world, own_ms)
        ms = max(ranks)
        sustained = None
        if sustain:
            replays = int(min(500, max(2, math.ceil(args.sustain_seconds * 1e3 / max(ms, 1e-3)))))
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            start_ev.record(stream)
            for _ in range(replays):
                timed.replay()
            clocks.mark()
            end_ev.record(stream)
            torch.cuda.synchronize()
            s_ranks = rank_times(torch, dist, world, start_ev.elapsed_time(end_ev))
            s_ms = max(s_ranks)
            sustained = {"value": work.units_per_step() * world * steps * replays / (s_ms / 1e3),
                         "unit": work.unit, "replays": replays, "steps": steps * replays,
                         "ms_per_step": s_ms / (steps * replays), "timed_region_s": s_ms / 1e3,
                         "rank_ms": s_ranks,
                         "how": "the timed graph replayed back to back (same K steps each "
                                "replay), slowest rank"}
    ms_per_step = ms / steps
    value = work.units_per_step() * world * steps / (ms / 1e3)

    # ---- kernel timing: average launch duration, launched from a graph ----
    kernel = {}
    layers = work.layers
    for name, fn, amount in work.kernels(warmup):
        launch_ms = graph_time_ms(torch, lambda i: fn(i % layers), 2 * layers)
        kernel[name] = {"launch_ms": launch_ms, "work_per_launch": amount}

    e2e = e2e_pipeline(torch, dist, work, world, warmup, steps)

    # ---- the reference's GPU computation on the same tensors, for context:
    # graph-replayed where the reference captures it (decoder steps), eager
    # where it does not (the encoder, admission) ----
    ref_fn = work.torch_reference_step(torch)
    r_start, r_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if work.reference_in_graph:
        ref_graph = CapturedGraph(lambda: [ref_fn(t) for t in range(warmup, total)], warmup=1)
        ref_graph.replay()
        torch.cuda.synchronize()
        r_start.record(stream)
        ref_graph.replay()
        r_end.record(stream)
    else:
        for t in range(min(warmup, 3)):
            ref_fn(t)
        torch.cuda.synchronize()
        r_start.record(stream)
        for t in range(warmup, total):
            ref_fn(t)
        r_end.record(stream)
    torch.cuda.synchronize()
    ref_ms = r_start.elapsed_time(r_end) / steps
    ref_graph = None
    flash = None
    if hasattr(work, "torch_flash_step"):
        fn = work.torch_flash_step(torch)
        for t in range(3):
            fn(t)
        torch.cuda.synchronize()
        r_start.record(stream)
        for t in range(steps):
            fn(t)
        r_end.record(stream)
        torch.cuda.synchronize()
        c_ms = r_start.elapsed_time(r_end) / steps
        flash = {"ms_per_step": c_ms, "value": work.units_per_step() / (c_ms * 1e-3),
                 "unit": work.unit, "what": "torch SDPA with the flash backend forced, eager"}

    dominant = work.kernels(warmup)[0]
    dom = kernel[dominant[0]]
    peak, peak_kind = peak_for(work.bound)
    scale = 1e9 if work.bound == "hbm" else 1e12
    unit = "GB/s" if work.bound == "hbm" else "TFLOP/s"
    achieved = dom["work_per_launch"] / (dom["launch_ms"] * 1e-3) / scale
    traffic = profiled_traffic(work.profile)
    status = attention.read_status(device)
    result = {
        "metric": work.metric, "value": value, "unit": work.unit, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": work.config(world),
        "e2e": e2e,
        "roofline": {"bound": work.bound, "kernel": dominant[0], "achieved": achieved,
                     "peak": peak, "unit": unit, "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "work_per_launch": dom["work_per_launch"],
                     "launch_ms": dom["launch_ms"]},
        "kernels": {
            name: dict(k, rate=k["work_per_launch"] / (k["launch_ms"] * 1e-3) / scale,
                       rate_unit=unit)
            for name, k in kernel.items()},
        "step_rate": {"value": work.step_work(warmup, steps) / steps / (ms_per_step * 1e-3)
                      / scale, "unit": unit},
        "rank_ms": ranks,
        "rank_spread": max(ranks) / min(ranks),
        "timing": "the K timed steps captured as one CUDA graph, one replay, slowest rank",
        "sustained": sustained,
        "torch_gpu_reference": {
            "ms_per_step": ref_ms, "value": work.units_per_step() / (ref_ms * 1e-3),
            "unit": work.unit,
            "what": "the reference's attention computation in torch on this GPU (same tensors)"},
        "torch_gpu_flash": flash,
        "gpu_launches": work.launches_per_step() * steps,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if work.name == "whisper-encoder":
        result["admission"] = measure_admission(torch, dist, device, world)
    max_over_ranks(0.0)  # every rank reaches the CPU leg together
    if cpu and rank == 0 and world == 1:
        result["cpu_baseline"] = work.cpu_rate(args.cpu_seconds, os.cpu_count() or 1)
    return result


def summary(name: str, line: dict) -> dict:
    """A short record of one workload's line (rounded), for the end of the
    printed line."""
    def r(x, digits=4):
        return None if x is None else float(f"{x:.{digits}g}")

    out = {"value": r(line["value"]), "unit": line["unit"], "ms": r(line["ms_per_step"])}
    if line.get("roofline"):
        out["frac"] = r(line["roofline"]["frac"], 3)
    if line.get("e2e"):
        out["e2e"] = r(line["e2e"]["value"])
    out["torch_gpu"] = r(line["torch_gpu_reference"]["value"])
    if line.get("torch_gpu_flash"):
        out["flash"] = r(line["torch_gpu_flash"]["value"])
    if line.get("cpu_baseline"):
        out["cpu"] = r(line["cpu_baseline"]["value"])
    if line.get("admission") and "value" in line["admission"]:
        out["admission"] = r(line["admission"]["value"])
        out["admission_torch"] = r(line["admission"]["torch"])
        out["admission_cross_only"] = r(line["admission"]["cross_only"])
    if line.get("paced"):
        out["paced"] = r(line["paced"]["value"])
        out["p99_s"] = r(line["paced"]["latency_s_p99"], 3)
    return out


def run_native(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    work = WORKLOADS[args.workload](args.batch)
    if args.layers:
        work.layers = args.layers
    cpu = not args.no_cpu_baseline
    if args.workload == "qwen3-serve":
        line = measure_serve(args, work, torch, dist, device, rank, world, 3 * work.max_batch,
                             cpu=cpu, paced=True)
        line["workloads"] = {work.name: summary(work.name, line)}
        if rank == 0:
            print(json.dumps(line), flush=True)
        return
    line = measure(args, work, torch, dist, device, rank, world, args.steps, args.warmup,
                   cpu=cpu, sustain=True)
    if cpu and rank == 0 and world == 1 and hasattr(work, "oracle_rate"):
        line["cpu_crosscheck"] = work.oracle_rate(min(args.cpu_seconds, 5.0),
                                                  os.cpu_count() or 1)
    short = {args.workload: summary(args.workload, line)}
    if args.workload == "whisper-decode" and not args.no_extras and args.batch is None:
        # Short runs of the other workloads (their K steps capped at 16), with
        # their own CPU baselines.
        extras = {}
        for name in ("whisper-encoder", "qwen3-decode", "qwen3-prefill", "qwen3-audio",
                     "whisper-step", "qwen3-step", "whisper-cross-kv", "whisper-prefix"):
            del work
            torch.cuda.empty_cache()
            work = WORKLOADS[name](None)
            r = measure(args, work, torch, dist, device, rank, world, min(args.steps, 16),
                        max(3, min(args.warmup, 5)), cpu=cpu, sustain=False)
            extras[name] = {k: r.get(k) for k in (
                "metric", "value", "unit", "ms_per_step", "e2e", "roofline", "step_rate",
                "rank_ms", "torch_gpu_reference", "torch_gpu_flash", "cpu_baseline", "clocks",
                "device_status", "config", "admission")}
            short[name] = summary(name, r)
        del work
        torch.cuda.empty_cache()
        work = WORKLOADS["qwen3-serve"](None)
        r = measure_serve(args, work, torch, dist, device, rank, world, 3 * work.max_batch,
                          cpu=cpu, paced=False)
        extras["qwen3-serve"] = {k: r.get(k) for k in (
            "metric", "value", "unit", "ms_per_step", "rank_ms", "serving", "torch_gpu_reference",
            "cpu_baseline", "clocks", "config")}
        short["qwen3-serve"] = summary("qwen3-serve", r)
        line["other_workloads"] = extras
    # The short records go last, so that the end of the line holds every
    # workload's figures.
    line["workloads"] = short
    if rank == 0:
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
        run_reference(args, rank)
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
