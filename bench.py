"""Benchmarks of asrback's attention hot path on B200 (one replica per GPU).

Default workload (the headline configuration): Whisper large-v3-turbo
decoder-step attention in bf16 -- 4 decoder layers, 20 heads x 64, batch 64
slots whose self-attention lengths start uniform in [1, 448] and grow by one
per step (rows that reach position 447, the last the cache holds, stay
computed, as in the reference), cross-attention over 1500 encoder frames whose
keys/values come from N(0, 1) encoder states through the decoder's own k/v
projections (seeded weights). One step = per layer, the self-attention with its
key/value write, then the cross-attention; the 8 launches replay from one CUDA
graph. Unit: decoded tokens (64 per step per GPU).

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
                   cross-attention over 1500 frames, 4 layers; unit: windows.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]
                    [--workload NAME] [--batch B]

``--impl reference`` times the reference's CPU path for the same workload (the
CPU oracle port of its attention in float32, all host threads) on a bounded
sample. Under torchrun every rank runs its own replica (weak scaling, no
collective on the data path); rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from concurrent.futures import ThreadPoolExecutor
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
    parser.add_argument("--workload", choices=("whisper-decode", "whisper-encoder", "qwen3-decode",
                                               "qwen3-prefill", "qwen3-audio", "whisper-step",
                                               "qwen3-step", "whisper-cross-kv",
                                               "whisper-prefix"),
                        default="whisper-decode")
    parser.add_argument("--batch", type=int, default=None,
                        help="override the workload's batch (small profiling cases)")
    parser.add_argument("--layers", type=int, default=None,
                        help="override the workload's layer count (small profiling cases that "
                             "keep the batch; not a bench line)")
    parser.add_argument("--cpu-seconds", type=float, default=10.0,
                        help="time budget of the CPU baseline sample")
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


def run_cpu(fn, rows, budget_s: float, threads: int):
    """Runs fn(step, row) over rows (a list) per step on `threads` threads until
    `budget_s` seconds have passed (at least one step); returns (steps, seconds)."""
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:  # pragma: no cover
        threadpool_limits = None
    limit = threadpool_limits(1) if threadpool_limits else None
    try:
        with ThreadPoolExecutor(max_workers=threads) as pool:
            start = time.perf_counter()
            done = 0
            while True:
                list(pool.map(lambda r: fn(done, r), rows))
                done += 1
                if time.perf_counter() - start >= budget_s or done >= 1024:
                    break
            elapsed = time.perf_counter() - start
    finally:
        if limit is not None and hasattr(limit, "unregister"):
            limit.unregister()
    return done, elapsed


# -------------------------------------------------------------- workloads ----

class WhisperDecode:
    """The headline: Whisper large-v3-turbo decoder-step attention."""

    name = "whisper-decode"
    metric = DECODE_METRIC
    unit = "tokens/s"
    bound = "hbm"
    reference_in_graph = True
    layers, heads, head_dim, target, source, width = 4, 20, 64, 448, 1500, 1280
    profile = "whisper_cross_decode_b64_bf16.md"

    def __init__(self, batch: int | None):
        self.batch = batch or 64

    def config(self, world: int) -> dict:
        return {
            "workload": "whisper-large-v3-turbo decoder-step attention (BASELINE config 2)",
            "model": "whisper-large-v3-turbo decoder attention, random init seed 1",
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

    def setup(self, torch, device, seed: int, total: int) -> None:
        from asrback_b200 import whisper
        from asrback_b200.synthetic import seeded_parameters

        dtype = torch.bfloat16
        rng = np.random.default_rng(seed)
        lengths = self.lengths(rng)
        start = lengths - 1
        self.schedule = np.minimum(start[None, :] + np.arange(total)[:, None],
                                   self.target - 1).astype(np.int64)
        config = whisper.large_v3_turbo_config()
        model = whisper.WhisperForConditionalGeneration(config, encoder=False)
        seeded_parameters(model.model.decoder, SEED)
        model = model.to(device, dtype).eval()
        self.cache = model.allocate_cache(self.batch)
        gen = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for b0 in range(0, self.batch, 16):
                b1 = min(self.batch, b0 + 16)
                states = torch.randn((b1 - b0, self.source, self.width), generator=gen,
                                     device=device, dtype=dtype)
                model.set_encoder_output(self.cache.rows(b0, b1), states)
            for layer in range(self.layers):
                for b in range(self.batch):
                    p = int(lengths[b]) - 1
                    if p > 0:
                        self.cache.self_keys[layer, b, :, :p].normal_(generator=gen)
                        self.cache.self_values[layer, b, :, :p].normal_(generator=gen)
        del model
        shape = (self.layers, 4, self.batch, self.heads, self.head_dim)
        self.inputs = torch.randn((total,) + shape, generator=gen, device=device, dtype=dtype)
        self.positions_all = torch.from_numpy(self.schedule).to(device)
        self.step_in = torch.empty(shape, device=device, dtype=dtype)
        self.pos = torch.empty((self.batch,), device=device, dtype=torch.int64)
        self.outputs: list = [None] * (2 * self.layers)

    def step(self) -> None:
        from asrback_b200 import attention

        c = self.cache
        for layer in range(self.layers):
            x = self.step_in[layer]
            self.outputs[2 * layer] = attention.whisper_self_attention_step(
                x[0], x[1], x[2], c.self_keys[layer], c.self_values[layer], self.pos)
            self.outputs[2 * layer + 1] = attention.whisper_cross_attention_step(
                x[3], c.cross_keys[layer], c.cross_values[layer])

    def launches_per_step(self) -> int:
        return 2 * self.layers

    def refresh(self, t: int) -> None:
        self.step_in.copy_(self.inputs[t])
        self.pos.copy_(self.positions_all[t])

    def host_step_inputs(self, torch, first: int, count: int):
        """Pinned host copies of steps first..first+count and their device targets."""
        host_in = torch.empty((count,) + tuple(self.step_in.shape), dtype=self.step_in.dtype,
                              pin_memory=True)
        host_in.copy_(self.inputs[first:first + count].cpu())
        host_pos = torch.from_numpy(self.schedule[first:first + count].copy()).pin_memory()
        return [(host_in, self.step_in), (host_pos, self.pos)]

    def row_bytes(self) -> int:
        return self.heads * self.head_dim * 2 * 2  # K and V, bf16

    def kernels(self, t: int):
        """(name, launch function, algorithmic bytes of one launch) per kernel."""
        from asrback_b200 import attention

        c, x, pos = self.cache, self.inputs, self.positions_all
        self_bytes = float((self.schedule[t] + 1).sum()) * self.row_bytes()
        cross_bytes = float(self.batch * self.source * self.row_bytes())
        return [
            ("cross", lambda layer: attention.whisper_cross_attention_step(
                x[t, layer, 3], c.cross_keys[layer], c.cross_values[layer]), cross_bytes),
            ("self", lambda layer: attention.whisper_self_attention_step(
                x[t, layer, 0], x[t, layer, 1], x[t, layer, 2], c.self_keys[layer],
                c.self_values[layer], pos[t]), self_bytes),
        ]

    def step_work(self, first: int, count: int) -> float:
        """Algorithmic bytes of steps first..first+count."""
        sched = self.schedule[first:first + count]
        per_row = self.row_bytes() * self.layers
        return float(((sched + 1).sum() + count * self.batch * self.source) * per_row)

    def torch_reference_step(self, torch):
        """The reference's own GPU computation of one step's attention (torch SDPA
        with its bool step mask and cuDNN-first backend priority, as
        whisper.py:58-63 and :222-240 run it), for context."""
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        c, x = self.cache, self.step_in
        key_positions = torch.arange(self.target, device=x.device)
        backends = [SDPBackend.CUDNN_ATTENTION, SDPBackend.FLASH_ATTENTION,
                    SDPBackend.EFFICIENT_ATTENTION, SDPBackend.MATH]
        rows = torch.arange(self.batch, device=x.device)

        def run():
            mask = (key_positions[None, :] <= self.pos[:, None])[:, None, None, :]
            with sdpa_kernel(backends, set_priority=True):
                for layer in range(self.layers):
                    q, k, v, qc = (x[layer, i][:, :, None, :] for i in range(4))
                    c.self_keys[layer][rows, :, self.pos] = k[:, :, 0]
                    c.self_values[layer][rows, :, self.pos] = v[:, :, 0]
                    F.scaled_dot_product_attention(q, c.self_keys[layer], c.self_values[layer],
                                                   attn_mask=mask)
                    F.scaled_dot_product_attention(qc, c.cross_keys[layer], c.cross_values[layer])
        return run

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import attention as oracle

        rows, steps = 16, 64
        rng = np.random.default_rng(seed)
        lengths = self.lengths(rng)[:rows]
        positions = np.minimum(lengths[None, :] - 1 + np.arange(steps)[:, None], self.target - 1)
        f32 = np.float32
        sk = rng.standard_normal((self.layers, rows, self.heads, self.target, self.head_dim), dtype=f32)
        sv = rng.standard_normal(sk.shape, dtype=f32)
        ck = rng.standard_normal((self.layers, rows, self.heads, self.source, self.head_dim), dtype=f32)
        cv = rng.standard_normal(ck.shape, dtype=f32)
        q = rng.standard_normal((steps, self.layers, 4, rows, self.heads, self.head_dim), dtype=f32)

        def one(t, b):
            t %= steps
            for layer in range(self.layers):
                oracle.whisper_self_attention_step(
                    q[t, layer, 0, b:b + 1], q[t, layer, 1, b:b + 1], q[t, layer, 2, b:b + 1],
                    sk[layer, b:b + 1], sv[layer, b:b + 1], positions[t, b:b + 1],
                    compute=f32, copy=False)
                oracle.whisper_cross_attention(q[t, layer, 3, b:b + 1], ck[layer, b:b + 1],
                                               cv[layer, b:b + 1], compute=f32)

        done, elapsed = run_cpu(one, list(range(rows)), budget_s, threads)
        return {"value": rows * done / elapsed, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{rows} of {self.batch} rows x {done} steps x {self.layers} layers "
                          f"(self with in-place append + cross over {self.source}), float32 "
                          f"numpy oracle, {elapsed:.1f} s"}


class WhisperEncoder:
    """Whisper large-v3-turbo encoder self-attention prefill."""

    name = "whisper-encoder"
    metric = "encoder windows/s/GPU (32 windows x 1500 frames, 32 layers, bf16); attention TFLOP/s"
    unit = "windows/s"
    bound = "tensor"
    reference_in_graph = False
    layers, heads, head_dim, length = 32, 20, 64, 1500
    profile = "whisper_encoder_attention_b32_bf16.md"

    def __init__(self, batch: int | None):
        self.batch = batch or 32

    def config(self, world: int) -> dict:
        return {
            "workload": "whisper-large-v3-turbo encoder self-attention prefill (BASELINE config 3)",
            "layers": self.layers, "heads": self.heads, "head_dim": self.head_dim,
            "frames": self.length, "batch_per_gpu": self.batch, "global_batch": self.batch * world,
            "step": "32 layers of non-causal attention over the batch's windows",
            "inputs": "N(0,1) bf16 q/k/v per layer in the projections' (B, S, H*D) layout",
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2 (369 MB of q/k/v per layer)",
        }

    def units_per_step(self) -> int:
        return self.batch

    def flops_per_layer(self) -> float:
        return 4.0 * self.length ** 2 * self.head_dim * self.heads * self.batch

    def setup(self, torch, device, seed: int, total: int) -> None:
        gen = torch.Generator(device=device).manual_seed(seed)
        shape = (self.batch, self.length, self.heads * self.head_dim)
        self.qkv = [[torch.randn(shape, generator=gen, device=device, dtype=torch.bfloat16)
                     for _ in range(3)] for _ in range(self.layers)]
        self.outputs: list = [None] * self.layers

    def views(self, layer: int):
        b, s, h, d = self.batch, self.length, self.heads, self.head_dim
        return [t.view(b, s, h, d).transpose(1, 2) for t in self.qkv[layer]]

    def step(self) -> None:
        from asrback_b200 import attention

        for layer in range(self.layers):
            self.outputs[layer] = attention.whisper_encoder_attention(*self.views(layer))

    def launches_per_step(self) -> int:
        return self.layers

    def refresh(self, t: int) -> None:
        pass

    def host_step_inputs(self, torch, first: int, count: int):
        # One layer's q/k/v in pinned memory, copied into every layer's inputs.
        host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in self.qkv[0]]
        for h, d in zip(host, self.qkv[0]):
            h.copy_(d.cpu())
        pairs = []
        for layer in range(self.layers):
            for i in range(3):
                pairs.append((host[i][None].expand(count, *host[i].shape), self.qkv[layer][i]))
        return pairs

    def kernels(self, t: int):
        from asrback_b200 import attention

        return [("encoder", lambda layer: attention.whisper_encoder_attention(*self.views(layer)),
                 self.flops_per_layer())]

    def step_work(self, first: int, count: int) -> float:
        return self.flops_per_layer() * self.layers * count

    def torch_reference_step(self, torch):
        """torch SDPA on the same tensors (the reference's encoder call, default
        backend priority, eager as the reference runs it), for context."""
        import torch.nn.functional as F

        def run():
            for layer in range(self.layers):
                F.scaled_dot_product_attention(*self.views(layer))
        return run

    def torch_cudnn_step(self, torch):
        """The same with torch's cuDNN attention backend forced (the fastest
        torch kernel for this shape on B200)."""
        import torch.nn.functional as F
        from torch.nn.attention import SDPBackend, sdpa_kernel

        def run():
            with sdpa_kernel([SDPBackend.CUDNN_ATTENTION]):
                for layer in range(self.layers):
                    F.scaled_dot_product_attention(*self.views(layer))
        return run

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import attention as oracle

        rng = np.random.default_rng(seed)
        f32 = np.float32
        q, k, v = (rng.standard_normal((self.heads, self.length, self.head_dim), dtype=f32)
                   for _ in range(3))

        def one(_t, h):
            oracle.sdpa(q[h], k[h], v[h], compute=f32)

        done, elapsed = run_cpu(one, list(range(self.heads)), budget_s, threads)
        # `done` layer-windows (all heads) in `elapsed`; a window needs 32 layers.
        rate = done / elapsed / self.layers
        return {"value": rate, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{done} layer-windows (20 heads x 1500 x 1500 each), float32 numpy "
                          f"oracle, {elapsed:.1f} s, scaled by 1/32 layers"}


class Qwen3Decode:
    """Qwen3-1.7B-style decode attention."""

    name = "qwen3-decode"
    metric = "decoder tokens/s/GPU (Qwen3 1.7B-style, batch 64, bf16); attention HBM GB/s"
    unit = "tokens/s"
    bound = "hbm"
    reference_in_graph = True
    layers, heads, kv_heads, head_dim, cache_length, prompt = 28, 16, 8, 128, 1024, 410
    profile = "qwen3_decode_b64_bf16.md"

    def __init__(self, batch: int | None):
        self.batch = batch or 64

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

    def setup(self, torch, device, seed: int, total: int) -> None:
        from asrback_b200 import qwen3_asr

        dtype = torch.bfloat16
        gen = torch.Generator(device=device).manual_seed(seed)
        config = qwen3_asr.text_config_1_7b()
        self.cache = qwen3_asr.KVCache.allocate(config, self.batch, self.cache_length,
                                                device=device, dtype=dtype)
        self.cache.keys[:, :, :self.prompt].normal_(generator=gen)
        self.cache.values[:, :, :self.prompt].normal_(generator=gen)
        self.cos, self.sin = qwen3_asr.rope_tables(1e6, self.head_dim, self.cache_length,
                                                   device=device, dtype=dtype)
        self.norms = (1 + 0.1 * torch.randn((self.layers, 2, self.head_dim), generator=gen,
                                            device=device)).to(dtype)
        width = (self.heads + 2 * self.kv_heads) * self.head_dim
        self.inputs = torch.randn((total, self.layers, self.batch, width), generator=gen,
                                  device=device, dtype=dtype)
        self.schedule = np.minimum(self.prompt + np.arange(total)[:, None]
                                   + np.zeros((1, self.batch), np.int64),
                                   self.cache_length - 1).astype(np.int64)
        self.positions_all = torch.from_numpy(self.schedule).to(device)
        self.step_in = torch.empty((self.layers, self.batch, width), device=device, dtype=dtype)
        self.pos = torch.empty((self.batch,), device=device, dtype=torch.int64)
        self.outputs: list = [None] * self.layers

    def attend(self, layer, qkv, pos):
        from asrback_b200 import attention

        return attention.qwen3_attention_step(
            qkv, self.norms[layer, 0], self.norms[layer, 1], 1e-6, self.cos, self.sin, pos,
            self.cache.keys[layer], self.cache.values[layer], self.heads, self.kv_heads)

    def step(self) -> None:
        for layer in range(self.layers):
            self.outputs[layer] = self.attend(layer, self.step_in[layer], self.pos)

    def launches_per_step(self) -> int:
        return self.layers

    def refresh(self, t: int) -> None:
        self.step_in.copy_(self.inputs[t])
        self.pos.copy_(self.positions_all[t])

    def host_step_inputs(self, torch, first: int, count: int):
        host_in = torch.empty((count,) + tuple(self.step_in.shape), dtype=self.step_in.dtype,
                              pin_memory=True)
        host_in.copy_(self.inputs[first:first + count].cpu())
        host_pos = torch.from_numpy(self.schedule[first:first + count].copy()).pin_memory()
        return [(host_in, self.step_in), (host_pos, self.pos)]

    def row_bytes(self) -> int:
        return self.kv_heads * self.head_dim * 2 * 2

    def kernels(self, t: int):
        x, pos = self.inputs, self.positions_all
        bytes_ = float((self.schedule[t] + 1).sum()) * self.row_bytes()
        return [("qwen3", lambda layer: self.attend(layer, x[t, layer], pos[t]), bytes_)]

    def step_work(self, first: int, count: int) -> float:
        sched = self.schedule[first:first + count]
        return float((sched + 1).sum()) * self.row_bytes() * self.layers

    def torch_reference_step(self, torch):
        """The reference's GPU fallback on torch 2.11 (varlen_attn lacks the
        kwargs it passes): q/k RMSNorm + RoPE in bf16, cache write, SDPA with
        the bucket mask over the grouped heads (qwen3_asr.py:366-372, 392-432)."""
        import torch.nn.functional as F

        h, kvh, d = self.heads, self.kv_heads, self.head_dim
        rows = torch.arange(self.batch, device=self.pos.device)
        key_positions = torch.arange(self.cache_length, device=self.pos.device)

        def rotate(x, cos, sin):
            first, second = x.chunk(2, dim=-1)
            return x * cos[:, None, :] + torch.cat((-second, first), dim=-1) * sin[:, None, :]

        def run():
            cos, sin = self.cos[self.pos], self.sin[self.pos]
            mask = (key_positions[None, :] <= self.pos[:, None])[:, None, None, :]
            for layer in range(self.layers):
                q, k, v = self.step_in[layer].split([h * d, kvh * d, kvh * d], dim=-1)
                q = rotate(F.rms_norm(q.reshape(-1, h, d), (d,), self.norms[layer, 0], 1e-6), cos, sin)
                k = rotate(F.rms_norm(k.reshape(-1, kvh, d), (d,), self.norms[layer, 1], 1e-6), cos, sin)
                keys, values = self.cache.keys[layer], self.cache.values[layer]
                keys[rows, self.pos] = k
                values[rows, self.pos] = v.reshape(-1, kvh, d)
                F.scaled_dot_product_attention(q.view(-1, kvh, h // kvh, d), keys.transpose(1, 2),
                                               values.transpose(1, 2), attn_mask=mask)
        return run

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import attention as oracle

        rows = 8
        rng = np.random.default_rng(seed)
        f32 = np.float32
        width = (self.heads + 2 * self.kv_heads) * self.head_dim
        keys = rng.standard_normal((rows, self.cache_length, self.kv_heads, self.head_dim), dtype=f32)
        values = rng.standard_normal(keys.shape, dtype=f32)
        qkv = rng.standard_normal((rows, width), dtype=f32)
        w = np.ones(self.head_dim, f32)
        cos, sin = oracle.rope_tables(1e6, self.head_dim, self.cache_length)

        def one(t, b):
            pos = np.array([min(self.prompt + t, self.cache_length - 1)])
            for _layer in range(self.layers):
                oracle.qwen3_decode_attention(qkv[b:b + 1], w, w, 1e-6, cos, sin, pos,
                                              keys[b:b + 1], values[b:b + 1], self.heads,
                                              self.kv_heads)

        done, elapsed = run_cpu(one, list(range(rows)), budget_s, threads)
        return {"value": rows * done / elapsed, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{rows} of {self.batch} rows x {done} steps x {self.layers} layers, "
                          f"numpy oracle, {elapsed:.1f} s"}


class Qwen3Prefill:
    """Admission prefill of the Qwen3 decode workload's prompts: causal grouped-query
    attention within the packed prompts (TextAttention.prefill's `attend`)."""

    name = "qwen3-prefill"
    metric = ("prefill tokens/s/GPU (Qwen3 1.7B-style, 64 packed prompts x 410 tokens, 28 layers, "
              "bf16); attention TFLOP/s")
    unit = "tokens/s"
    bound = "tensor"
    reference_in_graph = False
    layers, heads, kv_heads, head_dim, prompt = 28, 16, 8, 128, 410
    profile = "qwen3_prefill_b64_bf16.md"

    def __init__(self, batch: int | None):
        self.batch = batch or 64

    def config(self, world: int) -> dict:
        return {
            "workload": "Qwen3-ASR-1.7B-style packed prompt prefill attention (BASELINE config 4 "
                        "admission: 390 audio + 20 prompt positions per row)",
            "layers": self.layers, "heads": self.heads, "kv_heads": self.kv_heads,
            "head_dim": self.head_dim, "causal": True, "prompts_per_gpu": self.batch,
            "prompt_tokens": self.prompt, "global_batch": self.batch * world,
            "step": "28 layers of causal varlen attention over the packed prompts",
            "inputs": "N(0,1) bf16 q (tokens, 16, 128), k/v (tokens, 8, 128) per layer",
            "parallelism": f"replicas x{world} (no collective)",
            "l2": "inputs larger than L2 (215 MB of q/k/v per layer)",
        }

    def units_per_step(self) -> int:
        return self.batch * self.prompt

    def flops_per_layer(self) -> float:
        # Causal: query i reads i + 1 keys; 2 flops per multiply-add, QK and PV.
        pairs = self.prompt * (self.prompt + 1) / 2
        return 4.0 * pairs * self.head_dim * self.heads * self.batch

    def setup(self, torch, device, seed: int, total: int) -> None:
        gen = torch.Generator(device=device).manual_seed(seed)
        tokens = self.batch * self.prompt
        dtype = torch.bfloat16
        self.q = [torch.randn((tokens, self.heads, self.head_dim), generator=gen, device=device,
                              dtype=dtype) for _ in range(self.layers)]
        self.k = [torch.randn((tokens, self.kv_heads, self.head_dim), generator=gen, device=device,
                              dtype=dtype) for _ in range(self.layers)]
        self.v = [torch.randn((tokens, self.kv_heads, self.head_dim), generator=gen, device=device,
                              dtype=dtype) for _ in range(self.layers)]
        self.starts = (torch.arange(self.batch + 1, device=device) * self.prompt).to(torch.int32)
        self.outputs: list = [None] * self.layers

    def attend(self, layer):
        from asrback_b200 import attention

        return attention.varlen_attention(self.q[layer], self.k[layer], self.v[layer],
                                          self.starts, self.prompt, True)

    def step(self) -> None:
        for layer in range(self.layers):
            self.outputs[layer] = self.attend(layer)

    def launches_per_step(self) -> int:
        return self.layers

    def refresh(self, t: int) -> None:
        pass

    def host_step_inputs(self, torch, first: int, count: int):
        # One layer's q/k/v in pinned memory, copied into every layer's inputs.
        host = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
                for t in (self.q[0], self.k[0], self.v[0])]
        for h, d in zip(host, (self.q[0], self.k[0], self.v[0])):
            h.copy_(d.cpu())
        pairs = []
        for layer in range(self.layers):
            for h, d in zip(host, (self.q[layer], self.k[layer], self.v[layer])):
                pairs.append((h[None].expand(count, *h.shape), d))
        return pairs

    def kernels(self, t: int):
        return [("varlen", self.attend, self.flops_per_layer())]

    def step_work(self, first: int, count: int) -> float:
        return self.flops_per_layer() * self.layers * count

    def torch_reference_step(self, torch):
        """The reference's `attend` on its GPU path under torch 2.11 (varlen_attn
        lacks the kwargs it passes, so the padded batch): gather the prompts,
        SDPA with the valid & causal mask and grouped heads, keep the valid
        rows (qwen3_asr.py:136-149, 166-181), on the same tensors."""
        import torch.nn.functional as F

        device = self.starts.device
        offsets = torch.arange(self.prompt, device=device)
        sizes = self.starts[1:] - self.starts[:-1]
        valid = offsets[None, :] < sizes[:, None]
        last = (self.starts[1:] - 1)[:, None]
        gather = torch.minimum(self.starts[:-1, None] + offsets, last)
        causal = torch.ones((self.prompt, self.prompt), dtype=torch.bool, device=device).tril()
        mask = valid[:, None, None, :] & causal

        def run():
            for layer in range(self.layers):
                out = F.scaled_dot_product_attention(
                    *(t[gather].transpose(1, 2) for t in (self.q[layer], self.k[layer], self.v[layer])),
                    attn_mask=mask, enable_gqa=True)
                out.transpose(1, 2)[valid]
        return run

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import attention as oracle

        rng = np.random.default_rng(seed)
        f32 = np.float32
        q = rng.standard_normal((self.prompt, self.heads, self.head_dim), dtype=f32)
        k = rng.standard_normal((self.prompt, self.kv_heads, self.head_dim), dtype=f32)
        v = rng.standard_normal((self.prompt, self.kv_heads, self.head_dim), dtype=f32)
        starts = np.array([0, self.prompt])

        def one(_t, _p):
            oracle.varlen_attention(q, k, v, starts, True, compute=f32)

        done, elapsed = run_cpu(one, list(range(threads)), budget_s, threads)
        # `done` rounds of `threads` prompt-layers in `elapsed`; a prompt needs 28 layers.
        layers_done = done * threads
        rate = layers_done / elapsed / self.layers * self.prompt
        return {"value": rate, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{layers_done} prompt-layers (16 heads x 410 x 410 causal each), float32 "
                          f"numpy oracle, {elapsed:.1f} s, scaled by 1/28 layers"}


class Qwen3AudioWindows(Qwen3Prefill):
    """Qwen3-ASR audio encoder attention: non-causal attention within 104-token
    windows of packed audio tokens (AudioAttention.forward's `attend`)."""

    name = "qwen3-audio"
    metric = ("audio tokens/s/GPU (Qwen3-ASR-style audio encoder attention, 64 x 30 s requests "
              "in 104-token windows, bf16); attention TFLOP/s")
    unit = "tokens/s"
    bound = "tensor"
    # 30 s of audio = 30 chunks of 13 tokens = 390 tokens per request: windows
    # of 104 tokens (8 chunks) and a last window of 78.
    layers, heads, kv_heads, head_dim, prompt = 24, 16, 16, 64, 390
    window = 104
    profile = "qwen3_audio_b64_bf16.md"

    def config(self, world: int) -> dict:
        return {
            "workload": "Qwen3-ASR-style audio encoder window attention (admission of audio windows)",
            "layers": self.layers, "heads": self.heads, "head_dim": self.head_dim,
            "causal": False, "requests_per_gpu": self.batch, "tokens_per_request": self.prompt,
            "window_tokens": self.window, "global_batch": self.batch * world,
            "assumed": "24 layers, 16 heads of 64 (d_model 1024); the checkpoint's audio config "
                       "is not available here",
            "step": "24 layers of non-causal varlen attention over the packed windows",
            "inputs": "N(0,1) bf16 q/k/v (tokens, 16, 64) per layer",
            "parallelism": f"replicas x{world} (no collective)",
        }

    def lengths(self) -> list[int]:
        per = [self.window] * (self.prompt // self.window)
        if self.prompt % self.window:
            per.append(self.prompt % self.window)
        return per * self.batch

    def flops_per_layer(self) -> float:
        return float(sum(4.0 * n * n * self.head_dim * self.heads for n in self.lengths()))

    def setup(self, torch, device, seed: int, total: int) -> None:
        super().setup(torch, device, seed, total)
        lengths = torch.tensor(self.lengths())
        self.starts = torch.nn.functional.pad(lengths.cumsum(0), (1, 0)).to(torch.int32).to(device)

    def attend(self, layer):
        from asrback_b200 import attention

        return attention.varlen_attention(self.q[layer], self.k[layer], self.v[layer],
                                          self.starts, self.window, False)

    def torch_reference_step(self, torch):
        """The reference's padded path for the windows: gather, SDPA with the
        valid mask (no causal part), keep the valid rows."""
        import torch.nn.functional as F

        device = self.starts.device
        offsets = torch.arange(self.window, device=device)
        sizes = self.starts[1:] - self.starts[:-1]
        valid = offsets[None, :] < sizes[:, None]
        last = (self.starts[1:] - 1)[:, None]
        gather = torch.minimum(self.starts[:-1, None] + offsets, last)
        mask = valid[:, None, None, :]

        def run():
            for layer in range(self.layers):
                out = F.scaled_dot_product_attention(
                    *(t[gather].transpose(1, 2) for t in (self.q[layer], self.k[layer], self.v[layer])),
                    attn_mask=mask)
                out.transpose(1, 2)[valid]
        return run

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import attention as oracle

        rng = np.random.default_rng(seed)
        f32 = np.float32
        q = rng.standard_normal((self.prompt, self.heads, self.head_dim), dtype=f32)
        k = rng.standard_normal(q.shape, dtype=f32)
        v = rng.standard_normal(q.shape, dtype=f32)
        starts = np.concatenate([[0], np.cumsum(self.lengths()[: len(self.lengths()) // self.batch])])

        def one(_t, _p):
            oracle.varlen_attention(q, k, v, starts, False, compute=f32)

        done, elapsed = run_cpu(one, list(range(threads)), budget_s, threads)
        layers_done = done * threads
        rate = layers_done / elapsed / self.layers * self.prompt
        return {"value": rate, "unit": self.unit, "cores": threads, "kind": "port",
                "sample": f"{layers_done} request-layers (16 heads x windows of 104), float32 numpy "
                          f"oracle, {elapsed:.1f} s, scaled by 1/24 layers"}


class WhisperCrossKV:
    """Admission of 32 encoded windows into the decoder:
    `set_encoder_output` (whisper.py:313-319), each of the 4 decoder
    layers' cross-attention keys/values projected from the encoder output and
    written into the cache."""

    name = "whisper-cross-kv"
    metric = ("cross-attention K/V fill windows/s/GPU (Whisper large-v3-turbo set_encoder_output: "
              "32 windows x 1500 frames, 4 decoder layers, bf16); projection TFLOP/s")
    unit = "windows/s"
    bound = "tensor"
    reference_in_graph = False
    layers, width, tokens, heads = 4, 1280, 1500, 20
    profile = "cross_kv_projection_b32_bf16.md"

    def __init__(self, batch: int | None):
        self.batch = batch or 32

    def config(self, world: int) -> dict:
        return {
            "workload": "Whisper large-v3-turbo set_encoder_output: k_proj/v_proj of the encoder "
                        "output into the cross-attention cache (window admission)",
            "layers": self.layers, "width": self.width, "heads": self.heads,
            "frames": self.tokens, "windows_per_gpu": self.batch,
            "global_batch": self.batch * world,
            "step": "4 decoder layers' projections into the cache",
            "inputs": "encoder output N(0, 1) bf16, weights N(0, 1/width), v_proj bias N(0, 0.02)",
            "parallelism": f"replicas x{world} (no collective)",
        }

    def units_per_step(self) -> int:
        return self.batch

    def flops_per_layer(self) -> float:
        return 2.0 * self.batch * self.tokens * 2 * self.width * self.width

    def setup(self, torch, device, seed: int, total: int) -> None:
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
        self.outputs = [self.keys[layer, 0, 0, 0] for layer in range(self.layers)]

    def attend(self, layer: int) -> None:
        from asrback_b200 import attention

        attention.whisper_cross_kv_projection(self.x, self.wk[layer], self.wv[layer],
                                              self.bv[layer], self.keys[layer],
                                              self.values[layer])

    def step(self) -> None:
        for layer in range(self.layers):
            self.attend(layer)

    def launches_per_step(self) -> int:
        return self.layers

    def refresh(self, t: int) -> None:
        pass

    def host_step_inputs(self, torch, first: int, count: int):
        host = torch.empty(self.x.shape, dtype=self.x.dtype, pin_memory=True)
        host.copy_(self.x.cpu())
        return [(host[None].expand(count, *host.shape), self.x)]

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

        def run():
            for layer in range(self.layers):
                self.keys[layer, :self.batch] = split(F.linear(self.x, self.wk[layer]))
                self.values[layer, :self.batch] = split(
                    F.linear(self.x, self.wv[layer], self.bv[layer]))
        return run

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import attention as oracle

        rng = np.random.default_rng(seed)
        w = self.width
        x = rng.standard_normal((1, self.tokens, w), dtype=np.float32)
        wk = rng.standard_normal((w, w), dtype=np.float32) / w ** 0.5
        wv = rng.standard_normal((w, w), dtype=np.float32) / w ** 0.5
        bv = rng.standard_normal((w,), dtype=np.float32) * 0.02

        def one(_t, _p):
            oracle.cross_kv_projection(x, wk, wv, bv, compute=np.float32)

        done, elapsed = run_cpu(one, list(range(threads)), budget_s, threads)
        layers_done = done * threads
        return {"value": layers_done / elapsed / self.layers, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{layers_done} window-layers (1500 x 1280 @ 1280 x 2560), float32 "
                          f"numpy oracle, {elapsed:.1f} s, scaled by 1/4 layers"}


class WhisperPrefix:
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
    reference_in_graph = False
    layers, heads, dim, frames, bucket = 4, 20, 64, 1500, 448
    profile = "whisper_prefix_b32_bf16.md"

    def __init__(self, batch: int | None, tokens: int = 4):
        self.batch = batch or 32
        self.tokens = tokens

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

    def setup(self, torch, device, seed: int, total: int) -> None:
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
        self.outputs: list = [None] * (2 * self.layers)

    def _query(self, x):
        b, p, _ = x.shape
        return x.view(b, p, self.heads, self.dim).transpose(1, 2)

    def attend_self(self, layer: int):
        from asrback_b200 import attention

        layer %= self.layers
        p = self.tokens
        return attention.whisper_self_attention_prefix(
            self._query(self.self_q), self.self_k[layer][:, :, :p], self.self_v[layer][:, :, :p])

    def attend_cross(self, layer: int):
        from asrback_b200 import attention

        layer %= self.layers
        return attention.whisper_cross_attention_prefix(
            self._query(self.cross_q), self.cross_k[layer], self.cross_v[layer])

    def step(self) -> None:
        for layer in range(self.layers):
            self.outputs[2 * layer] = self.attend_self(layer)
            self.outputs[2 * layer + 1] = self.attend_cross(layer)

    def launches_per_step(self) -> int:
        return 2 * self.layers

    def refresh(self, t: int) -> None:
        pass

    def host_step_inputs(self, torch, first: int, count: int):
        pairs = []
        for dev in (self.self_q, self.cross_q):
            host = torch.empty(dev.shape, dtype=dev.dtype, pin_memory=True)
            host.copy_(dev.cpu())
            pairs.append((host[None].expand(count, *host.shape), dev))
        return pairs

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

        def run():
            for layer in range(self.layers):
                F.scaled_dot_product_attention(
                    self._query(self.self_q), self.self_k[layer][:, :, :p],
                    self.self_v[layer][:, :, :p], is_causal=p > 1)
                F.scaled_dot_product_attention(
                    self._query(self.cross_q), self.cross_k[layer], self.cross_v[layer])
        return run

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import attention as oracle

        rng = np.random.default_rng(seed)
        h, p, d = self.heads, self.tokens, self.dim
        q = rng.standard_normal((1, h, p, d), dtype=np.float32)
        k = rng.standard_normal((1, h, p, d), dtype=np.float32)
        ck = rng.standard_normal((1, h, self.frames, d), dtype=np.float32)
        cv = rng.standard_normal((1, h, self.frames, d), dtype=np.float32)
        mask = np.arange(p)[None, :] <= np.arange(p)[:, None]

        def one(_t, _p):
            oracle.sdpa(q, k, k, mask, compute=np.float32)
            oracle.whisper_cross_attention_prefix(q, ck, cv, compute=np.float32)

        done, elapsed = run_cpu(one, list(range(threads)), budget_s, threads)
        layers_done = done * threads
        return {"value": layers_done / elapsed / self.layers, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{layers_done} window-layers (20 heads, {p} prompt tokens, self + cross "
                          f"over 1500 frames), float32 numpy oracle, {elapsed:.1f} s, scaled by "
                          f"1/4 layers"}


class WhisperGreedyStep:
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
    vocab, width, length, eos = 51866, 1280, 448, (50257,)
    copies = 4  # weight copies, rotated so that no launch finds its weights in L2
    profile = "greedy_step_whisper_b64_bf16.md"

    def __init__(self, batch: int | None):
        self.batch = batch or 64
        self.layers = self.copies

    def config(self, world: int) -> dict:
        return {
            "workload": f"{self.family} greedy step epilogue (logits GEMM + _choose + state "
                        "update after the decoder)",
            "vocab": self.vocab, "hidden": self.width, "rows_per_gpu": self.batch,
            "global_batch": self.batch * world, "suppress": self.family == "whisper",
            "eos_ids": list(self.eos), "steps_per_replay": self.copies,
            "step": f"{self.copies} greedy steps per graph replay, each over its own weight copy",
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

    def setup(self, torch, device, seed: int, total: int) -> None:
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
        self.outputs = [self.tokens]

    def attend(self, i: int) -> None:
        from asrback_b200 import step

        step.greedy_step(self.hidden[i], self.weights[i], self.tokens, self.position, self.end,
                         self.finished, self.sum_logprobs, self.generated, self.eos,
                         self.suppress)

    def step(self) -> None:
        for i in range(self.copies):
            self.attend(i)

    def launches_per_step(self) -> int:
        return self.copies

    def refresh(self, t: int) -> None:
        pass

    def host_step_inputs(self, torch, first: int, count: int):
        pairs = []
        for h in self.hidden:
            host = torch.empty(h.shape, dtype=h.dtype, pin_memory=True)
            host.copy_(h.cpu())
            pairs.append((host[None].expand(count, *host.shape), h))
        return pairs

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

        def run():
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

    def cpu_rate(self, seed: int, budget_s: float, threads: int) -> dict:
        from oracle import step as oracle_step

        rng = np.random.default_rng(seed)
        weight = (rng.standard_normal((self.vocab, self.width), dtype=np.float32) * 0.02)
        hidden = rng.standard_normal((threads, 1, self.width), dtype=np.float32)
        suppress = None
        if self.family == "whisper":
            suppress = np.zeros(self.vocab, bool)
            suppress[50364:] = True

        def one(_t, row):
            oracle_step.choose(oracle_step.logits(weight, hidden[row], False, np.float32),
                               suppress)

        done, elapsed = run_cpu(one, list(range(threads)), budget_s, threads)
        return {"value": threads * done / elapsed, "unit": self.unit, "cores": threads,
                "kind": "port",
                "sample": f"{threads * done} rows (logits over {self.vocab} x {self.width} + "
                          f"_choose), float32 numpy oracle, {elapsed:.1f} s"}


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


WORKLOADS = {cls.name: cls for cls in (WhisperDecode, WhisperEncoder, Qwen3Decode, Qwen3Prefill,
                                       Qwen3AudioWindows, WhisperGreedyStep, Qwen3GreedyStep,
                                       WhisperCrossKV, WhisperPrefix)}


# ------------------------------------------------------------------ arms ----

def run_reference(args, rank: int) -> None:
    """The reference arm: rank 0 times the CPU path of the workload."""
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT))
    work = WORKLOADS[args.workload](args.batch)
    threads = os.cpu_count() or 1
    result = work.cpu_rate(SEED, args.cpu_seconds, threads)
    line = {
        "impl": "reference", "metric": work.metric, "value": result["value"], "unit": work.unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": work.units_per_step() / result["value"] * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": work.config(args.gpus), "cpu_baseline": result,
        "e2e": {"value": result["value"], "unit": work.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "reference CPU path = CPU oracle port of the reference's attention in float32 "
                "(the Python reference is not present on the GPU box)",
    }
    print(json.dumps(line), flush=True)


def graph_time_ms(torch, fn, reps: int, replays: int = 4) -> float:
    """Average device time of fn() launched `reps` times back to back from a
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


def measure(args, work, torch, dist, device, rank: int, world: int, steps: int, warmup: int,
            cpu: bool) -> dict:
    """Runs one workload: graph-replayed timed region, per-kernel timing, e2e."""
    from asrback_b200 import attention
    from asrback_b200.transcription import CapturedGraph

    seed = SEED + 1000 * rank
    total = warmup + steps
    work.setup(torch, device, seed, total)
    stream = torch.cuda.current_stream()
    work.refresh(0)
    graph = CapturedGraph(work.step)
    for t in range(warmup):
        work.refresh(t)
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()

    uuid = getattr(torch.cuda.get_device_properties(device), "uuid", None)
    uuid = str(uuid) if uuid else None

    from asrback_b200.replicas import max_over_ranks

    # ---- timed region: device-resident inputs, one graph replay per step ----
    start_ev, end_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(uuid) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.nvtx.range_push("timed")
        start_ev.record(stream)
        for t in range(warmup, total):
            work.refresh(t)
            graph.replay()
        clocks.mark()
        end_ev.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    ms = max_over_ranks(start_ev.elapsed_time(end_ev))
    ms_per_step = ms / steps
    value = work.units_per_step() * world * steps / (ms / 1e3)

    # ---- kernel timing: average launch duration, launched from a graph ----
    kernel = {}
    layers = work.launches_per_step() if work.name != "whisper-decode" else work.layers
    for name, fn, amount in work.kernels(warmup):
        launch_ms = graph_time_ms(torch, lambda i: fn(i % layers), 2 * layers)
        kernel[name] = {"launch_ms": launch_ms, "work_per_launch": amount}

    # ---- e2e: pinned host inputs in, outputs back, every step ----
    e2e_steps = min(steps, 4) if work.name == "whisper-encoder" else steps
    pairs = work.host_step_inputs(torch, warmup, e2e_steps)
    outs = [o for o in work.outputs]
    out_bytes = sum(o.numel() * o.element_size() for o in outs)
    host_out = torch.empty((out_bytes,), dtype=torch.uint8, pin_memory=True)
    in_bytes = sum(dev.numel() * dev.element_size() for _, dev in pairs)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for i in range(e2e_steps):
        for host, dev in pairs:
            dev.copy_(host[i], non_blocking=True)
        graph.replay()
        offset = 0
        for o in outs:
            n = o.numel() * o.element_size()
            host_out[offset:offset + n].copy_(o.reshape(-1).view(torch.uint8), non_blocking=True)
            offset += n
    e_end.record(stream)
    torch.cuda.synchronize()
    e_ms = max_over_ranks(e_start.elapsed_time(e_end))
    e2e = work.units_per_step() * world * e2e_steps / (e_ms / 1e3)

    # ---- the reference's GPU computation on the same tensors, for context:
    # graph-replayed where the reference captures it (decoder steps), eager
    # where it does not (the encoder) ----
    ref_fn = work.torch_reference_step(torch)
    if work.reference_in_graph:
        ref_graph = CapturedGraph(ref_fn)
        ref_fn = ref_graph.replay
    else:
        for _ in range(3):
            ref_fn()
    r_start, r_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    r_start.record(stream)
    for t in range(warmup, total):
        work.refresh(t)
        ref_fn()
    r_end.record(stream)
    torch.cuda.synchronize()
    ref_ms = r_start.elapsed_time(r_end) / steps
    ref_graph = None
    cudnn = None
    if hasattr(work, "torch_cudnn_step"):
        fn = work.torch_cudnn_step(torch)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        r_start.record(stream)
        for _ in range(steps):
            fn()
        r_end.record(stream)
        torch.cuda.synchronize()
        c_ms = r_start.elapsed_time(r_end) / steps
        cudnn = {"ms_per_step": c_ms, "value": work.units_per_step() / (c_ms * 1e-3),
                 "unit": work.unit, "what": "torch SDPA with the cuDNN backend forced, eager"}

    dominant = work.kernels(warmup)[0]
    dom = kernel[dominant[0]]
    peak, peak_kind = peak_for(work.bound)
    if work.bound == "hbm":
        achieved = dom["work_per_launch"] / (dom["launch_ms"] * 1e-3) / 1e9
        unit = "GB/s"
    else:
        achieved = dom["work_per_launch"] / (dom["launch_ms"] * 1e-3) / 1e12
        unit = "TFLOP/s"
    traffic = profiled_traffic(work.profile)
    status = attention.read_status(device)
    result = {
        "metric": work.metric, "value": value, "unit": work.unit, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "config": work.config(world),
        "e2e": {"value": e2e, "unit": work.unit, "h2d_bytes_per_step": in_bytes,
                "d2h_bytes_per_step": out_bytes, "steps": e2e_steps},
        "roofline": {"bound": work.bound, "kernel": dominant[0], "achieved": achieved,
                     "peak": peak, "unit": unit, "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": traffic, "work_per_launch": dom["work_per_launch"],
                     "launch_ms": dom["launch_ms"]},
        "kernels": {
            name: dict(k, rate=(k["work_per_launch"] / (k["launch_ms"] * 1e-3)
                                / (1e9 if work.bound == "hbm" else 1e12)),
                       rate_unit=unit)
            for name, k in kernel.items()},
        "step_rate": {"value": work.step_work(warmup, steps) / steps / (ms_per_step * 1e-3)
                      / (1e9 if work.bound == "hbm" else 1e12), "unit": unit},
        "torch_gpu_reference": {
            "ms_per_step": ref_ms, "value": work.units_per_step() / (ref_ms * 1e-3),
            "unit": work.unit,
            "what": "the reference's attention computation in torch on this GPU (same tensors)"},
        "torch_gpu_cudnn": cudnn,
        "gpu_launches": work.launches_per_step() * steps,
        "clocks": clocks.summary(),
        "device_status": status,
    }
    if cpu and rank == 0 and world == 1:
        result["cpu_baseline"] = work.cpu_rate(SEED, args.cpu_seconds, os.cpu_count() or 1)
    return result


def run_native(args, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    work = WORKLOADS[args.workload](args.batch)
    if args.layers:
        work.layers = args.layers
    line = measure(args, work, torch, dist, device, rank, world, args.steps, args.warmup,
                   cpu=not args.no_cpu_baseline)
    if args.workload == "whisper-decode" and not args.no_extras and args.batch is None:
        # Short runs of the other workloads, for context.
        extras = {}
        for name in ("whisper-encoder", "qwen3-decode", "qwen3-prefill", "qwen3-audio",
                     "whisper-step", "qwen3-step", "whisper-cross-kv", "whisper-prefix"):
            del work
            torch.cuda.empty_cache()
            work = WORKLOADS[name](None)
            r = measure(args, work, torch, dist, device, rank, world, min(args.steps, 16),
                        max(3, min(args.warmup, 5)), cpu=False)
            extras[name] = {k: r[k] for k in ("metric", "value", "unit", "ms_per_step", "e2e",
                                              "roofline", "step_rate", "torch_gpu_reference",
                                              "torch_gpu_cudnn", "clocks", "device_status",
                                              "config")}
        line["other_workloads"] = extras
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
