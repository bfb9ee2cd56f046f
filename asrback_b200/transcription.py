"""CUDA graph capture of a fixed-address step, as the reference's engine does it.

``CapturedGraph`` keeps the contract of ``src/asrback/transcription.py:158-179``:
three warm-up calls on a side stream (so lazy set-up, here the kernels' shared
memory attributes and the split-KV workspace, stays out of the graph), then one
capture with ``capture_error_mode="thread_local"``. The attention kernels read
row positions on the device and allocate nothing during the step, so a graph
captured at a (batch bucket, cache view) pair replays for any positions.
"""

from __future__ import annotations

from typing import Callable

import torch

__all__ = ["CapturedGraph"]


class CapturedGraph:
    """A function of fixed-address tensors captured once as a CUDA graph.
    Graphs that never replay concurrently can share a memory ``pool``."""

    def __init__(self, function: Callable[[], None], pool=None, warmup: int = 3) -> None:
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                function()
        torch.cuda.current_stream().wait_stream(stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, pool=pool, capture_error_mode="thread_local"):
            function()

    def replay(self) -> None:
        self.graph.replay()
