"""One independent replica per GPU: host-side plumbing.

The hot path shards by request: windows and decoding rows are independent, so
every GPU runs its own replica of the model with its own caches and scheduler
and nothing crosses NVLink on the data path (no collective). What remains on
the host is (a) sending each request to a replica, least-loaded first, and
(b) timing a multi-GPU run as the slowest rank's device time.
"""

from __future__ import annotations

import heapq
import threading

__all__ = ["ReplicaDispatcher", "max_over_ranks"]


class ReplicaDispatcher:
    """Assigns requests to ``replicas`` replicas, each to the one with the least
    outstanding work (ties: lowest index), and tracks completions.
    Thread-safe: request threads submit, worker threads complete."""

    def __init__(self, replicas: int) -> None:
        if replicas <= 0:
            raise ValueError("replicas must be positive")
        self._lock = threading.Lock()
        self._load = [0.0] * replicas
        self._heap = [(0.0, index) for index in range(replicas)]

    @property
    def replicas(self) -> int:
        return len(self._load)

    def load(self, replica: int) -> float:
        with self._lock:
            return self._load[replica]

    def assign(self, cost: float = 1.0) -> int:
        """The replica that takes a request of ``cost`` (e.g. its audio seconds)."""
        if cost < 0:
            raise ValueError("cost must be non-negative")
        with self._lock:
            while True:
                load, index = heapq.heappop(self._heap)
                if load == self._load[index]:  # skip stale heap entries
                    break
            self._load[index] = load + cost
            heapq.heappush(self._heap, (self._load[index], index))
            return index

    def complete(self, replica: int, cost: float = 1.0) -> None:
        """Marks a request of ``cost`` on ``replica`` done."""
        with self._lock:
            load = self._load[replica] - cost
            if load < -1e-9:
                raise ValueError(f"replica {replica} completes more work than it was given")
            self._load[replica] = max(load, 0.0)
            heapq.heappush(self._heap, (self._load[replica], replica))


def max_over_ranks(value: float, device=None) -> float:
    """The largest ``value`` over the ranks of the default process group (the
    value itself without one): a multi-GPU run is as fast as its slowest rank."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) \
            if dist.get_backend() == "nccl" else torch.device("cpu")
    tensor = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(tensor, op=dist.ReduceOp.MAX)
    return float(tensor.item())
