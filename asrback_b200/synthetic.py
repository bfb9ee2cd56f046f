"""Seeded synthetic weights and inputs (no checkpoints or datasets are available).

Every parameter is drawn from its own CPU generator seeded by ``(seed, name)``,
so a module gets the same weights whatever else it holds, on any machine with
this torch version: the reference's modules (same parameter names) and these
mirrors can be filled identically.
"""

from __future__ import annotations

import math
import zlib

import torch
from torch import nn

__all__ = ["parameter_seed", "seeded_parameters", "seeded_normal"]


def parameter_seed(seed: int, name: str) -> int:
    return (seed * 1_000_003 + zlib.crc32(name.encode())) % (2**62)


def seeded_normal(shape, seed: int, std: float = 1.0, mean: float = 0.0) -> torch.Tensor:
    """``N(mean, std^2)`` float32 CPU tensor from a generator seeded with ``seed``."""
    generator = torch.Generator().manual_seed(seed)
    return torch.randn(tuple(shape), generator=generator) * std + mean


@torch.no_grad()
def seeded_parameters(module: nn.Module, seed: int) -> nn.Module:
    """Fills ``module``'s parameters: biases ``N(0, 0.02)``, 1-d weights (norms)
    ``N(1, 0.1)``, embeddings ``N(0, 0.02)``, other weights ``N(0, 1/fan_in)``."""
    for name, param in module.named_parameters():
        shape = tuple(param.shape)
        pseed = parameter_seed(seed, name)
        if name.endswith("bias"):
            value = seeded_normal(shape, pseed, 0.02)
        elif len(shape) == 1:
            value = seeded_normal(shape, pseed, 0.1, 1.0)
        elif "embed" in name:
            value = seeded_normal(shape, pseed, 0.02)
        else:
            fan_in = math.prod(shape[1:])
            value = seeded_normal(shape, pseed, 1.0 / math.sqrt(fan_in))
        param.copy_(value.to(param.dtype))
    return module
