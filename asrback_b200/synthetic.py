"""Seeded synthetic weights and inputs (no checkpoints or datasets are available).

Every parameter is drawn from its own CPU generator seeded by ``(seed, name)``,
so a module gets the same weights whatever else it holds, on any machine with
this torch version: the reference's modules and tensors built by parameter
name alone (``seeded_parameter``) are filled identically.
"""

from __future__ import annotations

import math
import zlib

import torch
from torch import nn

__all__ = ["parameter_seed", "seeded_parameter", "seeded_parameters", "seeded_normal"]


def parameter_seed(seed: int, name: str) -> int:
    return (seed * 1_000_003 + zlib.crc32(name.encode())) % (2**62)


def seeded_normal(shape, seed: int, std: float = 1.0, mean: float = 0.0) -> torch.Tensor:
    """``N(mean, std^2)`` float32 CPU tensor from a generator seeded with ``seed``."""
    generator = torch.Generator().manual_seed(seed)
    return torch.randn(tuple(shape), generator=generator) * std + mean


def seeded_parameter(name: str, shape, seed: int) -> torch.Tensor:
    """The float32 value :func:`seeded_parameters` gives a parameter called
    ``name`` of this shape: biases ``N(0, 0.02)``, 1-d weights (norms)
    ``N(1, 0.1)``, embeddings ``N(0, 0.02)``, other weights ``N(0, 1/fan_in)``."""
    shape = tuple(shape)
    pseed = parameter_seed(seed, name)
    if name.endswith("bias"):
        return seeded_normal(shape, pseed, 0.02)
    if len(shape) == 1:
        return seeded_normal(shape, pseed, 0.1, 1.0)
    if "embed" in name:
        return seeded_normal(shape, pseed, 0.02)
    return seeded_normal(shape, pseed, 1.0 / math.sqrt(math.prod(shape[1:])))


@torch.no_grad()
def seeded_parameters(module: nn.Module, seed: int) -> nn.Module:
    """Fills every parameter of ``module`` with :func:`seeded_parameter` of
    its qualified name."""
    for name, param in module.named_parameters():
        param.copy_(seeded_parameter(name, param.shape, seed).to(param.dtype))
    return module
