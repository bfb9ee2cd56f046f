"""Qwen3-ASR's text decoder step with attention on the sm_100a kernel.

Mirrors the reference's ``src/asrback/models/qwen3_asr.py`` interface on the hot
path: ``RMSNorm`` (``:316-323``), ``KVCache`` (``(layers, batch, length,
kv_heads, head_dim)``, ``:333-347``), ``TextAttention`` with the fused
``qkv_proj`` (``:350-364``), ``TextMLP``, ``DecoderLayer`` and
``TextModel.step`` (``:494-524``), with the same module and parameter names.
``TextAttention.step`` hands ``qkv_proj``'s output to one kernel that does the
per-head q/k RMSNorm, the RoPE rotation, the cache write and the grouped-query
attention over each row's written keys (the reference does these in
``_project``, ``:366-372``, and ``step``, ``:392-432``). The packed causal
prompt prefill (``TextAttention.prefill``, ``:374-390``; ``TextModel.prefill``,
``:471-490``) runs ``attend`` (``:152-181``) on the varlen kernel, with
``Segments`` holding the packed prompts' starts (``:122-149``).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import attention as ops

__all__ = [
    "CACHE_LENGTH",
    "Segments",
    "attend",
    "rotate",
    "RMSNorm",
    "KVCache",
    "TextAttention",
    "TextMLP",
    "DecoderLayer",
    "TextModel",
    "rope_tables",
    "text_config_1_7b",
    "text_config_0_6b",
]

# Positions per cache row (prompt plus generated tokens), as in the reference.
CACHE_LENGTH = 1024


def text_config_1_7b(vocab_size: int = 151936, intermediate_size: int = 6144) -> dict:
    """Qwen3-1.7B-style text decoder: 28 layers, hidden 2048, 16 q / 8 kv heads."""
    return dict(hidden_size=2048, num_hidden_layers=28, num_attention_heads=16,
                num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                intermediate_size=intermediate_size, vocab_size=vocab_size)


def text_config_0_6b(vocab_size: int = 151936, intermediate_size: int = 3072) -> dict:
    """Qwen3-0.6B-style text decoder: 28 layers, hidden 1024, 16 q / 8 kv heads."""
    return dict(hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, rope_theta=1e6,
                intermediate_size=intermediate_size, vocab_size=vocab_size)


def rope_tables(theta: float, head_dim: int, length: int = CACHE_LENGTH,
                device=None, dtype=torch.float32) -> tuple[Tensor, Tensor]:
    """``(length, head_dim)`` cos/sin tables: fp32 angles ``p * theta^(-2i/D)``
    repeated over both halves, then cast (``qwen3_asr.py:795-803``)."""
    inverse = 1.0 / (theta ** (torch.arange(0, head_dim, 2).float() / head_dim))
    angles = torch.arange(length).float()[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos().to(device, dtype), angles.sin().to(device, dtype)


class RMSNorm(nn.Module):
    def __init__(self, width: int, eps: float) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        return F.rms_norm(x, self.weight.shape, self.weight, self.eps)


@dataclass
class KVCache:
    """Preallocated keys and values, ``(layers, batch, length, kv_heads, head_dim)``."""

    keys: Tensor
    values: Tensor

    @classmethod
    def allocate(cls, config: dict, batch_size: int, length: int = CACHE_LENGTH,
                 device=None, dtype=torch.bfloat16) -> "KVCache":
        shape = (config["num_hidden_layers"], batch_size, length,
                 config["num_key_value_heads"], config["head_dim"])
        return cls(torch.zeros(shape, dtype=dtype, device=device),
                   torch.zeros(shape, dtype=dtype, device=device))

    def narrow(self, batch_size: int, length: int) -> "KVCache":
        return KVCache(self.keys[:, :batch_size, :length], self.values[:, :batch_size, :length])


@dataclass
class Segments:
    """Boundaries of the sequences laid out back to back in a packed tensor:
    ``starts`` ``(sequences + 1,)`` int32 cumulative lengths on the device and
    the longest length (the reference's ``Segments``, ``qwen3_asr.py:122-149``)."""

    starts: Tensor
    longest: int

    @classmethod
    def from_lengths(cls, lengths: list[int], device: torch.device) -> "Segments":
        sizes = torch.tensor(lengths, dtype=torch.int64)
        starts = F.pad(sizes.cumsum(0), (1, 0)).to(torch.int32)
        return cls(starts.to(device), max(lengths))


def attend(q: Tensor, k: Tensor, v: Tensor, segments: Segments, causal: bool) -> Tensor:
    """Attention within each segment of packed ``(tokens, heads, head_dim)``
    tensors; ``k`` and ``v`` may have fewer heads than ``q`` (grouped-query)."""
    return ops.varlen_attention(q, k, v, segments.starts, segments.longest, causal)


def rotate(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotary embedding (rotate-half) of ``(tokens, heads, head_dim)`` with
    ``cos``/``sin`` ``(tokens, head_dim)`` (``qwen3_asr.py:326-330``)."""
    half = x.shape[-1] // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None] + rotated * sin[:, None]


class TextAttention(nn.Module):
    def __init__(self, config: dict) -> None:
        super().__init__()
        width = config["hidden_size"]
        self.head_dim = config["head_dim"]
        self.heads = config["num_attention_heads"]
        self.kv_heads = config["num_key_value_heads"]
        self.sizes = [size * self.head_dim for size in (self.heads, self.kv_heads, self.kv_heads)]
        self.qkv_proj = nn.Linear(width, sum(self.sizes), bias=False)
        self.o_proj = nn.Linear(self.heads * self.head_dim, width, bias=False)
        self.q_norm = RMSNorm(self.head_dim, config["rms_norm_eps"])
        self.k_norm = RMSNorm(self.head_dim, config["rms_norm_eps"])

    def step(self, x: Tensor, keys: Tensor, values: Tensor, positions: Tensor, cos: Tensor,
             sin: Tensor) -> Tensor:
        """One token per row (``x`` ``(B, W)``) at ``positions``; ``keys``/``values``
        are this layer's ``(B, L, kv_heads, D)`` cache view; ``cos``/``sin`` the
        full tables (the kernel gathers each row's)."""
        out = ops.qwen3_attention_step(
            self.qkv_proj(x), self.q_norm.weight, self.k_norm.weight, self.q_norm.eps,
            cos, sin, positions, keys, values, self.heads, self.kv_heads,
        )
        return self.o_proj(out)

    def _project(self, x: Tensor, cos: Tensor, sin: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        """``(tokens, heads, head_dim)`` queries, keys and values for
        ``(tokens, width)``: q/k RMSNorm, then RoPE with each token's
        ``cos``/``sin`` rows."""
        shape = (len(x), -1, self.head_dim)
        q, k, v = self.qkv_proj(x).split(self.sizes, dim=-1)
        q = rotate(self.q_norm(q.reshape(shape)), cos, sin)
        k = rotate(self.k_norm(k.reshape(shape)), cos, sin)
        return q, k, v.reshape(shape)

    def prefill(self, x: Tensor, keys: Tensor, values: Tensor, rows: Tensor, positions: Tensor,
                segments: Segments, cos: Tensor, sin: Tensor) -> Tensor:
        """Causal attention within each packed prompt; every token's key and
        value go to its row and position of the cache."""
        q, k, v = self._project(x, cos, sin)
        keys[rows, positions] = k
        values[rows, positions] = v
        return self.o_proj(attend(q, k, v, segments, causal=True).flatten(1))


class TextMLP(nn.Module):
    def __init__(self, config: dict) -> None:
        super().__init__()
        width, hidden = config["hidden_size"], config["intermediate_size"]
        self.gate_up_proj = nn.Linear(width, 2 * hidden, bias=False)
        self.down_proj = nn.Linear(hidden, width, bias=False)

    def forward(self, x: Tensor) -> Tensor:
        gate, up = self.gate_up_proj(x).chunk(2, dim=-1)
        return self.down_proj(F.silu(gate) * up)


class DecoderLayer(nn.Module):
    def __init__(self, config: dict) -> None:
        super().__init__()
        self.input_layernorm = RMSNorm(config["hidden_size"], config["rms_norm_eps"])
        self.self_attn = TextAttention(config)
        self.post_attention_layernorm = RMSNorm(config["hidden_size"], config["rms_norm_eps"])
        self.mlp = TextMLP(config)

    def forward(self, x: Tensor, keys: Tensor, values: Tensor, positions: Tensor, cos: Tensor,
                sin: Tensor) -> Tensor:
        x = x + self.self_attn.step(self.input_layernorm(x), keys, values, positions, cos, sin)
        return x + self.mlp(self.post_attention_layernorm(x))

    def prefill(self, x: Tensor, keys: Tensor, values: Tensor, rows: Tensor, positions: Tensor,
                segments: Segments, cos: Tensor, sin: Tensor) -> Tensor:
        x = x + self.self_attn.prefill(self.input_layernorm(x), keys, values, rows, positions,
                                       segments, cos, sin)
        return x + self.mlp(self.post_attention_layernorm(x))


class TextModel(nn.Module):
    def __init__(self, config: dict) -> None:
        super().__init__()
        self.embed_tokens = nn.Embedding(config["vocab_size"], config["hidden_size"])
        self.layers = nn.ModuleList(DecoderLayer(config) for _ in range(config["num_hidden_layers"]))
        self.norm = RMSNorm(config["hidden_size"], config["rms_norm_eps"])

    def step(self, tokens: Tensor, positions: Tensor, cache: KVCache, cos: Tensor,
             sin: Tensor) -> Tensor:
        """Hidden states for one token per row (``tokens``, ``positions``:
        ``(B,)``) over a fixed-shape cache view; each row reads only its keys
        up to its position, so no mask and no varlen triple is built."""
        return self.step_embeddings(self.embed_tokens(tokens), positions, cache, cos, sin)

    def step_embeddings(self, x: Tensor, positions: Tensor, cache: KVCache, cos: Tensor,
                        sin: Tensor) -> Tensor:
        """As :meth:`step`, from input embeddings ``(B, W)``."""
        for index, layer in enumerate(self.layers):
            x = layer(x, cache.keys[index], cache.values[index], positions, cos, sin)
        return self.norm(x)

    def prefill(self, x: Tensor, cache: KVCache, rows: Tensor, positions: Tensor,
                segments: Segments, cos: Tensor, sin: Tensor) -> Tensor:
        """Hidden states of packed prompts ``x`` ``(tokens, width)``; token ``i``
        is at ``positions[i]`` of cache row ``rows[i]``; ``cos``/``sin`` are the
        tokens' rows of the tables."""
        for index, layer in enumerate(self.layers):
            x = layer.prefill(x, cache.keys[index], cache.values[index], rows, positions, segments,
                              cos, sin)
        return self.norm(x)
