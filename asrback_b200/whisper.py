"""Whisper's decoder step and encoder, with the attention on the sm_100a kernels.

The modules mirror the reference's ``src/asrback/models/whisper.py`` interface
on the hot path: the same class names, submodule and parameter names (so a
reference state dict loads unchanged), the same cache layout
(``DecoderCache``, ``(layers, batch, heads, length, head_dim)``,
``whisper.py:156-196``) and the same call signatures
(``decode(tokens, positions, cache)``, ``set_encoder_output``, ``logits``).
What differs is what runs: the fixed-shape step's self-attention (key/value
write plus masked attention, ``whisper.py:222-237``) is one kernel that reads
only each row's written positions, the cross-attention (``:239-240``) another,
and the encoder's attention (``:108-110``) a third. The eager prompt pass
(``decode(tokens, positions[:P], cache, length=P)``, used by the prefill and
by language detection) writes its keys/values with ``index_copy_`` as the
reference does (``whisper.py:229-233``) and runs causal self-attention and
cross-attention for all P tokens of each window on the same kernel, one
query row per (window, token). Linear layers, norms and embeddings stay
torch (cuBLAS), as in the reference.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from . import attention as ops

__all__ = [
    "MultiHeadAttention",
    "EncoderLayer",
    "WhisperEncoder",
    "DecoderCache",
    "DecoderLayer",
    "WhisperDecoder",
    "WhisperForConditionalGeneration",
    "tiny_config",
    "large_v3_turbo_config",
]


def tiny_config(vocab_size: int = 51865) -> dict:
    """Whisper-tiny dimensions (the CPU fp32 anchor configuration)."""
    return dict(d_model=384, encoder_attention_heads=6, decoder_attention_heads=6,
                encoder_layers=4, decoder_layers=4, encoder_ffn_dim=1536, decoder_ffn_dim=1536,
                num_mel_bins=80, max_source_positions=1500, max_target_positions=448,
                vocab_size=vocab_size)


def large_v3_turbo_config() -> dict:
    """Whisper large-v3-turbo dimensions (32 encoder / 4 decoder layers)."""
    return dict(d_model=1280, encoder_attention_heads=20, decoder_attention_heads=20,
                encoder_layers=32, decoder_layers=4, encoder_ffn_dim=5120, decoder_ffn_dim=5120,
                num_mel_bins=128, max_source_positions=1500, max_target_positions=448,
                vocab_size=51866)


class MultiHeadAttention(nn.Module):
    """Projections of ``whisper.py:73-91`` (``k_proj`` has no bias)."""

    def __init__(self, width: int, heads: int) -> None:
        super().__init__()
        if width % heads:
            raise ValueError(f"d_model ({width}) must be divisible by heads ({heads})")
        self.heads = heads
        self.head_dim = width // heads
        self.k_proj = nn.Linear(width, width, bias=False)
        self.v_proj = nn.Linear(width, width)
        self.q_proj = nn.Linear(width, width)
        self.out_proj = nn.Linear(width, width)

    def _split_heads(self, x: Tensor) -> Tensor:
        batch, length, width = x.shape
        return x.view(batch, length, self.heads, width // self.heads).transpose(1, 2)

    def project_key_value(self, x: Tensor) -> tuple[Tensor, Tensor]:
        """``(batch, heads, length, head_dim)`` views of the key/value projections."""
        return self._split_heads(self.k_proj(x)), self._split_heads(self.v_proj(x))

    def forward(self, x: Tensor) -> Tensor:
        """Unmasked self-attention (the encoder's), on the encoder kernel."""
        query = self._split_heads(self.q_proj(x))
        key, value = self.project_key_value(x)
        return self.out_proj(ops.whisper_encoder_attention(query, key, value))

    def step_self(self, x: Tensor, key_cache: Tensor, value_cache: Tensor,
                  positions: Tensor) -> Tensor:
        """One decoder step of self-attention: ``x`` ``(B, 1, W)``; the row's
        key/value go into the caches at ``positions`` and it attends to keys
        ``0..positions[b]``."""
        query = self._split_heads(self.q_proj(x))
        key, value = self.project_key_value(x)
        out = ops.whisper_self_attention_step(query, key, value, key_cache, value_cache, positions)
        return self.out_proj(out)

    def step_cross(self, x: Tensor, key_cache: Tensor, value_cache: Tensor) -> Tensor:
        """One decoder step of cross-attention over the window's encoder keys."""
        query = self._split_heads(self.q_proj(x))
        return self.out_proj(ops.whisper_cross_attention_step(query, key_cache, value_cache))

    def prefix_self(self, x: Tensor, key_cache: Tensor, value_cache: Tensor,
                    positions: Tensor) -> Tensor:
        """Self-attention of a prompt pass, ``x`` ``(B, P, W)``: the tokens'
        keys/values go into the caches at ``positions`` (``index_copy_``,
        ``whisper.py:231-232``) and token ``t`` attends causally to keys
        ``0..t`` of the first P positions (``is_causal`` over
        ``cache[:, :, :P]``)."""
        query = self._split_heads(self.q_proj(x))
        key, value = self.project_key_value(x)
        key_cache.index_copy_(2, positions, key)
        value_cache.index_copy_(2, positions, value)
        tokens = x.shape[1]
        out = ops.whisper_self_attention_prefix(query, key_cache[:, :, :tokens],
                                                value_cache[:, :, :tokens])
        return self.out_proj(out)

    def prefix_cross(self, x: Tensor, key_cache: Tensor, value_cache: Tensor) -> Tensor:
        """Cross-attention of a prompt pass over the window's encoder keys."""
        query = self._split_heads(self.q_proj(x))
        return self.out_proj(ops.whisper_cross_attention_prefix(query, key_cache, value_cache))


class EncoderLayer(nn.Module):
    def __init__(self, config: dict) -> None:
        super().__init__()
        width = config["d_model"]
        self.self_attn = MultiHeadAttention(width, config["encoder_attention_heads"])
        self.self_attn_layer_norm = nn.LayerNorm(width)
        self.fc1 = nn.Linear(width, config["encoder_ffn_dim"])
        self.fc2 = nn.Linear(config["encoder_ffn_dim"], width)
        self.final_layer_norm = nn.LayerNorm(width)

    def forward(self, x: Tensor) -> Tensor:
        x = x + self.self_attn(self.self_attn_layer_norm(x))
        return x + self.fc2(F.gelu(self.fc1(self.final_layer_norm(x))))


class WhisperEncoder(nn.Module):
    """Conv stem, learned positions, pre-norm layers (``whisper.py:128-153``)."""

    def __init__(self, config: dict) -> None:
        super().__init__()
        width = config["d_model"]
        self.conv1 = nn.Conv1d(config["num_mel_bins"], width, 3, padding=1)
        self.conv2 = nn.Conv1d(width, width, 3, stride=2, padding=1)
        self.embed_positions = nn.Embedding(config["max_source_positions"], width)
        self.layers = nn.ModuleList(EncoderLayer(config) for _ in range(config["encoder_layers"]))
        self.layer_norm = nn.LayerNorm(width)

    def forward(self, mel: Tensor) -> Tensor:
        x = F.gelu(self.conv1(mel))
        x = F.gelu(self.conv2(x)).transpose(1, 2).contiguous()
        if x.shape[1] != self.embed_positions.num_embeddings:
            raise ValueError(
                f"expected {self.embed_positions.num_embeddings * 2} mel frames, got {mel.shape[-1]}"
            )
        x = x + self.embed_positions.weight
        for layer in self.layers:
            x = layer(x)
        return self.layer_norm(x)


@dataclass
class DecoderCache:
    """Preallocated keys and values, ``(layers, batch, heads, length, head_dim)``.

    Self-attention entries are written in place at each step's positions, so the
    tensors keep fixed addresses (CUDA graphs need them)."""

    self_keys: Tensor
    self_values: Tensor
    cross_keys: Tensor
    cross_values: Tensor

    @property
    def batch_size(self) -> int:
        return self.self_keys.shape[1]

    def narrow(self, batch_size: int, length: int | None = None) -> "DecoderCache":
        """The first ``batch_size`` rows (and self-attention positions), same storage."""
        return self.rows(0, batch_size, length)

    def rows(self, start: int, stop: int, length: int | None = None) -> "DecoderCache":
        return DecoderCache(
            self.self_keys[:, start:stop, :, :length],
            self.self_values[:, start:stop, :, :length],
            self.cross_keys[:, start:stop],
            self.cross_values[:, start:stop],
        )

    def copy_rows(self, source: "DecoderCache", rows: Tensor, length: int) -> None:
        """Copies every row of ``source`` (its first ``length`` self positions)
        into rows ``rows`` of this cache."""
        pairs = (
            (self.self_keys[:, :, :, :length], source.self_keys[:, :, :, :length]),
            (self.self_values[:, :, :, :length], source.self_values[:, :, :, :length]),
            (self.cross_keys, source.cross_keys),
            (self.cross_values, source.cross_values),
        )
        for target, values in pairs:
            target.index_copy_(1, rows, values)


class DecoderLayer(nn.Module):
    def __init__(self, config: dict) -> None:
        super().__init__()
        width = config["d_model"]
        heads = config["decoder_attention_heads"]
        self.self_attn = MultiHeadAttention(width, heads)
        self.self_attn_layer_norm = nn.LayerNorm(width)
        self.encoder_attn = MultiHeadAttention(width, heads)
        self.encoder_attn_layer_norm = nn.LayerNorm(width)
        self.fc1 = nn.Linear(width, config["decoder_ffn_dim"])
        self.fc2 = nn.Linear(config["decoder_ffn_dim"], width)
        self.final_layer_norm = nn.LayerNorm(width)

    def forward(self, x: Tensor, cache: tuple[Tensor, Tensor, Tensor, Tensor],
                positions: Tensor, length: int | None = None) -> Tensor:
        """The step (``length`` None): one token per row (``x`` ``(B, 1, W)``)
        at ``positions`` ``(B,)``. The prompt pass: P tokens per row at
        ``positions`` ``(P,)`` with ``length == P``."""
        self_keys, self_values, cross_keys, cross_values = cache
        if length is None:
            x = x + self.self_attn.step_self(self.self_attn_layer_norm(x), self_keys,
                                             self_values, positions)
            x = x + self.encoder_attn.step_cross(self.encoder_attn_layer_norm(x), cross_keys,
                                                 cross_values)
        else:
            if length != x.shape[1]:
                raise NotImplementedError(
                    f"asrback_b200 runs the eager pass with length == tokens (the form the "
                    f"prompt pass and language detection use); got length {length} for "
                    f"{x.shape[1]} tokens"
                )
            x = x + self.self_attn.prefix_self(self.self_attn_layer_norm(x), self_keys,
                                               self_values, positions)
            x = x + self.encoder_attn.prefix_cross(self.encoder_attn_layer_norm(x), cross_keys,
                                                   cross_values)
        return x + self.fc2(F.gelu(self.fc1(self.final_layer_norm(x))))


class WhisperDecoder(nn.Module):
    def __init__(self, config: dict) -> None:
        super().__init__()
        width = config["d_model"]
        self.embed_tokens = nn.Embedding(config["vocab_size"], width)
        self.embed_positions = nn.Embedding(config["max_target_positions"], width)
        self.layers = nn.ModuleList(DecoderLayer(config) for _ in range(config["decoder_layers"]))
        self.layer_norm = nn.LayerNorm(width)

    def forward(self, tokens: Tensor, positions: Tensor, cache: DecoderCache,
                length: int | None = None) -> Tensor:
        """Hidden states for ``tokens`` ``(B, 1)`` at ``positions`` ``(B,)``
        (the step; keys past each row's position are never read, so no mask is
        built), or, with ``length`` given, for ``tokens`` ``(B, P)`` at the
        shared ``positions`` ``(P,)`` (the prompt pass, ``whisper.py:265-266``)."""
        if length is None:
            x = self.embed_tokens(tokens) + self.embed_positions(positions)[:, None]
        else:
            x = self.embed_tokens(tokens) + self.embed_positions(positions)
        for index, layer in enumerate(self.layers):
            layer_cache = (cache.self_keys[index], cache.self_values[index],
                           cache.cross_keys[index], cache.cross_values[index])
            x = layer(x, layer_cache, positions, length)
        return self.layer_norm(x)


class WhisperModel(nn.Module):
    def __init__(self, config: dict, encoder: bool = True) -> None:
        super().__init__()
        if encoder:
            self.encoder = WhisperEncoder(config)
        self.decoder = WhisperDecoder(config)


class WhisperForConditionalGeneration(nn.Module):
    """``whisper.py:280-342``: the network with the cache and logits helpers.
    ``encoder=False`` builds the decoder alone (the decode benchmarks feed
    encoder states directly)."""

    def __init__(self, config: dict, encoder: bool = True) -> None:
        super().__init__()
        self.config = config
        self.model = WhisperModel(config, encoder)

    def allocate_cache(self, batch_size: int) -> DecoderCache:
        config = self.config
        weight = self.model.decoder.embed_tokens.weight
        heads = config["decoder_attention_heads"]
        head_dim = config["d_model"] // heads

        def zeros(length: int) -> Tensor:
            shape = (config["decoder_layers"], batch_size, heads, length, head_dim)
            return torch.zeros(shape, dtype=weight.dtype, device=weight.device)

        target, source = config["max_target_positions"], config["max_source_positions"]
        return DecoderCache(zeros(target), zeros(target), zeros(source), zeros(source))

    def set_encoder_output(self, cache: DecoderCache, encoder_output: Tensor) -> None:
        """Fills the first ``len(encoder_output)`` rows' cross keys/values
        (``whisper.py:313-319``): each layer's projections are written into
        the cache by one kernel."""
        batch_size = encoder_output.shape[0]
        for index, layer in enumerate(self.model.decoder.layers):
            attn = layer.encoder_attn
            ops.whisper_cross_kv_projection(
                encoder_output, attn.k_proj.weight, attn.v_proj.weight, attn.v_proj.bias,
                cache.cross_keys[index, :batch_size], cache.cross_values[index, :batch_size])

    def decode(self, tokens: Tensor, positions: Tensor, cache: DecoderCache,
               length: int | None = None) -> Tensor:
        return self.model.decoder(tokens, positions, cache, length)

    def logits(self, hidden: Tensor) -> Tensor:
        weight = self.model.decoder.embed_tokens.weight
        rows = hidden.flatten(0, -2)
        return (weight @ rows.T).T.unflatten(0, hidden.shape[:-1])
