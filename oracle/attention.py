"""CPU oracle for asrback's attention hot path (numpy, float64 arithmetic).

TEST INFRASTRUCTURE ONLY. This module is the checker the parity tests, the
``smoke()`` entry and the CPU-baseline leg of ``bench.py`` compare the CUDA
kernels against. The product path (``asrback_b200``) never imports it and has
no CPU fallback.

What it restates. The reference keeps its attention arithmetic inside torch
(``F.scaled_dot_product_attention``, torch 2.14.1 pinned at ``uv.lock:2580``;
2.11.0 is what runs here). The published algorithm of that call is
``softmax(q @ k^T * scale + mask) @ v`` with ``scale = 1/sqrt(head_dim)`` and a
boolean mask that removes the keys where it is False. Every function below
restates that algorithm at one of the reference's call sites, in float64, and
names the reference lines it follows (paths relative to the asrback project).

Pinning. ``tests/golden/make_golden.py`` ran the reference's own modules (on
CPU, fp32 and bf16) and stored their inputs and outputs under ``tests/golden``;
``tests/test_oracle_golden.py`` checks every function here against them.

bf16. Where the reference runs in bfloat16, torch computes each elementwise op
in fp32 and rounds its result to bf16 (checked against torch for
``F.rms_norm``, which rounds once after ``x * rsqrt(mean(x^2) + eps) * w``, and
for the rotate-half products and sum). ``bf16=True`` replays those roundings.
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_round",
    "sdpa",
    "whisper_self_attention_step",
    "whisper_cross_attention",
    "whisper_self_attention_prefix",
    "whisper_cross_attention_prefix",
    "encoder_attention",
    "rope_tables",
    "rms_norm",
    "rotate",
    "qwen3_project",
    "qwen3_decode_attention",
    "varlen_attention",
    "cross_kv_projection",
]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round to the nearest bfloat16 (ties to even), returned as float32."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = np.isnan(x)
    lsb = (bits >> 16) & 1
    rounded = ((bits.astype(np.uint64) + 0x7FFF + lsb) >> 16 << 16).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    out[nan] = np.nan
    return out


def sdpa(q, k, v, mask=None, scale=None, compute=np.float64) -> np.ndarray:
    """``softmax(q k^T * scale, masked) v`` over the last two axes.

    ``q`` ``(..., Lq, D)``, ``k``/``v`` ``(..., Lk, D)``; ``mask`` is boolean and
    broadcasts to ``(..., Lq, Lk)``, True where a key is attended. Restates the
    call at ``src/asrback/models/whisper.py:102-104`` (torch's math backend).
    ``compute`` is the arithmetic type (float64 to check; float32, the
    reference's CPU dtype, when the oracle is timed as the CPU baseline).
    """
    q = np.asarray(q, dtype=compute)
    k = np.asarray(k, dtype=compute)
    v = np.asarray(v, dtype=compute)
    if scale is None:
        scale = 1.0 / np.sqrt(q.shape[-1])
    scores = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    if mask is not None:
        scores = np.where(mask, scores, -np.inf)
    top = scores.max(axis=-1, keepdims=True)
    weights = np.exp(scores - top)
    weights /= weights.sum(axis=-1, keepdims=True)
    return np.matmul(weights, v)


def whisper_self_attention_step(query, key, value, key_cache, value_cache, positions,
                                compute=np.float64, copy=True):
    """One decoder step of Whisper's masked self-attention.

    Follows ``DecoderLayer.forward``'s fixed-shape branch
    (``src/asrback/models/whisper.py:222-228``: ``scatter_`` of each row's key
    and value at its own position) and the step mask built in
    ``WhisperDecoder.forward`` (``whisper.py:262-264``: key ``j`` is attended by
    row ``b`` iff ``j <= positions[b]``), then ``attend`` (``whisper.py:93-106``).

    ``query``/``key``/``value`` ``(B, H, D)``; caches ``(B, H, L, D)``;
    ``positions`` ``(B,)``. Returns ``(out (B, H, D) float64, key_cache,
    value_cache)``, the caches as updated copies in their own dtype (with
    ``copy=False`` the given arrays are written in place, as ``scatter_`` does).
    """
    if copy:
        key_cache = np.array(key_cache, copy=True)
        value_cache = np.array(value_cache, copy=True)
    positions = np.asarray(positions, dtype=np.int64)
    batch, _, length, _ = key_cache.shape
    rows = np.arange(batch)
    key_cache[rows, :, positions] = key
    value_cache[rows, :, positions] = value
    mask = (np.arange(length)[None, :] <= positions[:, None])[:, None, None, :]
    out = sdpa(np.asarray(query)[:, :, None, :], key_cache, value_cache, mask, compute=compute)
    return out[:, :, 0, :], key_cache, value_cache


def whisper_cross_attention(query, key_cache, value_cache, compute=np.float64) -> np.ndarray:
    """Unmasked attention of one query per row over the window's encoder keys
    (``whisper.py:239-240`` calling ``attend`` without a mask).

    ``query`` ``(B, H, D)``, caches ``(B, H, S, D)`` → ``(B, H, D)``.
    """
    out = sdpa(np.asarray(query)[:, :, None, :], key_cache, value_cache, compute=compute)
    return out[:, :, 0, :]


def whisper_self_attention_prefix(query, key, value, key_cache, value_cache, positions, length,
                                  compute=np.float64):
    """Self-attention of the eager branch of ``DecoderLayer.forward``
    (``whisper.py:228-236``): ``index_copy_`` of the P tokens' keys/values at
    the shared ``positions``, the cache cut to its first ``length`` positions,
    then ``attend`` with ``is_causal = P > 1``, which torch aligns to the top
    left (query ``t`` attends keys ``0..t``).

    ``query``/``key``/``value`` ``(B, H, P, D)``; caches ``(B, H, L, D)``;
    ``positions`` ``(P,)``. Returns ``(out (B, H, P, D) float64, key_cache,
    value_cache)`` with the caches as updated copies.
    """
    key_cache = np.array(key_cache, copy=True)
    value_cache = np.array(value_cache, copy=True)
    positions = np.asarray(positions, dtype=np.int64)
    key_cache[:, :, positions] = key
    value_cache[:, :, positions] = value
    tokens = np.asarray(query).shape[2]
    mask = None
    if tokens > 1:
        mask = np.arange(length)[None, :] <= np.arange(tokens)[:, None]
    out = sdpa(query, key_cache[:, :, :length], value_cache[:, :, :length], mask, compute=compute)
    return out, key_cache, value_cache


def whisper_cross_attention_prefix(query, key_cache, value_cache, compute=np.float64) -> np.ndarray:
    """Cross-attention of the eager branch (``whisper.py:239-240``): every one
    of a window's P query tokens over all its encoder keys. ``query``
    ``(B, H, P, D)``, caches ``(B, H, S, D)`` -> ``(B, H, P, D)``."""
    return sdpa(query, key_cache, value_cache, compute=compute)


def encoder_attention(q, k, v) -> np.ndarray:
    """Non-causal self-attention of the Whisper encoder
    (``MultiHeadAttention.forward``, ``whisper.py:108-110``). ``(B, H, S, D)``."""
    return sdpa(q, k, v)


def rope_tables(theta: float, head_dim: int, length: int, bf16: bool = False):
    """The RoPE cos/sin tables ``(length, head_dim)`` of
    ``Qwen3ASRTranscriber.__init__`` (``qwen3_asr.py:795-803``): fp32 angles
    ``position * theta^(-2i/head_dim)`` repeated for both halves."""
    inverse = 1.0 / (
        np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim))
    ).astype(np.float32)
    angles = np.arange(length, dtype=np.float32)[:, None] * inverse[None, :].astype(np.float32)
    angles = np.concatenate((angles, angles), axis=-1).astype(np.float32)
    cos, sin = np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)
    if bf16:
        cos, sin = bf16_round(cos), bf16_round(sin)
    return cos, sin


def rms_norm(x, weight, eps: float, bf16: bool = False) -> np.ndarray:
    """``F.rms_norm`` over the last axis (``RMSNorm``, ``qwen3_asr.py:316-323``)."""
    x = np.asarray(x, dtype=np.float32)
    mean = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    out = x * (1.0 / np.sqrt(mean + eps)) * np.asarray(weight, dtype=np.float64)
    out = out.astype(np.float32)
    return bf16_round(out) if bf16 else out


def rotate(x, cos, sin, bf16: bool = False) -> np.ndarray:
    """Rotate-half RoPE (``rotate``, ``qwen3_asr.py:326-330``). ``x``
    ``(..., heads, D)``, ``cos``/``sin`` ``(..., D)``."""
    x = np.asarray(x, dtype=np.float32)
    first, second = np.split(x, 2, axis=-1)
    rotated = np.concatenate((-second, first), axis=-1)
    a = x * np.asarray(cos, dtype=np.float32)[..., None, :]
    b = rotated * np.asarray(sin, dtype=np.float32)[..., None, :]
    if bf16:
        return bf16_round(bf16_round(a) + bf16_round(b))
    return (a.astype(np.float64) + b).astype(np.float32)


def qwen3_project(qkv, heads, kv_heads, head_dim, q_norm_weight, k_norm_weight, eps,
                  cos_rows, sin_rows, bf16: bool = False):
    """``TextAttention._project`` after ``qkv_proj`` (``qwen3_asr.py:366-372``):
    split ``(B, (heads + 2 kv_heads) head_dim)`` into q/k/v, RMSNorm q and k per
    head, rotate both with the rows' cos/sin. Returns q ``(B, heads, D)``,
    k and v ``(B, kv_heads, D)``, as float32 (bf16-valued when ``bf16``)."""
    qkv = np.asarray(qkv, dtype=np.float32)
    batch = qkv.shape[0]
    q_size, kv_size = heads * head_dim, kv_heads * head_dim
    q = qkv[:, :q_size].reshape(batch, heads, head_dim)
    k = qkv[:, q_size:q_size + kv_size].reshape(batch, kv_heads, head_dim)
    v = qkv[:, q_size + kv_size:q_size + 2 * kv_size].reshape(batch, kv_heads, head_dim)
    q = rotate(rms_norm(q, q_norm_weight, eps, bf16), cos_rows, sin_rows, bf16)
    k = rotate(rms_norm(k, k_norm_weight, eps, bf16), cos_rows, sin_rows, bf16)
    return q, k, v.copy()


def qwen3_decode_attention(qkv, q_norm_weight, k_norm_weight, eps, cos, sin, positions,
                           key_cache, value_cache, heads, kv_heads, bf16: bool = False):
    """One Qwen3 decoder step of attention, between ``qkv_proj`` and ``o_proj``.

    Follows ``TextModel.step`` (``qwen3_asr.py:504-515``: ``cos``/``sin`` rows
    gathered at ``positions``; key ``j`` attended iff ``j <= positions[b]``) and
    ``TextAttention.step`` (``qwen3_asr.py:392-432``: project, write each row's
    key and value at its position, then the query heads sharing a key/value
    head attend as one group, q head ``h`` → kv head ``h // (heads/kv_heads)``).

    ``qkv`` ``(B, (heads + 2 kv_heads) D)``; ``cos``/``sin`` full tables
    ``(L_table, D)``; caches ``(B, L, kv_heads, D)``. Returns ``(out (B, heads*D)
    float64, key_cache, value_cache)`` with the caches as updated copies.
    """
    key_cache = np.array(key_cache, copy=True)
    value_cache = np.array(value_cache, copy=True)
    positions = np.asarray(positions, dtype=np.int64)
    batch, length, _, head_dim = key_cache.shape
    cos_rows, sin_rows = np.asarray(cos)[positions], np.asarray(sin)[positions]
    q, k, v = qwen3_project(qkv, heads, kv_heads, head_dim, q_norm_weight, k_norm_weight,
                            eps, cos_rows, sin_rows, bf16)
    rows = np.arange(batch)
    key_cache[rows, positions] = k
    value_cache[rows, positions] = v
    group = heads // kv_heads
    mask = (np.arange(length)[None, :] <= positions[:, None])[:, None, None, :]
    grouped = q.reshape(batch, kv_heads, group, head_dim)
    keys = np.asarray(key_cache, dtype=np.float64).transpose(0, 2, 1, 3)
    values = np.asarray(value_cache, dtype=np.float64).transpose(0, 2, 1, 3)
    out = sdpa(grouped, keys, values, mask)
    return out.reshape(batch, heads * head_dim), key_cache, value_cache


def varlen_attention(q, k, v, starts, causal, scale=None, compute=np.float64):
    """Attention within each segment of packed ``(tokens, heads, head_dim)``
    tensors: ``attend(q, k, v, segments, causal)`` (``qwen3_asr.py:152-181``).

    Segment ``s`` is tokens ``starts[s] .. starts[s+1]-1`` (the reference's
    ``Segments.starts``, ``:136-149``). Within it, token ``i`` attends to all
    tokens of the segment, or (``causal``) to tokens ``0..i`` of it: the padded
    path's ``valid`` mask and ``tril`` (``:163-175``), the varlen path's
    ``window_size=(-1, 0)`` (``:155-165``). ``k``/``v`` may have fewer heads:
    query head ``h`` reads key/value head ``h // (heads / kv_heads)``
    (``enable_gqa``). Returns ``(tokens, heads, head_dim)``.
    """
    q = np.asarray(q, dtype=compute)
    k = np.asarray(k, dtype=compute)
    v = np.asarray(v, dtype=compute)
    starts = np.asarray(starts, dtype=np.int64)
    tokens, heads, head_dim = q.shape
    group = heads // k.shape[1]
    out = np.zeros((tokens, heads, head_dim), dtype=compute)
    for s in range(len(starts) - 1):
        a, b = int(starts[s]), int(starts[s + 1])
        if b <= a:
            continue
        qs = q[a:b].transpose(1, 0, 2)                                 # (heads, L, D)
        ks = np.repeat(k[a:b].transpose(1, 0, 2), group, axis=0)       # (heads, L, D)
        vs = np.repeat(v[a:b].transpose(1, 0, 2), group, axis=0)
        mask = np.tril(np.ones((b - a, b - a), dtype=bool)) if causal else None
        out[a:b] = sdpa(qs, ks, vs, mask, scale, compute).transpose(1, 0, 2)
    return out


def cross_kv_projection(x, k_weight, v_weight, v_bias, bf16: bool = False, compute=np.float64):
    """One decoder layer of ``set_encoder_output`` (``whisper.py:313-319``):
    ``project_key_value`` (``:88-91``: ``k_proj`` without bias, ``v_proj`` with
    it, ``_split_heads`` into heads of 64) of ``x`` ``(B, S, W)``. Returns
    ``(keys, values)``, each ``(B, W / 64, S, 64)``. ``nn.Linear`` in bf16
    rounds each output once (after the bias), which ``bf16=True`` replays."""
    x = np.asarray(x, compute)
    k = x @ np.asarray(k_weight, compute).T
    v = x @ np.asarray(v_weight, compute).T
    if v_bias is not None:
        v = v + np.asarray(v_bias, compute)
    out = []
    for t in (k, v):
        t = t.astype(np.float32)
        if bf16:
            t = bf16_round(t)
        b, s, w = t.shape
        out.append(t.reshape(b, s, w // 64, 64).transpose(0, 2, 1, 3))
    return out[0], out[1]
