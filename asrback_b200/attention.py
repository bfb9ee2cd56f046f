"""Torch-facing attention ops over the C ABI of ``libasrback_attn.so``.

Each op takes the tensors the reference has at its attention call site, checks
them, and launches the sm_100a kernel on the current CUDA stream through
:mod:`asrback_b200._native`. The ops allocate only their outputs (from torch's
caching allocator, so they can be captured in a CUDA graph) plus, once per
device, a small status word and the split-KV workspace.

Reference call sites (asrback project paths):

- :func:`whisper_self_attention_step`: ``DecoderLayer.forward`` step branch,
  ``src/asrback/models/whisper.py:222-237`` (``scatter_`` then masked attend);
- :func:`whisper_cross_attention_step`: ``whisper.py:239-240``;
- :func:`whisper_self_attention_prefix` and
  :func:`whisper_cross_attention_prefix`: the same two calls in the eager
  branch (``whisper.py:228-236``, ``:239-240``) for a prompt pass of P tokens
  per window with ``length == P``;
- :func:`qwen3_attention_step`: ``TextAttention.step``,
  ``src/asrback/models/qwen3_asr.py:392-432`` with ``_project`` (``:366-372``);
- :func:`whisper_encoder_attention`: ``MultiHeadAttention.forward``,
  ``whisper.py:108-110``;
- :func:`whisper_cross_kv_projection`: ``set_encoder_output``,
  ``whisper.py:313-319`` (``project_key_value``, ``:88-91``, and the copy into
  the cross-attention cache), one decoder layer per call.
"""

from __future__ import annotations

import math
import threading

import torch
from torch import Tensor

from . import _native

__all__ = [
    "whisper_self_attention_step",
    "whisper_cross_attention_step",
    "qwen3_attention_step",
    "whisper_encoder_attention",
    "whisper_cross_kv_projection",
    "varlen_attention",
    "reserve_workspace",
    "read_status",
    "DeviceStatusError",
]

_DTYPES = {torch.bfloat16: _native.BF16, torch.float32: _native.F32}


class DeviceStatusError(RuntimeError):
    """A kernel flagged a row it could not process (see :func:`read_status`)."""


class _DeviceState:
    """Per-device status word and split-KV workspace (zero-filled, grown on
    demand outside graph capture; the kernels leave its counters at zero).

    A workspace that a call has used is never freed. The reference captures one
    graph per (batch, length) bucket in turn (``whisper.py:710-725``,
    ``qwen3_asr.py:930-948``), and the workspace a bucket needs is not monotonic
    in the bucket, so a later capture's warm-up may grow it; graphs captured
    before keep the old buffer's address baked in and must find it intact (its
    counters at zero) on every replay. Superseded buffers therefore stay alive
    in ``retired`` for the life of the process."""

    def __init__(self, device: torch.device) -> None:
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self.workspace = torch.zeros(0, dtype=torch.uint8, device=device)
        self.retired: list[Tensor] = []

    def workspace_for(self, nbytes: int) -> Tensor:
        if nbytes > self.workspace.numel():
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError(
                    "asrback_b200: the split-KV workspace must grow during CUDA graph "
                    "capture; run the step once before capturing it (CapturedGraph's "
                    "warm-up does) or call reserve_workspace() first"
                )
            if self.workspace.numel():
                self.retired.append(self.workspace)
            self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=self.status.device)
        return self.workspace


_states: dict[int, _DeviceState] = {}
_states_lock = threading.Lock()


def _state(device: torch.device) -> _DeviceState:
    index = device.index if device.index is not None else torch.cuda.current_device()
    state = _states.get(index)
    if state is None:
        with _states_lock:
            state = _states.get(index)
            if state is None:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError(
                        "asrback_b200: first call on a device happened during CUDA graph "
                        "capture; warm the step up first"
                    )
                state = _states[index] = _DeviceState(torch.device("cuda", index))
    return state


def _dtype_code(*tensors: Tensor) -> int:
    dtype = tensors[0].dtype
    for tensor in tensors:
        if tensor.dtype != dtype:
            raise TypeError(f"asrback_b200: mixed dtypes {dtype} and {tensor.dtype}")
        if not tensor.is_cuda:
            raise ValueError("asrback_b200: tensors must be on a CUDA device")
    if dtype not in _DTYPES:
        raise TypeError(f"asrback_b200: dtype {dtype} is not supported (bfloat16, float32)")
    return _DTYPES[dtype]


def _heads(t: Tensor, name: str) -> Tensor:
    """``(B, H, D)`` view of a ``(B, H, D)`` or ``(B, H, 1, D)`` tensor."""
    if t.dim() == 4:
        if t.shape[2] != 1:
            raise ValueError(f"asrback_b200: {name} must hold one token per row, got {tuple(t.shape)}")
        t = t[:, :, 0]
    if t.dim() != 3 or t.stride(-1) != 1:
        raise ValueError(f"asrback_b200: {name} must be (batch, heads, head_dim) with unit last stride")
    return t


def _cache(t: Tensor, name: str) -> Tensor:
    """A ``(B, H, L, D)`` cache view whose rows of one head are contiguous."""
    if t.dim() != 4 or t.stride(-1) != 1 or t.stride(2) != t.shape[3]:
        raise ValueError(
            f"asrback_b200: {name} must be (batch, heads, length, head_dim) with contiguous rows"
        )
    return t


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def reserve_workspace(device: torch.device | int | str, batch: int, heads: int, head_dim: int,
                      max_keys: int) -> None:
    """Grows the device's split-KV workspace to cover calls up to these sizes,
    so no later call (e.g. inside graph capture) needs to grow it."""
    device = torch.device(device) if not isinstance(device, torch.device) else device
    if device.type != "cuda":
        device = torch.device("cuda", device.index if device.index is not None else 0)
    lib = _native.load()
    with torch.cuda.device(device):
        need = lib.asrback_decode_workspace_bytes(batch, heads, head_dim, max_keys)
        _state(device).workspace_for(need)


def _workspace(state: _DeviceState, batch: int, heads: int, head_dim: int, max_keys: int):
    lib = _native.load()
    need = lib.asrback_decode_workspace_bytes(batch, heads, head_dim, max_keys)
    workspace = state.workspace_for(need)
    return workspace.data_ptr() if workspace.numel() else None, workspace.numel()


def read_status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """The device's status bits (``_native.STATUS_*``) set by kernels since the
    last clear. Synchronizes with the device, so never call it inside capture."""
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    elif not isinstance(device, torch.device):
        device = torch.device("cuda", device)
    state = _state(device)
    value = int(state.status.item())
    if clear and value:
        state.status.zero_()
    return value


def whisper_self_attention_step(query: Tensor, key: Tensor, value: Tensor, key_cache: Tensor,
                                value_cache: Tensor, positions: Tensor,
                                scale: float | None = None) -> Tensor:
    """Writes each row's ``key``/``value`` into the caches at ``positions[b]``
    and attends with ``query`` to keys ``0..positions[b]``.

    ``query``/``key``/``value``: ``(B, H, D)`` or ``(B, H, 1, D)`` (the
    reference's ``_split_heads`` views); caches ``(B, H, L, D)`` views of
    ``DecoderCache``; ``positions`` ``(B,)`` int64. Returns ``(B, 1, H*D)``, the
    layout ``attend`` hands to ``out_proj``.
    """
    query, key, value = _heads(query, "query"), _heads(key, "key"), _heads(value, "value")
    key_cache, value_cache = _cache(key_cache, "key_cache"), _cache(value_cache, "value_cache")
    dtype = _dtype_code(query, key, value, key_cache, value_cache)
    batch, heads, head_dim = query.shape
    if key.shape != query.shape or value.shape != query.shape:
        raise ValueError("asrback_b200: query, key and value shapes differ")
    if key.stride() != value.stride():
        raise ValueError("asrback_b200: key and value must share strides")
    if key_cache.shape[:2] != (batch, heads) or key_cache.shape[3] != head_dim:
        raise ValueError(f"asrback_b200: cache {tuple(key_cache.shape)} does not match query {tuple(query.shape)}")
    if value_cache.shape != key_cache.shape or value_cache.stride() != key_cache.stride():
        raise ValueError("asrback_b200: key and value caches differ in shape or strides")
    if positions.dtype != torch.int64 or positions.shape != (batch,) or positions.device != query.device:
        raise ValueError("asrback_b200: positions must be (batch,) int64 on the query's device")
    positions = positions.contiguous()
    length = key_cache.shape[2]
    out = torch.empty((batch, 1, heads * head_dim), dtype=query.dtype, device=query.device)
    state = _state(query.device)
    ws, ws_bytes = _workspace(state, batch, heads, head_dim, length)
    _native.call(
        "asrback_whisper_self_attention_step",
        dtype, batch, heads, head_dim, length,
        query.data_ptr(), query.stride(0), query.stride(1),
        key.data_ptr(), value.data_ptr(), key.stride(0), key.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(), key_cache.stride(0), key_cache.stride(1),
        positions.data_ptr(),
        out.data_ptr(), heads * head_dim, head_dim,
        scale if scale is not None else 1.0 / math.sqrt(head_dim),
        ws, ws_bytes, state.status.data_ptr(), _stream(query.device),
    )
    return out


def whisper_cross_attention_step(query: Tensor, key_cache: Tensor, value_cache: Tensor,
                                 scale: float | None = None) -> Tensor:
    """Unmasked attention of one query per row over the window's encoder keys.
    ``query`` ``(B, H, D)`` or ``(B, H, 1, D)``; caches ``(B, H, S, D)``.
    Returns ``(B, 1, H*D)``."""
    query = _heads(query, "query")
    key_cache, value_cache = _cache(key_cache, "key_cache"), _cache(value_cache, "value_cache")
    dtype = _dtype_code(query, key_cache, value_cache)
    batch, heads, head_dim = query.shape
    if key_cache.shape[:2] != (batch, heads) or key_cache.shape[3] != head_dim:
        raise ValueError(f"asrback_b200: cache {tuple(key_cache.shape)} does not match query {tuple(query.shape)}")
    if value_cache.shape != key_cache.shape or value_cache.stride() != key_cache.stride():
        raise ValueError("asrback_b200: key and value caches differ in shape or strides")
    length = key_cache.shape[2]
    out = torch.empty((batch, 1, heads * head_dim), dtype=query.dtype, device=query.device)
    state = _state(query.device)
    ws, ws_bytes = _workspace(state, batch, heads, head_dim, length)
    _native.call(
        "asrback_whisper_cross_attention_step",
        dtype, batch, heads, head_dim, length,
        query.data_ptr(), query.stride(0), query.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(), key_cache.stride(0), key_cache.stride(1),
        out.data_ptr(), heads * head_dim, head_dim,
        scale if scale is not None else 1.0 / math.sqrt(head_dim),
        ws, ws_bytes, state.status.data_ptr(), _stream(query.device),
    )
    return out


def _prefix_query(t: Tensor, name: str) -> tuple[Tensor, int]:
    """A ``(B, H, P, D)`` query view and its token stride, with the (window,
    token) rows evenly spaced (row ``b*P + t`` at ``(b*P + t) * stride``), as
    ``_split_heads`` of a ``(B, P, W)`` projection lays them out. Other
    layouts are copied into that one first."""
    if t.dim() != 4 or t.stride(-1) != 1:
        raise ValueError(f"asrback_b200: {name} must be (batch, heads, tokens, head_dim) with unit last stride")
    batch, _, tokens, _ = t.shape
    stride = t.stride(2) if tokens > 1 else t.stride(0)
    if batch > 1 and tokens > 1 and t.stride(0) != tokens * stride:
        t = t.transpose(1, 2).contiguous().transpose(1, 2)
        stride = t.stride(2)
    return t, stride


def _prefix_call(name: str, query: Tensor, key_cache: Tensor, value_cache: Tensor, length: int,
                 scale: float | None) -> Tensor:
    query, token_stride = _prefix_query(query, "query")
    key_cache, value_cache = _cache(key_cache, "key_cache"), _cache(value_cache, "value_cache")
    dtype = _dtype_code(query, key_cache, value_cache)
    batch, heads, tokens, head_dim = query.shape
    if key_cache.shape[:2] != (batch, heads) or key_cache.shape[3] != head_dim:
        raise ValueError(f"asrback_b200: cache {tuple(key_cache.shape)} does not match query {tuple(query.shape)}")
    if value_cache.shape != key_cache.shape or value_cache.stride() != key_cache.stride():
        raise ValueError("asrback_b200: key and value caches differ in shape or strides")
    out = torch.empty((batch, tokens, heads * head_dim), dtype=query.dtype, device=query.device)
    state = _state(query.device)
    lib = _native.load()
    need = lib.asrback_whisper_prefix_workspace_bytes(batch, tokens, heads, head_dim, length)
    workspace = state.workspace_for(need)
    ws, ws_bytes = (workspace.data_ptr() if workspace.numel() else None), workspace.numel()
    _native.call(
        name,
        dtype, batch, tokens, heads, head_dim, length,
        query.data_ptr(), token_stride, query.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(), key_cache.stride(0), key_cache.stride(1),
        out.data_ptr(), heads * head_dim, head_dim,
        scale if scale is not None else 1.0 / math.sqrt(head_dim),
        ws, ws_bytes, state.status.data_ptr(), _stream(query.device),
    )
    return out


def whisper_self_attention_prefix(query: Tensor, key_cache: Tensor, value_cache: Tensor,
                                  scale: float | None = None) -> Tensor:
    """Causal self-attention of a prompt pass: token ``t`` of each window
    attends to cache keys ``0..t``, which the caller has written (the
    reference's ``index_copy_``, ``whisper.py:231-232``); the caches are read
    only.

    ``query`` ``(B, H, P, D)`` (the ``_split_heads`` view); caches
    ``(B, H, L, D)`` with ``L >= P``. Returns ``(B, P, H*D)``, the layout
    ``attend`` hands to ``out_proj``.
    """
    return _prefix_call("asrback_whisper_self_attention_prefix", query, key_cache, value_cache,
                        key_cache.shape[2], scale)


def whisper_cross_attention_prefix(query: Tensor, key_cache: Tensor, value_cache: Tensor,
                                   scale: float | None = None) -> Tensor:
    """Unmasked attention of every prompt token over its window's encoder
    keys. ``query`` ``(B, H, P, D)``; caches ``(B, H, S, D)``. Returns
    ``(B, P, H*D)``."""
    length = key_cache.shape[2] if key_cache.dim() == 4 else 0
    return _prefix_call("asrback_whisper_cross_attention_prefix", query, key_cache, value_cache,
                        length, scale)


def qwen3_attention_step(qkv: Tensor, q_norm_weight: Tensor, k_norm_weight: Tensor, eps: float,
                         cos: Tensor, sin: Tensor, positions: Tensor, keys: Tensor, values: Tensor,
                         heads: int, kv_heads: int, scale: float | None = None) -> Tensor:
    """Qwen3 attention for one token per row, from ``qkv_proj``'s output to
    ``o_proj``'s input: q/k RMSNorm + RoPE at ``positions``, the key/value
    written into ``keys``/``values`` ``(B, L, kv_heads, D)`` at each row's
    position, then grouped-query attention over keys ``0..positions[b]``.
    ``cos``/``sin`` are the full ``(table_length, D)`` tables. Returns
    ``(B, heads*D)``."""
    dtype = _dtype_code(qkv, q_norm_weight, k_norm_weight, cos, sin, keys, values)
    if qkv.dim() != 2 or qkv.stride(1) != 1:
        raise ValueError("asrback_b200: qkv must be (batch, width) with unit last stride")
    batch = qkv.shape[0]
    if keys.dim() != 4:
        raise ValueError("asrback_b200: keys must be (batch, length, kv_heads, head_dim)")
    _, length, kvh, head_dim = keys.shape
    if kvh != kv_heads or qkv.shape[1] != (heads + 2 * kv_heads) * head_dim:
        raise ValueError("asrback_b200: qkv width or cache heads do not match heads/kv_heads")
    if keys.shape[0] != batch or values.shape != keys.shape or values.stride() != keys.stride():
        raise ValueError("asrback_b200: keys/values shapes or strides differ from the batch")
    if keys.stride(3) != 1 or keys.stride(2) != head_dim or keys.stride(1) != kv_heads * head_dim:
        raise ValueError("asrback_b200: each cache row (position) must be contiguous kv_heads x head_dim")
    for table in (cos, sin):
        if table.dim() != 2 or table.shape[1] != head_dim or table.stride(1) != 1:
            raise ValueError("asrback_b200: cos/sin must be (table_length, head_dim)")
    if cos.stride(0) != sin.stride(0) or cos.shape != sin.shape:
        raise ValueError("asrback_b200: cos and sin must share shape and strides")
    for weight in (q_norm_weight, k_norm_weight):
        if weight.shape != (head_dim,) or not weight.is_contiguous():
            raise ValueError("asrback_b200: norm weights must be contiguous (head_dim,)")
    if positions.dtype != torch.int64 or positions.shape != (batch,) or positions.device != qkv.device:
        raise ValueError("asrback_b200: positions must be (batch,) int64 on qkv's device")
    positions = positions.contiguous()
    out = torch.empty((batch, heads * head_dim), dtype=qkv.dtype, device=qkv.device)
    state = _state(qkv.device)
    ws, ws_bytes = _workspace(state, batch, heads, head_dim, length)
    _native.call(
        "asrback_qwen3_attention_step",
        dtype, batch, heads, kv_heads, head_dim, length,
        qkv.data_ptr(), qkv.stride(0),
        q_norm_weight.data_ptr(), k_norm_weight.data_ptr(), float(eps),
        cos.data_ptr(), sin.data_ptr(), cos.stride(0), cos.shape[0],
        positions.data_ptr(),
        keys.data_ptr(), values.data_ptr(), keys.stride(0),
        out.data_ptr(), out.stride(0),
        scale if scale is not None else 1.0 / math.sqrt(head_dim),
        ws, ws_bytes, state.status.data_ptr(), _stream(qkv.device),
    )
    return out


def whisper_encoder_attention(q: Tensor, k: Tensor, v: Tensor, scale: float | None = None) -> Tensor:
    """Non-causal self-attention over ``(B, H, S, D)`` views sharing strides
    (the reference's ``_split_heads`` of ``(B, S, H*D)`` projections). Returns
    ``(B, S, H*D)``, the layout ``attend`` hands to ``out_proj``."""
    dtype = _dtype_code(q, k, v)
    if q.dim() != 4 or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("asrback_b200: q, k, v must be (batch, heads, length, head_dim) of one shape")
    if q.stride() != k.stride() or q.stride() != v.stride():
        raise ValueError("asrback_b200: q, k and v must share strides")
    if q.stride(3) != 1:
        raise ValueError("asrback_b200: head_dim must have unit stride")
    batch, heads, length, head_dim = q.shape
    out = torch.empty((batch, length, heads * head_dim), dtype=q.dtype, device=q.device)
    view = out.view(batch, length, heads, head_dim).transpose(1, 2)
    if view.stride() != q.stride():
        # Inputs not in the (B, S, H*D) projection layout: lay q/k/v out that way.
        q, k, v = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    state = _state(q.device)
    _native.call(
        "asrback_whisper_encoder_attention",
        dtype, batch, heads, head_dim, length,
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
        q.stride(0), q.stride(1), q.stride(2),
        scale if scale is not None else 1.0 / math.sqrt(head_dim),
        state.status.data_ptr(), _stream(q.device),
    )
    return out


def whisper_cross_kv_projection(encoder_output: Tensor, k_weight: Tensor, v_weight: Tensor,
                                v_bias: Tensor | None, keys: Tensor, values: Tensor) -> None:
    """One decoder layer's cross-attention keys and values, written into its
    cache rows: ``keys[:, h, :S] = (x @ k_weight.T)`` split into heads of 64,
    ``values`` likewise with ``v_bias`` (``encoder_output`` ``(B, S, W)``;
    ``keys``/``values`` the ``(B, H, L >= S, 64)`` views
    ``cross_keys[layer, :B]`` / ``cross_values[layer, :B]``)."""
    dtype = _dtype_code(encoder_output, k_weight, v_weight, keys, values)
    if v_bias is not None:
        _dtype_code(encoder_output, v_bias)
    if encoder_output.dim() != 3 or encoder_output.stride(2) != 1:
        raise ValueError("asrback_b200: encoder_output must be (batch, tokens, width) with "
                         "contiguous rows")
    batch, tokens, width = encoder_output.shape
    for name, w in (("k_weight", k_weight), ("v_weight", v_weight)):
        if w.shape != (width, width) or w.stride(1) != 1 or w.stride(0) != k_weight.stride(0):
            raise ValueError(f"asrback_b200: {name} must be ({width}, {width}) with contiguous "
                             "rows, both weights with one stride")
    if v_bias is not None and (v_bias.shape != (width,) or v_bias.stride(0) != 1):
        raise ValueError(f"asrback_b200: v_bias must be a contiguous ({width},) tensor")
    for name, c in (("keys", keys), ("values", values)):
        if c.dim() != 4 or c.shape[0] != batch or c.shape[1] * c.shape[3] != width \
                or c.shape[3] != 64 or c.shape[2] < tokens or c.stride(3) != 1:
            raise ValueError(f"asrback_b200: {name} must be a (batch, heads, length >= tokens, 64) "
                             "cache view with contiguous rows")
    if keys.stride() != values.stride():
        raise ValueError("asrback_b200: keys and values must share strides")
    state = _state(encoder_output.device)
    _native.call(
        "asrback_whisper_cross_kv_projection", dtype, batch, tokens, width,
        encoder_output.data_ptr(), encoder_output.stride(0), encoder_output.stride(1),
        k_weight.data_ptr(), v_weight.data_ptr(), k_weight.stride(0),
        None if v_bias is None else v_bias.data_ptr(),
        keys.data_ptr(), values.data_ptr(), keys.stride(0), keys.stride(1), keys.stride(2),
        state.status.data_ptr(), _stream(encoder_output.device),
    )


def varlen_attention(q: Tensor, k: Tensor, v: Tensor, starts: Tensor, longest: int, causal: bool,
                     scale: float | None = None) -> Tensor:
    """Attention within each segment of packed ``(tokens, heads, head_dim)``
    tensors: the reference's ``attend(q, k, v, segments, causal)``
    (``qwen3_asr.py:152-181``) with ``segments.starts`` and
    ``segments.longest``. ``k``/``v`` may have fewer heads than ``q`` (query
    head ``h`` reads key/value head ``h // (heads / kv_heads)``); ``causal``
    lets token ``i`` of a segment see tokens ``0..i`` of it. ``starts`` is
    ``(segments + 1,)`` int32 on the tensors' device. Returns ``(tokens,
    heads, head_dim)``."""
    dtype = _dtype_code(q, k, v)
    if q.dim() != 3 or k.dim() != 3 or v.dim() != 3:
        raise ValueError("asrback_b200: q, k, v must be (tokens, heads, head_dim)")
    tokens, heads, head_dim = q.shape
    kv_heads = k.shape[1]
    if k.shape != (tokens, kv_heads, head_dim) or v.shape != k.shape:
        raise ValueError(f"asrback_b200: k {tuple(k.shape)} / v {tuple(v.shape)} do not match q {tuple(q.shape)}")
    if q.stride(2) != 1 or k.stride(2) != 1 or v.stride(2) != 1:
        raise ValueError("asrback_b200: head_dim must have unit stride")
    if starts.dtype != torch.int32 or starts.dim() != 1 or starts.device != q.device:
        raise ValueError("asrback_b200: starts must be (segments + 1,) int32 on the tensors' device")
    starts = starts.contiguous()
    segments = starts.shape[0] - 1
    out = torch.empty((tokens, heads, head_dim), dtype=q.dtype, device=q.device)
    state = _state(q.device)
    _native.call(
        "asrback_varlen_attention",
        dtype, tokens, heads, kv_heads, head_dim,
        q.data_ptr(), q.stride(0), q.stride(1),
        k.data_ptr(), k.stride(0), k.stride(1),
        v.data_ptr(), v.stride(0), v.stride(1),
        starts.data_ptr(), segments, int(longest), 1 if causal else 0,
        out.data_ptr(), out.stride(0), out.stride(1),
        scale if scale is not None else 1.0 / math.sqrt(head_dim),
        state.status.data_ptr(), _stream(q.device),
    )
    return out
