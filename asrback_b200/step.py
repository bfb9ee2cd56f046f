"""Greedy step epilogue over the C ABI: the logits, ``_choose`` and the
decode-state update of one step in one kernel launch.

Reference (asrback project paths), on the greedy path (``temperatures`` None):

- ``Transcriber._step`` after the decoder, ``src/asrback/models/whisper.py:949-960``:
  ``logits`` (``:337-342``, the tied ``embed_tokens`` weight), ``_choose``
  (``:962-975``, with the suppress mask) and the state update;
- ``Qwen3ASRTranscriber._step``, ``src/asrback/models/qwen3_asr.py:1189-1201``:
  ``_lm_head``, ``_choose`` (``:1203-1213``) and the state update with several
  EOS ids (``torch.isin``).

bf16 runs the logits on the tensor cores (fp32 sums rounded to bf16, as the
reference's bf16 matmul returns them); float32 runs a SIMT kernel. Sampling
(a positive temperature) is not fused: the reference's graphs cover greedy
steps only, and the patched ``_step`` hands sampled steps to the original.
"""

from __future__ import annotations

import ctypes
import threading
from collections.abc import Sequence

import torch
from torch import Tensor

from . import _native, attention

__all__ = ["greedy_choose", "greedy_step", "MAX_BATCH"]

MAX_BATCH = 128  # bf16; float32 takes up to 64 rows

_workspaces: dict[int, Tensor] = {}
_lock = threading.Lock()


def _workspace(device: torch.device) -> Tensor:
    index = device.index if device.index is not None else torch.cuda.current_device()
    workspace = _workspaces.get(index)
    if workspace is None:
        with _lock:
            workspace = _workspaces.get(index)
            if workspace is None:
                if torch.cuda.is_current_stream_capturing():
                    raise RuntimeError(
                        "asrback_b200: the step workspace is allocated on a device's first "
                        "greedy step; run one step before capturing it")
                nbytes = _native.load().asrback_greedy_step_workspace_bytes(MAX_BATCH)
                workspace = torch.zeros(nbytes, dtype=torch.uint8,
                                        device=torch.device("cuda", index))
                _workspaces[index] = workspace
    return workspace


def _rows(t: Tensor, name: str) -> Tensor:
    if t.dim() != 2 or t.stride(-1) != 1:
        raise ValueError(f"asrback_b200: {name} must be 2-D with contiguous rows, got "
                         f"{tuple(t.shape)} strides {t.stride()}")
    return t


def _vector(t: Tensor, name: str, dtype: torch.dtype, batch: int) -> Tensor:
    if t.dtype != dtype or t.dim() != 1 or t.shape[0] != batch or t.stride(0) != 1:
        raise ValueError(f"asrback_b200: {name} must be a contiguous ({batch},) {dtype} tensor")
    return t


def _launch(hidden: Tensor, weight: Tensor, suppress: Tensor | None, out_token, out_logprob,
            state: dict | None, eos_ids: Sequence[int]) -> None:
    hidden = _rows(hidden, "hidden")
    weight = _rows(weight, "weight")
    dtype = attention._dtype_code(hidden, weight)
    batch, width = hidden.shape
    vocab = weight.shape[0]
    if weight.shape[1] != width:
        raise ValueError(f"asrback_b200: weight {tuple(weight.shape)} does not match hidden "
                         f"width {width}")
    if suppress is not None:
        if suppress.shape != (vocab,) or suppress.dtype not in (torch.bool, torch.uint8) \
                or suppress.stride(0) != 1 or suppress.device != hidden.device:
            raise ValueError(f"asrback_b200: suppress must be a contiguous ({vocab},) bool tensor "
                             "on the hidden states' device")
    eos = [int(e) for e in eos_ids]
    eos_host = (ctypes.c_int64 * max(len(eos), 1))(*eos)
    device = hidden.device
    workspace = _workspace(device)
    ptr = lambda t: None if t is None else t.data_ptr()  # noqa: E731
    if state is None:
        tokens = position = end = finished = sums = generated = None
        tokens_stride = generated_stride = generated_cols = 0
    else:
        tokens = state["tokens"]
        if tokens.dtype != torch.int64 or tokens.shape[0] != batch or tokens.numel() != batch:
            raise ValueError(f"asrback_b200: tokens must be ({batch},) or ({batch}, 1) int64")
        tokens_stride = tokens.stride(0)
        position = _vector(state["position"], "position", torch.int64, batch)
        end = _vector(state["end"], "end", torch.int64, batch)
        finished = _vector(state["finished"], "finished", torch.bool, batch)
        sums = _vector(state["sum_logprobs"], "sum_logprobs", torch.float32, batch)
        generated = state["generated"]
        if generated.dtype != torch.int64 or generated.dim() != 2 or generated.shape[0] != batch \
                or generated.stride(1) != 1:
            raise ValueError(f"asrback_b200: generated must be ({batch}, length) int64 with "
                             "contiguous rows")
        generated_stride, generated_cols = generated.stride(0), generated.shape[1]
        for t in (tokens, position, end, finished, sums, generated):
            if t.device != device:
                raise ValueError("asrback_b200: the decode state must be on the hidden states' "
                                 "device")
    with torch.cuda.device(device):
        _native.call(
            "asrback_greedy_step", dtype, batch, vocab, width,
            hidden.data_ptr(), hidden.stride(0), weight.data_ptr(), weight.stride(0),
            ptr(suppress), ptr(out_token), ptr(out_logprob),
            ptr(tokens), tokens_stride, ptr(position), ptr(end), ptr(finished), ptr(sums),
            ptr(generated), generated_stride, generated_cols,
            eos_host, len(eos),
            workspace.data_ptr(), workspace.numel(), attention._state(device).status.data_ptr(),
            attention._stream(device))


def greedy_choose(hidden: Tensor, weight: Tensor,
                  suppress: Tensor | None = None) -> tuple[Tensor, Tensor]:
    """Greedy ``_choose`` of ``hidden (batch, d) @ weight (vocab, d).T``:
    ``(token int64, logprob float32)``, each ``(batch,)``."""
    batch = hidden.shape[0]
    token = torch.empty(batch, dtype=torch.int64, device=hidden.device)
    logprob = torch.empty(batch, dtype=torch.float32, device=hidden.device)
    _launch(hidden, weight, suppress, token, logprob, None, ())
    return token, logprob


def greedy_step(hidden: Tensor, weight: Tensor, tokens: Tensor, position: Tensor, end: Tensor,
                finished: Tensor, sum_logprobs: Tensor, generated: Tensor,
                eos_ids: Sequence[int], suppress: Tensor | None = None) -> None:
    """One greedy ``_step`` after the decoder, updating the decode state in
    place: ``tokens`` ``(batch,)`` or ``(batch, 1)``, ``position``, ``end``
    (int64), ``finished`` (bool), ``sum_logprobs`` (float32), ``generated``
    ``(batch, length)`` (int64); ``eos_ids`` are host ints (at most 8)."""
    state = dict(tokens=tokens, position=position, end=end, finished=finished,
                 sum_logprobs=sum_logprobs, generated=generated)
    _launch(hidden, weight, suppress, None, None, state, eos_ids)
