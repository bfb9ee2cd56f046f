"""CPU oracle for asrback's greedy step epilogue (numpy).

TEST INFRASTRUCTURE ONLY. The parity tests, ``smoke()`` and the CPU-baseline
leg of ``bench.py`` compare the fused CUDA step epilogue against these
functions; the product path (``asrback_b200``) never imports them.

What it restates (paths relative to the asrback project):

- the logits: ``WhisperForConditionalGeneration.logits``
  (``src/asrback/models/whisper.py:337-342``, ``weight @ rows.T`` with the tied
  ``embed_tokens`` weight) and Qwen3's ``self._lm_head(hidden)``
  (``src/asrback/models/qwen3_asr.py:1189``, ``nn.Linear`` without bias), both
  then ``.float()``. In bfloat16 torch accumulates each dot product in fp32 and
  rounds it once to bf16; ``bf16=True`` replays that rounding on float64 dots;
- ``_choose`` on the greedy path (``whisper.py:962-975``, with the suppress
  mask; ``qwen3_asr.py:1203-1213``, without): ``argmax`` (first index of the
  maximum) and ``log_softmax(logits).gather(token)``;
- the state update of ``_step`` (``whisper.py:951-960``,
  ``qwen3_asr.py:1190-1201``): finished rows keep their token and position,
  active rows advance; ``sum_logprobs`` adds the log-probability of active
  rows; ``generated[row, position] = token``; a row finishes on an EOS token
  (``==`` for Whisper, ``isin`` over several ids for Qwen3) or at ``end``.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own
``Transcriber._step`` / ``Qwen3ASRTranscriber._step`` (with a stub in place
of the decoder) and stores their inputs and results as ``step_epilogue_*``;
``tests/test_oracle_golden.py`` checks these functions against them.
"""

from __future__ import annotations

import numpy as np

from .attention import bf16_round

__all__ = ["logits", "choose", "update_state", "greedy_step"]


def logits(weight, hidden, bf16: bool, compute=np.float64) -> np.ndarray:
    """``(batch, vocab)`` float32 logits of ``hidden (batch, d)`` against
    ``weight (vocab, d)``: float64 dot products, rounded to bf16 when the
    reference computes in bf16."""
    out = (np.asarray(hidden, compute) @ np.asarray(weight, compute).T).astype(np.float32)
    return bf16_round(out) if bf16 else out


def choose(logits_, suppress=None) -> tuple[np.ndarray, np.ndarray]:
    """Greedy ``_choose``: the masked logits' argmax (first maximal index) and
    its log-probability under ``log_softmax`` (float64 sums)."""
    x = np.array(logits_, dtype=np.float32, copy=True)
    if suppress is not None:
        x[:, np.asarray(suppress, bool)] = -np.inf
    token = np.argmax(x, axis=1)
    x64 = x.astype(np.float64)
    m = x64.max(axis=1, keepdims=True)
    lse = m[:, 0] + np.log(np.exp(x64 - m).sum(axis=1))
    logprob = x64[np.arange(len(token)), token] - lse
    return token.astype(np.int64), logprob.astype(np.float32)


def update_state(state: dict, token, logprob, eos_ids) -> dict:
    """The state update after ``_choose``; ``state`` holds ``tokens`` (batch,),
    ``position``, ``end``, ``finished`` (bool), ``sum_logprobs`` (float32) and
    ``generated`` (batch, length). Returns a new dict."""
    finished = np.asarray(state["finished"], bool)
    active = ~finished
    position = np.asarray(state["position"], np.int64) + active
    tokens = np.where(active, token, np.asarray(state["tokens"], np.int64))
    sums = np.asarray(state["sum_logprobs"], np.float32) + np.where(finished, 0.0, logprob).astype(
        np.float32)
    generated = np.array(state["generated"], np.int64, copy=True)
    generated[np.arange(len(tokens)), position] = tokens
    eos = np.isin(tokens, np.asarray(eos_ids, np.int64).reshape(-1))
    return dict(tokens=tokens, position=position, end=np.asarray(state["end"], np.int64),
                finished=finished | eos | (position >= np.asarray(state["end"], np.int64)),
                sum_logprobs=sums, generated=generated)


def greedy_step(weight, hidden, state: dict, eos_ids, suppress=None, bf16: bool = False):
    """Logits, ``_choose`` and the state update of one greedy ``_step``.
    Returns ``(token, logprob, new_state)``."""
    token, logprob = choose(logits(weight, hidden, bf16), suppress)
    return token, logprob, update_state(state, token, logprob, eos_ids)
