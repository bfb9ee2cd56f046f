"""Drop-in: puts the sm_100a kernels behind the reference's own attention call sites.

``install()`` patches, in place, the classes of the reference's modules
(``asrback.models.whisper`` and ``asrback.models.qwen3_asr``, or modules with
the same class names and attributes). Everything around the call sites stays
the reference's: its Transcriber classes, continuous-batching scheduler,
caches and ``CapturedGraph`` capture the patched steps unchanged, since the
kernels read row positions on the device and allocate nothing per call.

Patched call sites (asrback project paths):

- ``whisper.DecoderLayer.forward`` (``src/asrback/models/whisper.py:212-241``):
  the fixed-shape step branch (``length is None``) runs the self-attention
  with its key/value write as one kernel and the cross-attention as another;
  the eager branch (``length`` given) with ``length`` equal to its token count
  (the prompt pass and language detection, ``whisper.py:847-849``,
  ``:979-981``) keeps the reference's ``index_copy_`` and runs causal
  self-attention and cross-attention for every prompt token on the same
  kernels; any other eager call goes to the original method;
- ``whisper.MultiHeadAttention.forward`` (``whisper.py:108-110``): the
  encoder's unmasked self-attention;
- ``whisper.WhisperForConditionalGeneration.set_encoder_output``
  (``whisper.py:313-319``): each decoder layer's cross-attention keys and
  values are projected and written into the cache by one kernel;
- ``qwen3_asr.TextModel.step`` (``src/asrback/models/qwen3_asr.py:494-524``)
  and ``qwen3_asr.TextAttention.step`` (``qwen3_asr.py:392-432``): the decoder
  step hands ``qkv_proj``'s output, the full RoPE tables and the positions to
  one kernel (RMSNorm, RoPE, cache write, grouped-query attention); no mask
  or varlen triple is built;
- ``qwen3_asr.attend`` (``qwen3_asr.py:152-181``), the module function that
  ``TextAttention.prefill`` (causal prompt prefill, ``:374-390``) and
  ``AudioAttention.forward`` (non-causal audio windows, ``:214-219``) call:
  attention within the packed segments runs on the varlen kernel, whichever
  path (``varlen_attn`` or padded SDPA) the segments were built for;
- ``whisper.Transcriber._step`` (``whisper.py:942-960``) and
  ``qwen3_asr.Qwen3ASRTranscriber._step`` (``qwen3_asr.py:1180-1201``): after
  the decoder, a greedy step (``temperatures`` None) runs the logits,
  ``_choose`` and the state update as one kernel; a step that samples goes to
  the original method.

The patched methods run the kernels only: tensors on the CPU raise, as every
op of this package does (there is no fallback).
"""

from __future__ import annotations

import importlib

import torch.nn.functional as F

from . import attention, step

__all__ = ["install", "uninstall", "installed"]

_originals: dict[tuple[object, str], object] = {}


def _patch(cls, name: str, function) -> None:
    key = (cls, name)
    if key not in _originals:
        _originals[key] = cls.__dict__[name]
    setattr(cls, name, function)


def installed() -> bool:
    return bool(_originals)


def uninstall() -> None:
    """Restores every patched method."""
    for (cls, name), function in _originals.items():
        setattr(cls, name, function)
    _originals.clear()


def _whisper_decoder_layer_forward(original):
    def forward(self, x, cache, positions, length, mask):
        prefix = length is not None
        if prefix and (length != x.shape[1] or mask is not None):
            return original(self, x, cache, positions, length, mask)
        self_keys, self_values, cross_keys, cross_values = cache
        hidden = self.self_attn_layer_norm(x)
        query = self.self_attn._split_heads(self.self_attn.q_proj(hidden))
        key, value = self.self_attn.project_key_value(hidden)
        if prefix:
            # whisper.py:229-233: the tokens' keys/values at the shared
            # positions; token t then attends to keys 0..t of the first
            # `length` positions (is_causal).
            self_keys.index_copy_(2, positions, key)
            self_values.index_copy_(2, positions, value)
            out = attention.whisper_self_attention_prefix(
                query, self_keys[:, :, :length], self_values[:, :, :length])
        else:
            out = attention.whisper_self_attention_step(query, key, value, self_keys, self_values,
                                                        positions)
        x = x + self.self_attn.out_proj(out)
        hidden = self.encoder_attn_layer_norm(x)
        query = self.encoder_attn._split_heads(self.encoder_attn.q_proj(hidden))
        if prefix:
            out = attention.whisper_cross_attention_prefix(query, cross_keys, cross_values)
        else:
            out = attention.whisper_cross_attention_step(query, cross_keys, cross_values)
        x = x + self.encoder_attn.out_proj(out)
        return x + self.fc2(F.gelu(self.fc1(self.final_layer_norm(x))))

    forward.__doc__ = original.__doc__
    return forward


def _whisper_encoder_attention_forward(self, x):
    """Unmasked self-attention on the encoder kernel."""
    query = self._split_heads(self.q_proj(x))
    key, value = self.project_key_value(x)
    return self.out_proj(attention.whisper_encoder_attention(query, key, value))


def _whisper_set_encoder_output(self, cache, encoder_output):
    """Fills the first ``len(encoder_output)`` rows' cross keys/values, one
    projection kernel per decoder layer."""
    batch_size = encoder_output.shape[0]
    for index, layer in enumerate(self.model.decoder.layers):
        attn = layer.encoder_attn
        attention.whisper_cross_kv_projection(
            encoder_output, attn.k_proj.weight, attn.v_proj.weight, attn.v_proj.bias,
            cache.cross_keys[index, :batch_size], cache.cross_values[index, :batch_size])


def _qwen3_text_attention_step(self, x, keys, values, positions, mask, cos, sin):
    """One token per row; ``cos``/``sin`` are the full tables (the patched
    ``TextModel.step`` passes them ungathered), ``mask`` is unused."""
    out = attention.qwen3_attention_step(
        self.qkv_proj(x), self.q_norm.weight, self.k_norm.weight, self.q_norm.eps, cos, sin,
        positions, keys, values, self.heads, self.kv_heads)
    return self.o_proj(out)


def _qwen3_attend(q, k, v, segments, causal):
    """Attention within each segment of packed ``(tokens, heads, head_dim)``
    tensors on the varlen kernel (``segments.starts`` is already on the
    device)."""
    return attention.varlen_attention(q, k, v, segments.starts, segments.longest, causal)


def _qwen3_text_model_step(self, tokens, positions, cache, cos, sin, varlen):
    """Hidden states for one token per row over a fixed-shape cache view; each
    row reads only its written keys, whatever ``varlen`` says."""
    x = self.embed_tokens(tokens)
    for index, layer in enumerate(self.layers):
        keys, values = cache.keys[index], cache.values[index]
        x = layer(x, lambda attn, h, keys=keys, values=values: attn.step(
            h, keys, values, positions, None, cos, sin))
    return self.norm(x)


def _whisper_transcriber_step(original):
    def _step(self, state, cache, temperatures=None):
        if temperatures is not None:
            return original(self, state, cache, temperatures)
        hidden = self.model.decode(state.tokens, state.position, cache)
        # `logits` (whisper.py:337-342) multiplies by the tied embedding.
        step.greedy_step(hidden[:, -1], self.model.model.decoder.embed_tokens.weight,
                         state.tokens, state.position, state.end, state.finished,
                         state.sum_logprobs, state.generated, (self._eos,), self._suppress)

    _step.__doc__ = original.__doc__
    return _step


def _qwen3_transcriber_step(original):
    def _step(self, state, cache, temperatures=None):
        if temperatures is not None:
            return original(self, state, cache, temperatures)
        hidden = self._text.step(state.tokens, state.position, cache, self._cos, self._sin,
                                 self._varlen)
        # The EOS ids live on the device; a host copy is taken on the first
        # (eager, uncaptured) step and kept.
        eos = self.__dict__.get("_asrback_eos_ids")
        if eos is None:
            eos = self._asrback_eos_ids = tuple(int(e) for e in self._eos_ids.reshape(-1).tolist())
        step.greedy_step(hidden, self._lm_head.weight, state.tokens, state.position, state.end,
                         state.finished, state.sum_logprobs, state.generated, eos)

    _step.__doc__ = original.__doc__
    return _step


def install(whisper_module=None, qwen3_module=None, *, encoder: bool = True) -> None:
    """Patches the reference's Whisper and Qwen3-ASR classes (importing
    ``asrback.models.whisper`` / ``asrback.models.qwen3_asr`` when no module is
    given; a module that cannot be imported is skipped).

    ``encoder=False`` leaves ``whisper.MultiHeadAttention.forward`` (the
    encoder's self-attention) to the reference: on B200 with torch 2.11 its
    SDPA call runs cuDNN's sm100 kernel, which is faster than this package's
    encoder kernel for the 1500-frame windows (about 460 against 555 us per
    layer over 32 windows)."""
    if whisper_module is None:
        whisper_module = _try_import("asrback.models.whisper")
    if qwen3_module is None:
        qwen3_module = _try_import("asrback.models.qwen3_asr")
    if whisper_module is not None:
        layer = whisper_module.DecoderLayer
        original = _originals.get((layer, "forward"), layer.__dict__["forward"])
        _patch(layer, "forward", _whisper_decoder_layer_forward(original))
        if encoder:
            _patch(whisper_module.MultiHeadAttention, "forward", _whisper_encoder_attention_forward)
        _patch(whisper_module.WhisperForConditionalGeneration, "set_encoder_output",
               _whisper_set_encoder_output)
        if hasattr(whisper_module, "Transcriber"):
            transcriber = whisper_module.Transcriber
            original = _originals.get((transcriber, "_step"), transcriber.__dict__["_step"])
            _patch(transcriber, "_step", _whisper_transcriber_step(original))
    if qwen3_module is not None:
        _patch(qwen3_module.TextAttention, "step", _qwen3_text_attention_step)
        _patch(qwen3_module.TextModel, "step", _qwen3_text_model_step)
        _patch(qwen3_module, "attend", _qwen3_attend)
        if hasattr(qwen3_module, "Qwen3ASRTranscriber"):
            transcriber = qwen3_module.Qwen3ASRTranscriber
            original = _originals.get((transcriber, "_step"), transcriber.__dict__["_step"])
            _patch(transcriber, "_step", _qwen3_transcriber_step(original))


def _try_import(name: str):
    try:
        return importlib.import_module(name)
    except ImportError:
        return None
