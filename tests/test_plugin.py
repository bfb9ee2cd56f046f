"""The plugin's wiring at the reference's own call sites (CPU, float32).

The reference's modules are imported read-only (skipped where they are not
mounted). With the plugin installed, the ops of asrback_b200.attention are
replaced here by CPU stand-ins built on the oracle (test-only; the product
ops have no CPU path), so the patched reference runs end to end on the host
and must reproduce the unpatched reference: same hidden states, same cache
writes. This pins the argument layouts the plugin hands to the kernels.
"""

from __future__ import annotations


import numpy as np
import pytest
import torch

from asrback_b200 import attention, plugin
from asrback_b200.synthetic import seeded_normal, seeded_parameters
from oracle import attention as oracle
from oracle import reference as reference_env

pytestmark = pytest.mark.skipif(reference_env.find() is None,
                                reason="asrback reference not found ($ASRBACK_REFERENCE or "
                                       "baseline/_ref)")


@pytest.fixture(scope="module")
def reference():
    ref = reference_env.load()
    return ref.whisper, ref.qwen3_asr


@pytest.fixture
def cpu_ops(monkeypatch):
    """Oracle-backed CPU stand-ins with the ops' signatures and side effects."""

    def self_step(query, key, value, key_cache, value_cache, positions, scale=None):
        q, k, v = (t[:, :, 0] if t.dim() == 4 else t for t in (query, key, value))
        out, kc, vc = oracle.whisper_self_attention_step(
            q.numpy(), k.numpy(), v.numpy(), key_cache.numpy(), value_cache.numpy(),
            positions.numpy())
        key_cache.copy_(torch.from_numpy(kc))
        value_cache.copy_(torch.from_numpy(vc))
        b, h, d = q.shape
        return torch.from_numpy(out).float().reshape(b, 1, h * d)

    def cross_step(query, key_cache, value_cache, scale=None):
        q = query[:, :, 0] if query.dim() == 4 else query
        out = oracle.whisper_cross_attention(q.numpy(), key_cache.numpy(), value_cache.numpy())
        b, h, d = q.shape
        return torch.from_numpy(out).float().reshape(b, 1, h * d)

    def self_prefix(query, key_cache, value_cache, scale=None):
        b, h, p, d = query.shape
        mask = np.arange(key_cache.shape[2])[None, :] <= np.arange(p)[:, None]
        out = oracle.sdpa(query.numpy(), key_cache.numpy(), value_cache.numpy(), mask)
        return torch.from_numpy(out).float().transpose(1, 2).reshape(b, p, h * d)

    def cross_prefix(query, key_cache, value_cache, scale=None):
        b, h, p, d = query.shape
        out = oracle.whisper_cross_attention_prefix(query.numpy(), key_cache.numpy(),
                                                    value_cache.numpy())
        return torch.from_numpy(out).float().transpose(1, 2).reshape(b, p, h * d)

    def encoder(q, k, v, scale=None):
        out = oracle.encoder_attention(q.numpy(), k.numpy(), v.numpy())
        b, h, s, d = q.shape
        return torch.from_numpy(out).float().transpose(1, 2).reshape(b, s, h * d)

    def qwen3_step(qkv, qn, kn, eps, cos, sin, positions, keys, values, heads, kv_heads,
                   scale=None):
        out, kc, vc = oracle.qwen3_decode_attention(
            qkv.detach().numpy(), qn.detach().numpy(), kn.detach().numpy(), eps, cos.numpy(),
            sin.numpy(), positions.numpy(), keys.numpy(), values.numpy(), heads, kv_heads)
        keys.copy_(torch.from_numpy(kc))
        values.copy_(torch.from_numpy(vc))
        return torch.from_numpy(out).float()

    def varlen(q, k, v, starts, longest, causal, scale=None):
        out = oracle.varlen_attention(q.detach().numpy(), k.detach().numpy(), v.detach().numpy(),
                                      starts.numpy(), causal)
        return torch.from_numpy(out).float()

    def cross_kv(x, wk, wv, bv, keys, values):
        k, v = oracle.cross_kv_projection(
            x.detach().float().numpy(), wk.detach().float().numpy(), wv.detach().float().numpy(),
            None if bv is None else bv.detach().float().numpy())
        tokens = x.shape[1]
        keys[:, :, :tokens].copy_(torch.from_numpy(k))
        values[:, :, :tokens].copy_(torch.from_numpy(v))

    monkeypatch.setattr(attention, "whisper_cross_kv_projection", cross_kv)
    monkeypatch.setattr(attention, "varlen_attention", varlen)
    monkeypatch.setattr(attention, "whisper_self_attention_step", self_step)
    monkeypatch.setattr(attention, "whisper_cross_attention_step", cross_step)
    monkeypatch.setattr(attention, "whisper_self_attention_prefix", self_prefix)
    monkeypatch.setattr(attention, "whisper_cross_attention_prefix", cross_prefix)
    monkeypatch.setattr(attention, "whisper_encoder_attention", encoder)
    monkeypatch.setattr(attention, "qwen3_attention_step", qwen3_step)
    yield
    plugin.uninstall()


def _whisper(whisper):
    config = dict(d_model=128, encoder_attention_heads=2, decoder_attention_heads=2,
                  encoder_layers=1, decoder_layers=2, encoder_ffn_dim=64, decoder_ffn_dim=64,
                  num_mel_bins=8, max_source_positions=24, max_target_positions=32, vocab_size=50)
    model = whisper.WhisperForConditionalGeneration(config).eval()
    seeded_parameters(model, 5)
    return model


@torch.no_grad()
def test_whisper_decoder_step(reference, cpu_ops):
    whisper, _ = reference
    model = _whisper(whisper)
    positions = torch.tensor([0, 3, 31])
    tokens = torch.tensor([[1], [7], [49]])

    def run():
        cache = model.allocate_cache(3)
        model.set_encoder_output(cache, seeded_normal((3, 24, 128), 1))
        for layer in range(2):
            cache.self_keys[layer].copy_(seeded_normal(cache.self_keys[layer].shape, 10 + layer))
            cache.self_values[layer].copy_(seeded_normal(cache.self_values[layer].shape, 20 + layer))
        hidden = model.decode(tokens, positions, cache)
        return hidden, cache

    want, want_cache = run()
    plugin.install(whisper, None)
    got, got_cache = run()
    assert torch.allclose(got, want, atol=1e-4), (got - want).abs().max()
    # Later layers' keys differ in the last bits (their inputs carry the first
    # layer's float64-oracle vs float32-SDPA difference).
    assert torch.allclose(got_cache.self_keys, want_cache.self_keys, atol=1e-5)
    assert torch.allclose(got_cache.self_values, want_cache.self_values, atol=1e-5)


@torch.no_grad()
def test_whisper_prefix_pass(reference, cpu_ops):
    """The eager pass with length == its token count (the prompt pass and
    language detection) runs on the prefix ops: same hidden states and cache
    as the reference's own code."""
    whisper, _ = reference
    model = _whisper(whisper)
    want_cache, got_cache = model.allocate_cache(2), model.allocate_cache(2)
    states = seeded_normal((2, 24, 128), 1)
    model.set_encoder_output(want_cache, states)
    tokens = torch.tensor([[1, 2, 3], [4, 5, 6]])
    want = [model.decode(tokens[:, :1], torch.arange(1), want_cache, length=1),
            model.decode(tokens, torch.arange(3), want_cache, length=3)]
    plugin.install(whisper, None)
    model.set_encoder_output(got_cache, states)
    got = [model.decode(tokens[:, :1], torch.arange(1), got_cache, length=1),
           model.decode(tokens, torch.arange(3), got_cache, length=3)]
    for g, w in zip(got, want):
        assert torch.allclose(g, w, atol=1e-4), (g - w).abs().max()
    assert torch.allclose(got_cache.self_keys, want_cache.self_keys, atol=1e-5)
    assert torch.allclose(got_cache.self_values, want_cache.self_values, atol=1e-5)


@torch.no_grad()
def test_whisper_eager_other_lengths_keep_reference_path(reference, cpu_ops):
    """An eager call whose length differs from its token count is not the
    plugin's: it runs the reference's own code, results unchanged."""
    whisper, _ = reference
    model = _whisper(whisper)
    cache = model.allocate_cache(2)
    model.set_encoder_output(cache, seeded_normal((2, 24, 128), 1))
    tokens = torch.tensor([[1, 2, 3], [4, 5, 6]])
    want = model.decode(tokens, torch.arange(3), cache, length=5)
    plugin.install(whisper, None)
    got = model.decode(tokens, torch.arange(3), cache, length=5)
    assert torch.equal(got, want)


@torch.no_grad()
def test_whisper_encoder_attention(reference, cpu_ops):
    whisper, _ = reference
    module = whisper.MultiHeadAttention(128, 2).eval()
    seeded_parameters(module, 6)
    x = seeded_normal((2, 40, 128), 2)
    want = module(x)
    plugin.install(whisper, None)
    got = module(x)
    assert torch.allclose(got, want, atol=1e-4), (got - want).abs().max()


@torch.no_grad()
def test_qwen3_text_model_step(reference, cpu_ops):
    _, qwen3 = reference
    config = dict(vocab_size=64, hidden_size=256, num_hidden_layers=2, num_attention_heads=16,
                  num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, intermediate_size=64)
    model = qwen3.TextModel(config).eval()
    seeded_parameters(model, 7)
    inverse = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    angles = torch.arange(48).float()[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    cos, sin = angles.cos(), angles.sin()
    positions = torch.tensor([0, 17, 47])
    tokens = torch.tensor([3, 9, 60])

    def run():
        keys = seeded_normal((2, 3, 48, 8, 128), 30)
        values = seeded_normal((2, 3, 48, 8, 128), 31)
        cache = qwen3.KVCache(keys, values)
        return model.step(tokens, positions, cache, cos, sin, varlen=False), cache

    want, want_cache = run()
    plugin.install(None, qwen3)
    got, got_cache = run()
    assert torch.allclose(got, want, atol=1e-4), (got - want).abs().max()
    rows = np.arange(3)
    np.testing.assert_allclose(got_cache.keys.numpy()[:, rows, positions.numpy()],
                               want_cache.keys.numpy()[:, rows, positions.numpy()], atol=1e-5)
    assert torch.allclose(got_cache.values, want_cache.values, atol=1e-5)


@torch.no_grad()
def test_qwen3_prefill_and_audio_attention(reference, cpu_ops):
    """TextAttention.prefill (causal, grouped-query, cache writes) and
    AudioAttention.forward (non-causal windows) through the patched attend."""
    _, qwen3 = reference
    config = dict(vocab_size=64, hidden_size=256, num_hidden_layers=1, num_attention_heads=16,
                  num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, intermediate_size=64)
    text = qwen3.TextAttention(config).eval()
    seeded_parameters(text, 8)
    audio = qwen3.AudioAttention(128, 2).eval()
    seeded_parameters(audio, 9)
    lengths = [5, 17, 1]
    tokens = sum(lengths)
    rows = torch.tensor([0] * 5 + [1] * 17 + [2])
    positions = torch.cat([torch.arange(n) for n in lengths])
    inverse = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    angles = positions.float()[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    cos, sin = angles.cos(), angles.sin()
    x = seeded_normal((tokens, 256), 40)
    xa = seeded_normal((tokens, 128), 41)

    def run():
        keys = torch.zeros((3, 20, 8, 128))
        values = torch.zeros_like(keys)
        segments = qwen3.Segments.from_lengths(lengths, torch.device("cpu"), False)
        out = text.prefill(x, keys, values, rows, positions, segments, cos, sin)
        return out, keys, values, audio(xa, segments)

    want = run()
    plugin.install(None, qwen3)
    assert qwen3.attend is not None and qwen3.attend.__name__ == "_qwen3_attend"
    got = run()
    for a, b in zip(got, want):
        assert torch.allclose(a, b, atol=1e-4), (a - b).abs().max()


@pytest.fixture
def cpu_step(monkeypatch):
    """Oracle-backed stand-in for ``step.greedy_step`` (same signature and
    in-place state update)."""
    from asrback_b200 import step
    from oracle import step as oracle_step

    calls = []

    def greedy_step(hidden, weight, tokens, position, end, finished, sum_logprobs, generated,
                    eos_ids, suppress=None):
        calls.append(tuple(hidden.shape))
        logits = oracle_step.logits(weight.detach().float().numpy(),
                                    hidden.detach().float().numpy(),
                                    hidden.dtype == torch.bfloat16)
        token, logprob = oracle_step.choose(logits, None if suppress is None else suppress.numpy())
        new = oracle_step.update_state(
            dict(tokens=tokens.reshape(-1).numpy(), position=position.numpy(), end=end.numpy(),
                 finished=finished.numpy(), sum_logprobs=sum_logprobs.numpy(),
                 generated=generated.numpy()), token, logprob, eos_ids)
        tokens.copy_(torch.from_numpy(new["tokens"]).reshape(tokens.shape))
        position.copy_(torch.from_numpy(new["position"]))
        finished.copy_(torch.from_numpy(new["finished"]))
        sum_logprobs.copy_(torch.from_numpy(new["sum_logprobs"]))
        generated.copy_(torch.from_numpy(new["generated"]))

    monkeypatch.setattr(step, "greedy_step", greedy_step)
    return calls


def _whisper_engine(whisper, hiddens):
    """A Transcriber stand-in: the reference's ``logits`` over a seeded
    embedding, its ``_choose``, and a decoder returning ``hiddens`` in turn."""
    import types

    config = dict(d_model=64, encoder_attention_heads=2, decoder_attention_heads=2,
                  encoder_layers=1, decoder_layers=1, encoder_ffn_dim=32, decoder_ffn_dim=32,
                  num_mel_bins=80, max_source_positions=40, max_target_positions=48,
                  vocab_size=3000)
    model = whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, 21)
    queue = list(hiddens)
    engine = types.SimpleNamespace(_eos=2999, _suppress=torch.arange(3000) % 7 == 3)
    engine.model = types.SimpleNamespace(decode=lambda *args: queue.pop(0), logits=model.logits,
                                         model=model.model)
    engine._choose = types.MethodType(whisper.Transcriber._choose, engine)
    state = whisper._DecodeState.allocate(5, 48, torch.device("cpu"))
    state.tokens[:, 0] = torch.tensor([5, 6, 7, 8, 9])
    state.position[:] = torch.tensor([3, 10, 46, 0, 20])
    state.end[:] = torch.tensor([47, 47, 47, 0, 47])
    state.finished[:] = torch.tensor([False, False, False, True, False])
    return engine, state


def _qwen3_engine(qwen3, hiddens):
    import types

    lm_head = torch.nn.Linear(64, 2000, bias=False)
    seeded_parameters(lm_head, 22)
    queue = list(hiddens)
    engine = types.SimpleNamespace(_lm_head=lm_head, _eos_ids=torch.tensor([1990, 1999]),
                                   _cos=None, _sin=None, _varlen=False)
    engine._text = types.SimpleNamespace(step=lambda *args: queue.pop(0))
    engine._choose = types.MethodType(qwen3.Qwen3ASRTranscriber._choose, engine)
    state = qwen3._DecodeState.allocate(4, torch.device("cpu"))
    state.tokens[:] = torch.tensor([1, 2, 3, 4])
    state.position[:] = torch.tensor([0, 500, 1022, 7])
    state.end[:] = torch.tensor([1023, 1023, 1023, 1023])
    state.finished[:] = torch.tensor([False, False, False, True])
    return engine, state


@pytest.mark.parametrize("family", ["whisper", "qwen3"])
def test_transcriber_greedy_step(reference, cpu_step, family):
    """The patched ``_step`` hands the decoder's last hidden state, the logits
    weight, the suppress mask and the EOS ids to the fused step and leaves the
    same decode state as the reference's own ``_step``."""
    whisper, qwen3 = reference
    module = whisper if family == "whisper" else qwen3
    cls = whisper.Transcriber if family == "whisper" else qwen3.Qwen3ASRTranscriber
    make = _whisper_engine if family == "whisper" else _qwen3_engine
    shape = (5, 1, 64) if family == "whisper" else (4, 64)
    hiddens = [seeded_normal(shape, 700 + i) * 3 for i in range(4)]
    engine, want = make(module, [h.clone() for h in hiddens])
    with torch.no_grad():
        for _ in hiddens:
            cls._step(engine, want, None, None)
    plugin.install(whisper, qwen3)
    try:
        engine, got = make(module, [h.clone() for h in hiddens])
        with torch.no_grad():
            for _ in hiddens:
                cls._step(engine, got, None, None)
    finally:
        plugin.uninstall()
    assert len(cpu_step) == len(hiddens)
    for name in ("tokens", "position", "finished", "generated"):
        assert torch.equal(getattr(got, name), getattr(want, name)), name
    torch.testing.assert_close(got.sum_logprobs, want.sum_logprobs, atol=1e-5, rtol=0)
    assert want.finished.sum() > 1  # an EOS or an end was reached


def test_transcriber_sampling_step_keeps_reference_path(reference, cpu_step):
    """A step with temperatures goes to the reference's own ``_step``."""
    whisper, qwen3 = reference
    engine, state = _whisper_engine(whisper, [seeded_normal((5, 1, 64), 710)])
    plugin.install(whisper, qwen3)
    try:
        torch.manual_seed(0)
        with torch.no_grad():
            whisper.Transcriber._step(engine, state, None, torch.full((5,), 0.7))
    finally:
        plugin.uninstall()
    assert cpu_step == []


def test_uninstall_restores_reference(reference):
    whisper, qwen3 = reference
    before = (whisper.DecoderLayer.forward, whisper.MultiHeadAttention.forward,
              qwen3.TextAttention.step, qwen3.TextModel.step, qwen3.attend,
              whisper.Transcriber._step, qwen3.Qwen3ASRTranscriber._step,
              whisper.WhisperForConditionalGeneration.set_encoder_output)
    plugin.install(whisper, qwen3)
    assert plugin.installed()
    assert whisper.DecoderLayer.forward is not before[0]
    assert qwen3.attend is not before[4]
    plugin.uninstall()
    after = (whisper.DecoderLayer.forward, whisper.MultiHeadAttention.forward,
             qwen3.TextAttention.step, qwen3.TextModel.step, qwen3.attend,
             whisper.Transcriber._step, qwen3.Qwen3ASRTranscriber._step,
             whisper.WhisperForConditionalGeneration.set_encoder_output)
    assert after == before


def test_install_without_encoder_keeps_reference_encoder_attention(reference):
    whisper, qwen3 = reference
    encoder_forward = whisper.MultiHeadAttention.forward
    decoder_forward = whisper.DecoderLayer.forward
    set_output = whisper.WhisperForConditionalGeneration.set_encoder_output
    plugin.install(whisper, qwen3, encoder=False)
    try:
        assert whisper.MultiHeadAttention.forward is encoder_forward
        assert whisper.DecoderLayer.forward is not decoder_forward
        assert whisper.WhisperForConditionalGeneration.set_encoder_output is not set_output
    finally:
        plugin.uninstall()
    assert whisper.DecoderLayer.forward is decoder_forward
    assert whisper.WhisperForConditionalGeneration.set_encoder_output is set_output
