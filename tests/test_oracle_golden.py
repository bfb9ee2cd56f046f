"""Pins the CPU oracle (oracle/attention.py) to the reference's own outputs.

The fixtures in tests/golden were recorded from the reference's modules
(asrback, torch CPU) by tests/golden/make_golden.py. Every oracle function the
GPU parity tests compare against is checked here first.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import attention as oracle
from tests.golden import load

# Oracle (float64) vs torch fp32: accumulation-order differences only.
F32_TOL = 2e-5
# vs torch bf16 outputs: one bf16 rounding of values of magnitude <~ 4.
BF16_TOL = 2e-2


@pytest.mark.parametrize("name", ["detect", "prompt"])
@pytest.mark.parametrize("tag,tol", [("fp32", F32_TOL), ("bf16", BF16_TOL)])
def test_whisper_prefix(tag, tol, name):
    """The eager pass (prompt, P = 7) and language detection (P = 1):
    index_copy_ at positions 0..P-1, then causal attention over the first P
    positions; cross-attention of every prompt token."""
    g = load(f"whisper_prefix_{tag}")
    q, k, v = g[f"{name}_self_q"], g[f"{name}_self_k"], g[f"{name}_self_v"]
    batch, heads, tokens, head_dim = q.shape
    # A cache longer than the pass, holding other values past it: they are
    # neither attended nor overwritten.
    rng = np.random.default_rng(0)
    cache_k = rng.standard_normal((batch, heads, 48, head_dim)).astype(np.float32)
    cache_v = rng.standard_normal((batch, heads, 48, head_dim)).astype(np.float32)
    out, k_after, v_after = oracle.whisper_self_attention_prefix(
        q, k, v, cache_k, cache_v, np.arange(tokens), tokens)
    np.testing.assert_allclose(out, g[f"{name}_self_out"], atol=tol, rtol=0)
    np.testing.assert_array_equal(k_after[:, :, :tokens], k)
    np.testing.assert_array_equal(k_after[:, :, tokens:], cache_k[:, :, tokens:])
    np.testing.assert_array_equal(v_after[:, :, :tokens], v)
    cross = oracle.whisper_cross_attention_prefix(g[f"{name}_cross_q"], g["cross_k"], g["cross_v"])
    np.testing.assert_allclose(cross, g[f"{name}_cross_out"], atol=tol, rtol=0)


@pytest.mark.parametrize("tag,tol", [("fp32", F32_TOL), ("bf16", BF16_TOL)])
def test_whisper_self_step(tag, tol):
    g = load(f"whisper_step_{tag}")
    out, k_after, v_after = oracle.whisper_self_attention_step(
        g["self_q"], g["self_k_new"], g["self_v_new"], g["self_k_before"], g["self_v_before"],
        g["positions"])
    # The step mask is "key position <= row position" (whisper.py:262-264).
    length = g["self_k_before"].shape[2]
    mask = np.arange(length)[None, :] <= g["positions"][:, None]
    np.testing.assert_array_equal(mask, g["self_mask"])
    np.testing.assert_allclose(out, g["self_out"], atol=tol, rtol=0)
    rows = np.arange(len(g["positions"]))
    np.testing.assert_array_equal(k_after[rows, :, g["positions"]], g["self_k_new"])
    untouched = np.ones(k_after.shape[:3], bool)
    untouched[rows, :, g["positions"]] = False
    np.testing.assert_array_equal(k_after[untouched], g["self_k_before"][untouched])
    np.testing.assert_array_equal(v_after[rows, :, g["positions"]], g["self_v_new"])


@pytest.mark.parametrize("tag,tol", [("fp32", F32_TOL), ("bf16", BF16_TOL)])
def test_whisper_cross_step(tag, tol):
    g = load(f"whisper_step_{tag}")
    out = oracle.whisper_cross_attention(g["cross_q"], g["cross_k"], g["cross_v"])
    np.testing.assert_allclose(out, g["cross_out"], atol=tol, rtol=0)


@pytest.mark.parametrize("tag,tol", [("fp32", F32_TOL), ("bf16", BF16_TOL)])
def test_encoder_attention(tag, tol):
    g = load(f"encoder_attention_{tag}")
    out = oracle.encoder_attention(g["q"], g["k"], g["v"])
    np.testing.assert_allclose(out, g["out"], atol=tol, rtol=0)


def test_rope_tables_match_reference_formula():
    for tag, bf16 in (("fp32", False), ("bf16", True)):
        g = load(f"qwen3_step_{tag}")
        cos, sin = oracle.rope_tables(g["meta"]["rope_theta"], 128, g["cos"].shape[0], bf16=bf16)
        # fp32 angles agree to an ulp or two (the power is evaluated differently).
        tol = 1e-2 if bf16 else 1e-5
        np.testing.assert_allclose(cos, g["cos"], atol=tol, rtol=0)
        np.testing.assert_allclose(sin, g["sin"], atol=tol, rtol=0)


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_qwen3_projection(tag):
    """q/k RMSNorm + RoPE (qwen3_asr.py:366-372): the keys the reference wrote
    and the queries it passed to SDPA."""
    g = load(f"qwen3_step_{tag}")
    bf16 = tag == "bf16"
    pos = g["positions"]
    q, k, v = oracle.qwen3_project(g["qkv"], 16, 8, 128, g["q_norm_weight"], g["k_norm_weight"],
                                   float(g["eps"]), g["cos"][pos], g["sin"][pos], bf16=bf16)
    # bf16: identical up to rare one-ulp flips from the rsqrt's last bit.
    q_tol, k_tol = (3e-2, 3e-2) if bf16 else (2e-5, 2e-5)
    sdpa_q = g["sdpa_q"].reshape(len(pos), 16, 128)
    np.testing.assert_allclose(q, sdpa_q, atol=q_tol, rtol=0)
    np.testing.assert_allclose(k, g["k_new"], atol=k_tol, rtol=0)
    np.testing.assert_array_equal(v, g["v_new"])
    if bf16:
        assert np.mean(q == sdpa_q) > 0.99 and np.mean(k == g["k_new"]) > 0.99


@pytest.mark.parametrize("tag,tol", [("fp32", F32_TOL), ("bf16", BF16_TOL)])
def test_qwen3_decode_attention(tag, tol):
    g = load(f"qwen3_step_{tag}")
    out, k_after, v_after = oracle.qwen3_decode_attention(
        g["qkv"], g["q_norm_weight"], g["k_norm_weight"], float(g["eps"]), g["cos"], g["sin"],
        g["positions"], g["k_before"], g["v_before"], 16, 8, bf16=tag == "bf16")
    length = g["k_before"].shape[1]
    mask = np.arange(length)[None, :] <= g["positions"][:, None]
    np.testing.assert_array_equal(mask, g["sdpa_mask"])
    np.testing.assert_allclose(out, g["out"], atol=tol, rtol=0)
    rows = np.arange(len(g["positions"]))
    np.testing.assert_allclose(k_after[rows, g["positions"]], g["k_new"],
                               atol=tol if tag == "bf16" else 2e-5, rtol=0)
    np.testing.assert_array_equal(v_after[rows, g["positions"]], g["v_new"])


@pytest.mark.parametrize("case", ["prefill", "audio"])
@pytest.mark.parametrize("tag,tol", [("fp32", F32_TOL), ("bf16", BF16_TOL)])
def test_varlen_attention(tag, tol, case):
    """attend() over packed segments (qwen3_asr.py:152-181): causal GQA
    prefill and non-causal audio windows."""
    g = load(f"qwen3_varlen_{tag}")
    meta = g["meta"]["cases"][case]
    starts = g[f"{case}_starts"]
    np.testing.assert_array_equal(np.diff(starts), meta["lengths"])
    out = oracle.varlen_attention(g[f"{case}_q"], g[f"{case}_k"], g[f"{case}_v"], starts,
                                  meta["causal"])
    np.testing.assert_allclose(out, g[f"{case}_out"], atol=tol, rtol=0)


def test_varlen_attention_causal_first_token_is_its_value():
    """A segment's first token sees only itself: its output is its value."""
    g = load("qwen3_varlen_fp32")
    starts = g["prefill_starts"]
    out = oracle.varlen_attention(g["prefill_q"], g["prefill_k"], g["prefill_v"], starts, True)
    group = g["prefill_q"].shape[1] // g["prefill_k"].shape[1]
    for a in starts[:-1]:
        np.testing.assert_allclose(out[a], np.repeat(g["prefill_v"][a], group, axis=0), atol=1e-12)


def test_bf16_round_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5e-3, 3.0e38, np.inf], np.float32)
    r = oracle.bf16_round(x)
    assert r[0] == 1.0
    assert r[1] == 1.0  # halfway between 1 and 1+2^-7: ties to even
    assert r[2] == np.float32(1.0078125)
    assert np.isinf(r[5])
    # Idempotent and within half an ulp.
    np.testing.assert_array_equal(oracle.bf16_round(r), r)


def test_model_fixtures_are_consistent():
    """The model-level fixtures hold ragged positions and varied tokens (a
    greedy decode that collapses to one token would pin little)."""
    for name in ("whisper_tiny_decode", "qwen3_small_decode"):
        g = load(name)
        assert len(np.unique(g["positions"][:, 0])) == g["positions"].shape[0]
        assert len(np.unique(g["argmax"])) > 20
        np.testing.assert_array_equal(g["tokens"][:, 1:], g["argmax"][:, :-1])


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
@pytest.mark.parametrize("family", ["whisper", "qwen3"])
def test_step_epilogue(family, tag):
    """Three greedy ``_step`` calls of the reference's Transcriber: the oracle's
    logits, ``_choose`` and state update give the same tokens, log-probabilities
    and state."""
    from oracle import step as oracle_step
    from tests.step_fixtures import initial_state, step_weight

    g = load(f"step_epilogue_{tag}")
    info = g["meta"][family]
    bf16 = tag == "bf16"
    weight = step_weight(family, g["meta"], bf16).float().numpy()
    suppress = g.get(f"{family}_suppress")
    state = initial_state(g, family)
    for step in range(g["meta"]["steps"]):
        logits = oracle_step.logits(weight, g[f"{family}_hidden"][step], bf16)
        token, logprob = oracle_step.choose(logits, suppress)
        np.testing.assert_array_equal(token, g[f"{family}_token"][step])
        np.testing.assert_allclose(logprob, g[f"{family}_logprob"][step], atol=1e-4, rtol=0)
        state = oracle_step.update_state(state, token, logprob, info["eos"])
        for name in ("tokens", "position", "finished"):
            np.testing.assert_array_equal(state[name], g[f"{family}_after_{name}"][step])
        np.testing.assert_allclose(state["sum_logprobs"], g[f"{family}_after_sum_logprobs"][step],
                                   atol=1e-4, rtol=0)
    np.testing.assert_array_equal(state["generated"], g[f"{family}_generated"])
    # The fixture reaches every branch: an EOS, a row at its end, a free row.
    assert np.isin(g[f"{family}_token"], info["eos"]).any()
    finished = g[f"{family}_after_finished"]
    assert finished[-1].sum() > g[f"{family}_finished0"].sum() + 1
    assert (g[f"{family}_after_position"][-1] == g[f"{family}_position0"])[
        g[f"{family}_finished0"]].all()


@pytest.mark.parametrize("tag,tol", [("fp32", F32_TOL), ("bf16", BF16_TOL)])
def test_cross_kv_projection(tag, tol):
    """``set_encoder_output`` of the reference: each layer's k/v projections,
    split into heads, in the cache rows of the windows given; other rows as
    allocated."""
    from tests.step_fixtures import cross_kv_weights

    g = load(f"cross_kv_{tag}")
    batch = g["states"].shape[0]
    for index, (k_weight, v_weight, v_bias) in enumerate(
            cross_kv_weights(g["meta"]["config"], g["meta"]["seed"], bf16=tag == "bf16")):
        keys, values = oracle.cross_kv_projection(g["states"], k_weight, v_weight, v_bias,
                                                  bf16=tag == "bf16")
        length = keys.shape[2]
        np.testing.assert_allclose(keys, g["cross_keys"][index, :batch, :, :length], atol=tol, rtol=0)
        np.testing.assert_allclose(values, g["cross_values"][index, :batch, :, :length], atol=tol,
                                   rtol=0)
        assert not g["cross_keys"][index, batch:].any()
