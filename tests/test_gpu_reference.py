"""The reference's own classes on the GPU with ``asrback_b200.plugin``
installed: its models, its ``Transcriber`` engine and its ``CapturedGraph``
run the patched call sites on the sm_100a kernels, against fixtures that
``tests/golden/make_golden.py`` recorded by running the same classes unpatched
on the CPU.

The reference (pure Python) is imported from ``$ASRBACK_REFERENCE`` or
``baseline/_ref`` (``oracle/reference.py``); every test here skips without it.

Tolerances: float32 encoder output 1e-4 and decoder hidden states 1e-3
(max-abs); bf16 hidden states within ``BF16_HIDDEN`` of the CPU bf16 run
(max-abs relative to the largest element: the CPU and GPU round their bf16
GEMMs differently at every layer); greedy tokens identical on >= 99 % of the
steps (teacher-forced on the reference's tokens where a step's choice would
otherwise feed the next); in bf16, a step may differ only where the
reference's own two largest logits lie within 4 bf16 steps of each other
(exact ties are common at bf16 resolution).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from asrback_b200 import attention, plugin
from oracle import reference as reference_env
from tests import reference_models as rm
from tests.golden import load

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(reference_env.find() is None,
                       reason="asrback reference not found ($ASRBACK_REFERENCE or baseline/_ref)"),
]

DEV = torch.device("cuda", 0)
BF16_HIDDEN = 5e-2


@pytest.fixture(scope="module")
def ref():
    """The reference's modules with the plugin installed on them."""
    loaded = reference_env.load()
    plugin.install(loaded.whisper, loaded.qwen3_asr)
    cudnn_tf32 = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False  # float32 convolutions stay float32
    yield loaded
    torch.backends.cudnn.allow_tf32 = cudnn_tf32
    plugin.uninstall()


@pytest.fixture(autouse=True)
def clean_status():
    attention.read_status()
    yield


def _relative(got: np.ndarray, want: np.ndarray) -> float:
    return float(np.abs(got - want).max() / np.abs(want).max())


def _bf16_ulp(x: np.ndarray) -> np.ndarray:
    """The spacing of bf16 numbers at ``|x|`` (8 significant bits)."""
    return np.exp2(np.floor(np.log2(np.maximum(np.abs(x), 1e-30))) - 7)


def _assert_greedy_tokens(got: np.ndarray, want: np.ndarray, top2: np.ndarray,
                          ulps: int = 4) -> None:
    """Greedy tokens identical on >= 99 % of the steps, or else every step that
    differs is a near-tie of the reference's own bf16 logits: its two largest
    logits within ``ulps`` bf16 steps of each other (bf16 logits tie exactly
    on some steps, and argmax then takes the lower id). At least 90 % of the
    steps must be identical either way."""
    same = got == want
    assert same.mean() >= 0.9, same.mean()
    if same.mean() >= 0.99:
        return
    margin = top2[..., 0] - top2[..., 1]
    tie = margin <= ulps * _bf16_ulp(top2[..., 0])
    assert (same | tie).all(), (np.argwhere(~same).tolist(), margin[~same].tolist())


# ------------------------------------------------------------- config 1 ----

def test_config1_model_through_plugin(ref):
    """BASELINE config 1 on the reference's classes: the encoder over the mel
    batch, ``set_encoder_output``, the 4-token prompt pass, then 64 greedy
    ``Transcriber._step`` calls replayed from the reference's
    ``CapturedGraph``; float32 on the GPU against the CPU run."""
    g = load("whisper_config1_model")
    model, mel = rm.whisper_config1(ref)
    out = rm.run_whisper_steps(ref, model.to(DEV), mel.to(DEV), rm.CONFIG1_STEPS, graph=True)
    assert attention.read_status() == 0
    assert np.abs(out["encoder_sample"] - g["encoder_sample"]).max() <= 1e-4
    assert np.abs(out["prompt_hidden"] - g["prompt_hidden"]).max() <= 1e-3
    assert np.abs(out["hidden"] - g["hidden"]).max() <= 1e-3
    np.testing.assert_array_equal(out["first_token"], g["first_token"])
    same = out["generated"] == g["generated"]
    assert same.mean() >= 0.99, same.mean()
    np.testing.assert_array_equal(out["position"], g["position"])
    np.testing.assert_array_equal(out["finished"], g["finished"])
    np.testing.assert_allclose(out["sum_logprobs"], g["sum_logprobs"], atol=1e-3, rtol=0)


def test_config1_engine_through_plugin(ref, tmp_path):
    """The reference's ``Transcriber`` (float32, CUDA graphs on: one graph per
    (batch, self-attention length) bucket, captured in ascending batch order)
    loads config 1's weights, takes the eight windows through its worker
    (language detection for two, a longer prompt for two) and returns the
    same results as on the CPU."""
    g = load("whisper_config1_engine")
    model, mel = rm.whisper_config1(ref)
    directory = rm.write_whisper_model_dir(tmp_path / "whisper-config1", model)
    transcriber = ref.whisper.Transcriber(directory, device="cuda:0", dtype="float32",
                                          max_batch_size=8, batch_wait_ms=500.0,
                                          cuda_graphs=True)
    assert len(transcriber._graphs) == 16
    results = rm.submit_whisper_jobs(ref, transcriber, mel.numpy(), g["meta"]["max_new_tokens"])
    assert attention.read_status() == 0
    assert [r["language"] for r in results] == g["meta"]["languages"]
    for index, result in enumerate(results):
        want = g["tokens"][index, :g["lengths"][index]].tolist()
        assert result["tokens"] == want, index
    np.testing.assert_allclose([r["avg_logprob"] for r in results], g["avg_logprob"], atol=1e-4,
                               rtol=0)
    np.testing.assert_allclose([r["no_speech_prob"] for r in results], g["no_speech_prob"],
                               atol=1e-4, rtol=0)


# --------------------------------------------------- production widths ----

def test_whisper_turbo_decoder_graph_bf16(ref):
    """The reference's decoder at large-v3-turbo widths (4 layers, bf16):
    ``set_encoder_output``, the prompt pass, ragged rows, then 24 fixed-shape
    steps over the 64-position bucket view replayed from its
    ``CapturedGraph``, teacher-forced on the CPU run's tokens."""
    g = load("whisper_turbo_decode_bf16")
    model = rm.whisper_turbo_decoder(ref, torch.bfloat16, DEV)
    forced = torch.from_numpy(g["tokens"]).to(DEV)
    out = rm.run_turbo_steps(ref, model, forced, graph=True)
    assert attention.read_status() == 0
    assert _relative(out["prompt_hidden"], g["prompt_hidden"]) <= BF16_HIDDEN
    assert _relative(out["hidden"], g["hidden"]) <= BF16_HIDDEN, _relative(out["hidden"],
                                                                         g["hidden"])
    assert _relative(out["self_keys"], g["self_keys"]) <= BF16_HIDDEN
    _assert_greedy_tokens(out["argmax"], g["argmax"], g["top2"])
    # The unpatched reference on the same GPU (torch SDPA, cuDNN first): only
    # the attention differs between the two runs.
    plugin.uninstall()
    try:
        torch_run = rm.run_turbo_steps(ref, model, forced, graph=True)
    finally:
        plugin.install(ref.whisper, ref.qwen3_asr)
    assert _relative(out["hidden"], torch_run["hidden"]) <= BF16_HIDDEN
    _assert_greedy_tokens(out["argmax"], torch_run["argmax"], torch_run["top2"])


def test_qwen3_text_model_graph_bf16(ref):
    """The reference's ``TextModel`` at Qwen3-1.7B widths (4 layers, bf16):
    packed causal prefill of four ragged prompts (patched ``attend``: the
    varlen kernel), then 16 ``TextModel.step`` calls (patched: the fused
    decode kernel) over the 512-position bucket view replayed from its
    ``CapturedGraph``, teacher-forced on the CPU run's tokens."""
    g = load("qwen3_graph_decode_bf16")
    model, lm_head = rm.qwen3_text_model(ref, torch.bfloat16, DEV)
    forced = torch.from_numpy(g["tokens"]).to(DEV)
    out = rm.run_qwen3_steps(ref, model, lm_head, forced, graph=True)
    assert attention.read_status() == 0
    assert _relative(out["prefill_last"], g["prefill_last"]) <= BF16_HIDDEN
    assert _relative(out["hidden"], g["hidden"]) <= BF16_HIDDEN, _relative(out["hidden"],
                                                                         g["hidden"])
    _assert_greedy_tokens(out["argmax"], g["argmax"], g["top2"])
    # The unpatched reference on the same GPU (padded-SDPA prefill, masked
    # SDPA steps: its torch 2.11 path).
    plugin.uninstall()
    try:
        torch_run = rm.run_qwen3_steps(ref, model, lm_head, forced, graph=True)
    finally:
        plugin.install(ref.whisper, ref.qwen3_asr)
    assert _relative(out["hidden"], torch_run["hidden"]) <= BF16_HIDDEN
    _assert_greedy_tokens(out["argmax"], torch_run["argmax"], torch_run["top2"])


# ------------------------------------------------ seeded small decoders ----

def _dev(a, dtype=torch.int64):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def test_whisper_tiny_greedy_steps_match_reference(ref):
    """Whisper-tiny decoder (fp32, seeded weights) over the fixture's ragged
    rows: hidden states within 1e-3 and argmax tokens identical on >= 99% of
    the steps (teacher-forced on the reference's tokens)."""
    from asrback_b200.synthetic import seeded_normal, seeded_parameters

    g = load("whisper_tiny_decode")
    meta = g["meta"]
    config = dict(meta["config"], encoder_layers=1)
    model = ref.whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, meta["seed"])
    model = model.to(DEV).eval()
    batch = len(meta["prompts"])
    cache = model.allocate_cache(batch)
    with torch.inference_mode():
        model.set_encoder_output(cache, seeded_normal((batch, 1500, 384),
                                                      meta["encoder_seed"]).to(DEV))
        for b, prompt in enumerate(meta["prompts"]):
            row = cache.rows(b, b + 1)
            for p, token in enumerate(prompt[:-1]):
                model.decode(torch.tensor([[token]], device=DEV), torch.tensor([p], device=DEV),
                             row)
        hidden_err, same = [], []
        for t in range(meta["steps"]):
            hidden = model.decode(_dev(g["tokens"][:, t:t + 1]), _dev(g["positions"][:, t]),
                                  cache)[:, -1]
            choice = model.logits(hidden).float().argmax(dim=-1)
            hidden_err.append(np.abs(hidden.float().cpu().numpy() - g["hidden"][:, t]).max())
            same.append(choice.cpu().numpy() == g["argmax"][:, t])
    assert attention.read_status() == 0
    assert max(hidden_err) < 1e-3, max(hidden_err)
    assert np.mean(same) >= 0.99, np.mean(same)


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_whisper_prefix_pass_matches_reference_decoder(ref, tag):
    """The patched eager pass (``decode(tokens, positions[:P], cache,
    length=P)``): language detection then the prompt pass of a 1-layer
    decoder with seeded weights; hidden states and cache keys against the
    reference's CPU run."""
    from asrback_b200.synthetic import seeded_normal, seeded_parameters

    dtype = torch.float32 if tag == "fp32" else torch.bfloat16
    g = load(f"whisper_prefix_{tag}")
    meta = g["meta"]
    batch, tokens = meta["batch"], meta["tokens"]
    model = ref.whisper.WhisperForConditionalGeneration(meta["config"])
    seeded_parameters(model.model.decoder, 1)
    model = model.to(DEV, dtype).eval()
    cache = model.allocate_cache(batch)
    positions = torch.arange(48, device=DEV)
    tol = 1e-3 if dtype == torch.float32 else 6e-2
    with torch.inference_mode():
        model.set_encoder_output(cache, seeded_normal((batch, 40, 384), 12).to(DEV, dtype))
        hidden = model.decode(torch.full((batch, 1), 5, device=DEV), positions[:1], cache,
                              length=1)
        np.testing.assert_allclose(hidden.float().cpu().numpy(), g["detect_hidden"], atol=tol,
                                   rtol=0)
        prompt = torch.arange(batch * tokens, device=DEV).view(batch, tokens) % 128
        hidden = model.decode(prompt, positions[:tokens], cache, length=tokens)
        np.testing.assert_allclose(hidden.float().cpu().numpy(), g["prompt_hidden"], atol=tol,
                                   rtol=0)
        np.testing.assert_allclose(cache.self_keys[0, :, :, :tokens].float().cpu().numpy(),
                                   g["prompt_self_k"], atol=tol, rtol=0)
    assert attention.read_status() == 0


def test_whisper_prefix_pass_equals_token_steps(ref):
    """Size-independent property: the prompt pass over P tokens gives each
    token the hidden state, and the cache the keys, that P one-token steps
    give it (fp32, Whisper large-v3-turbo widths, 2 layers, P = 40)."""
    from asrback_b200.synthetic import seeded_normal, seeded_parameters

    config = dict(rm.WHISPER_TURBO_4L, decoder_layers=2)
    model = ref.whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, 3)
    model = model.to(DEV).eval()
    batch, tokens = 4, 40
    prompt = torch.randint(0, 51866, (batch, tokens),
                           generator=torch.Generator().manual_seed(4)).to(DEV)
    positions = torch.arange(448, device=DEV)
    with torch.inference_mode():
        states = seeded_normal((batch, 1500, 1280), 5).to(DEV)
        pass_cache, step_cache = model.allocate_cache(batch), model.allocate_cache(batch)
        model.set_encoder_output(pass_cache, states)
        model.set_encoder_output(step_cache, states)
        together = model.decode(prompt, positions[:tokens], pass_cache, length=tokens)
        steps = torch.stack([
            model.decode(prompt[:, t:t + 1], positions[t].expand(batch), step_cache)[:, 0]
            for t in range(tokens)], dim=1)
    np.testing.assert_allclose(together.cpu().numpy(), steps.cpu().numpy(), atol=1e-3, rtol=0)
    np.testing.assert_allclose(pass_cache.self_keys[:, :, :, :tokens].cpu().numpy(),
                               step_cache.self_keys[:, :, :, :tokens].cpu().numpy(), atol=1e-4,
                               rtol=0)
    assert attention.read_status() == 0


def _qwen3_small(ref, meta):
    from asrback_b200.synthetic import seeded_parameters

    config = dict(meta["config"], rope_theta=meta["rope_theta"])
    model = ref.qwen3_asr.TextModel(config)
    lm_head = torch.nn.Linear(config["hidden_size"], config["vocab_size"], bias=False)
    seeded_parameters(model, meta["seed"])
    seeded_parameters(lm_head, meta["lm_head_seed"])
    cos, sin = (t.to(DEV) for t in rm.rope_tables(meta["rope_theta"], 128, 1024))
    shape = (config["num_hidden_layers"], len(meta["prompts"]), 1024, 8, 128)
    cache = ref.qwen3_asr.KVCache(torch.zeros(shape, device=DEV), torch.zeros(shape, device=DEV))
    return model.to(DEV).eval(), lm_head.to(DEV), cos, sin, cache


def _qwen3_steps(model, lm_head, g, cache, cos, sin):
    hidden_err, same = [], []
    for t in range(g["meta"]["steps"]):
        hidden = model.step(_dev(g["tokens"][:, t]), _dev(g["positions"][:, t]), cache, cos, sin,
                            False)
        choice = lm_head(hidden).argmax(dim=-1)
        hidden_err.append(np.abs(hidden.float().cpu().numpy() - g["hidden"][:, t]).max())
        same.append(choice.cpu().numpy() == g["argmax"][:, t])
    return hidden_err, same


def test_qwen3_small_greedy_steps_match_reference(ref):
    g = load("qwen3_small_decode")
    model, lm_head, cos, sin, cache = _qwen3_small(ref, g["meta"])
    with torch.inference_mode():
        for b, prompt in enumerate(g["meta"]["prompts"]):
            row = ref.qwen3_asr.KVCache(cache.keys[:, b:b + 1], cache.values[:, b:b + 1])
            for p, token in enumerate(prompt[:-1]):
                model.step(torch.tensor([token], device=DEV), torch.tensor([p], device=DEV), row,
                           cos, sin, False)
        hidden_err, same = _qwen3_steps(model, lm_head, g, cache, cos, sin)
    assert attention.read_status() == 0
    assert max(hidden_err) < 1e-3, max(hidden_err)
    assert np.mean(same) >= 0.99, np.mean(same)


def test_qwen3_small_packed_prefill_then_steps_match_reference(ref):
    """The prompts filled by one packed causal prefill (the reference's
    ``TextModel.prefill``, patched ``attend`` on the varlen kernel) instead of
    one position per step, then the same greedy steps: the same hidden states
    and tokens as the reference."""
    g = load("qwen3_small_decode")
    model, lm_head, cos, sin, cache = _qwen3_small(ref, g["meta"])
    prompts = [prompt[:-1] for prompt in g["meta"]["prompts"]]
    lengths = [len(prompt) for prompt in prompts]
    tokens = torch.tensor([t for prompt in prompts for t in prompt], device=DEV)
    rows = torch.tensor([b for b, n in enumerate(lengths) for _ in range(n)], device=DEV)
    positions = torch.cat([torch.arange(n) for n in lengths]).to(DEV)
    segments = ref.qwen3_asr.Segments.from_lengths(lengths, DEV, False)
    with torch.inference_mode():
        model.prefill(model.embed_tokens(tokens), cache, rows, positions, segments,
                      cos[positions], sin[positions])
        hidden_err, same = _qwen3_steps(model, lm_head, g, cache, cos, sin)
    assert attention.read_status() == 0
    assert max(hidden_err) < 1e-3, max(hidden_err)
    assert np.mean(same) >= 0.99, np.mean(same)
