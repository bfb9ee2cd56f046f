"""Generates the golden fixtures in this folder by running the reference's own
PyTorch modules (asrback, imported read-only) on CPU.

    python tests/golden/make_golden.py [--reference /path/to/asrback]

Without ``--reference`` the reference is looked up as ``oracle/reference.py``
describes (``$ASRBACK_REFERENCE``, then ``baseline/_ref``).

The reference imports ``asrfront`` (its audio front end), which is not
installed; none of the code run here calls into it, so a stub module with the
constants read at import time stands in for it. Each fixture records the
tensors at one attention call site: what the reference's modules passed to
``F.scaled_dot_product_attention`` and got back, plus the cache state around the
call. Two model-level fixtures record whole greedy decoder steps (hidden states
and argmax tokens) with weights from ``asrback_b200.synthetic.seeded_parameters``
so that the GPU tests can rebuild the same network without the reference.

Output: ``*.npz`` files; bf16 tensors are stored as their raw bits under
``<name>__bf16`` (``tests/golden/__init__.py`` decodes them to float32).
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from asrback_b200.synthetic import seeded_normal, seeded_parameters  # noqa: E402
from oracle import reference as reference_env  # noqa: E402
from oracle.reference import install_asrfront_stub  # noqa: E402,F401


class SdpaRecorder:
    """Wraps ``F.scaled_dot_product_attention`` and records every call."""

    def __init__(self) -> None:
        self.calls: list[dict] = []
        self.original = F.scaled_dot_product_attention

    def __enter__(self):
        def recorded(q, k, v, attn_mask=None, *args, **kwargs):
            out = self.original(q, k, v, attn_mask=attn_mask, *args, **kwargs)
            self.calls.append(dict(q=q.detach().clone(), k=k.detach().clone(),
                                   v=v.detach().clone(),
                                   mask=None if attn_mask is None else attn_mask.detach().clone(),
                                   out=out.detach().clone(), kwargs=dict(kwargs)))
            return out

        F.scaled_dot_product_attention = recorded
        return self

    def __exit__(self, *exc):
        F.scaled_dot_product_attention = self.original


def f32(t: torch.Tensor) -> np.ndarray:
    """float32 array, or for bfloat16 tensors their raw bits (``uint16``)."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.float().numpy()


def save(name: str, meta: dict, **arrays) -> None:
    path = HERE / f"{name}.npz"
    # bfloat16 bits go under "<name>__bf16"; tests/golden/__init__.py decodes them.
    arrays = {(f"{key}__bf16" if value.dtype == np.uint16 else key): value
              for key, value in arrays.items()}
    np.savez_compressed(path, meta=np.array(json.dumps(meta)), **arrays)
    print(f"{path.name}: {path.stat().st_size / 1024:.0f} KB")


def whisper_step(whisper, dtype: torch.dtype, tag: str) -> None:
    """One fixed-shape decoder step (``WhisperDecoder.forward`` with
    ``length=None``) of a 1-layer decoder: self call (scatter, then masked
    SDPA) and cross call."""
    config = dict(d_model=384, encoder_attention_heads=6, decoder_attention_heads=6,
                  encoder_layers=1, decoder_layers=1, encoder_ffn_dim=64, decoder_ffn_dim=64,
                  num_mel_bins=80, max_source_positions=40, max_target_positions=48,
                  vocab_size=128)
    torch.manual_seed(0)
    model = whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, 0)
    model = model.to(dtype)
    batch = 4
    positions = torch.tensor([0, 7, 20, 47])
    cache = model.allocate_cache(batch)
    states = seeded_normal((batch, 40, 384), 11).to(dtype)
    with torch.no_grad():
        model.set_encoder_output(cache, states)
        for b, p in enumerate(positions.tolist()):
            filled = seeded_normal((1, 6, p, 64), 100 + b, 0.5).to(dtype)
            cache.self_keys[0, b, :, :p] = filled[0]
            cache.self_values[0, b, :, :p] = -filled[0].flip(-1)
        k_before = cache.self_keys[0].clone()
        v_before = cache.self_values[0].clone()
        tokens = torch.tensor([[3], [50], [77], [127]])
        with SdpaRecorder() as rec:
            model.decode(tokens, positions, cache)
    self_call, cross_call = rec.calls
    rows = torch.arange(batch)
    # The attended cache is the old one with the step's rows written (scatter_).
    expected = k_before.clone()
    expected[rows, :, positions] = self_call["k"][rows, :, positions]
    assert torch.equal(expected, self_call["k"])
    save(f"whisper_step_{tag}",
         dict(config=config, dtype=str(dtype), site="whisper.py:222-240"),
         positions=positions.numpy(),
         self_q=f32(self_call["q"][:, :, 0]),
         self_k_new=f32(self_call["k"][rows, :, positions]),
         self_v_new=f32(self_call["v"][rows, :, positions]),
         self_k_before=f32(k_before), self_v_before=f32(v_before),
         self_mask=self_call["mask"][:, 0, 0].numpy(),
         self_out=f32(self_call["out"][:, :, 0]),
         cross_q=f32(cross_call["q"][:, :, 0]), cross_k=f32(cross_call["k"]),
         cross_v=f32(cross_call["v"]), cross_out=f32(cross_call["out"][:, :, 0]))


def whisper_prefix(whisper, dtype: torch.dtype, tag: str) -> None:
    """The eager prompt pass (``decode(tokens, positions[:P], cache,
    length=P)``, ``whisper.py:847-849``) and language detection (the same with
    P = 1, ``whisper.py:979-981``) of a 1-layer decoder: the self call
    (``index_copy_``, then causal SDPA over the first P positions) and the
    cross call of each."""
    config = dict(d_model=384, encoder_attention_heads=6, decoder_attention_heads=6,
                  encoder_layers=1, decoder_layers=1, encoder_ffn_dim=64, decoder_ffn_dim=64,
                  num_mel_bins=80, max_source_positions=40, max_target_positions=48,
                  vocab_size=128)
    torch.manual_seed(0)
    model = whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, 1)
    model = model.to(dtype)
    batch, tokens = 3, 7
    cache = model.allocate_cache(batch)
    states = seeded_normal((batch, 40, 384), 12).to(dtype)
    positions = torch.arange(48)
    arrays = {}
    with torch.no_grad():
        model.set_encoder_output(cache, states)
        for name, prompt in (("detect", torch.full((batch, 1), 5)),
                             ("prompt", torch.arange(batch * tokens).view(batch, tokens) % 128)):
            length = prompt.shape[1]
            with SdpaRecorder() as rec:
                hidden = model.decode(prompt, positions[:length], cache, length=length)
            self_call, cross_call = rec.calls
            assert self_call["kwargs"].get("is_causal") == (length > 1)
            arrays.update({
                f"{name}_self_q": f32(self_call["q"]), f"{name}_self_k": f32(self_call["k"]),
                f"{name}_self_v": f32(self_call["v"]), f"{name}_self_out": f32(self_call["out"]),
                f"{name}_cross_q": f32(cross_call["q"]), f"{name}_cross_out": f32(cross_call["out"]),
                f"{name}_hidden": f32(hidden),
            })
        arrays["cross_k"] = f32(cross_call["k"])
        arrays["cross_v"] = f32(cross_call["v"])
    save(f"whisper_prefix_{tag}",
         dict(config=config, dtype=str(dtype), tokens=tokens, batch=batch,
              site="whisper.py:228-240 (eager branch), 847-849, 979-981"),
         **arrays)


def qwen3_step(qwen3, dtype: torch.dtype, tag: str) -> None:
    """One ``TextModel.step`` (bucket-mask path) of a 1-layer Qwen3 text model
    with 16 query / 8 key-value heads of 128."""
    config = dict(vocab_size=64, hidden_size=256, num_hidden_layers=1, num_attention_heads=16,
                  num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, intermediate_size=64)
    model = qwen3.TextModel(config)
    seeded_parameters(model, 3)
    model = model.to(dtype)
    batch, length = 4, 40
    positions = torch.tensor([0, 9, 25, 39])
    inverse = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    angles = torch.arange(length).float()[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    cos, sin = angles.cos().to(dtype), angles.sin().to(dtype)
    keys = torch.zeros((1, batch, length, 8, 128), dtype=dtype)
    values = torch.zeros_like(keys)
    for b, p in enumerate(positions.tolist()):
        filled = seeded_normal((p, 8, 128), 200 + b, 0.5).to(dtype)
        keys[0, b, :p] = filled
        values[0, b, :p] = filled.flip(-1) * 0.7
    cache = qwen3.KVCache(keys, values)
    k_before, v_before = keys[0].clone(), values[0].clone()
    attention = model.layers[0].self_attn
    captured = {}
    hooks = [
        attention.qkv_proj.register_forward_hook(lambda m, i, o: captured.__setitem__("qkv", o.clone())),
        attention.o_proj.register_forward_pre_hook(lambda m, i: captured.__setitem__("out", i[0].clone())),
    ]
    with torch.no_grad(), SdpaRecorder() as rec:
        model.step(torch.tensor([1, 5, 9, 63]), positions, cache, cos, sin, varlen=False)
    for hook in hooks:
        hook.remove()
    (call,) = rec.calls
    rows = torch.arange(batch)
    expected = k_before.clone()
    expected[rows, positions] = keys[0][rows, positions]
    assert torch.equal(expected, keys[0])
    save(f"qwen3_step_{tag}",
         dict(config=config, dtype=str(dtype), site="qwen3_asr.py:366-432", rope_theta=1e6),
         positions=positions.numpy(), qkv=f32(captured["qkv"]),
         q_norm_weight=f32(attention.q_norm.weight), k_norm_weight=f32(attention.k_norm.weight),
         eps=np.float64(config["rms_norm_eps"]), cos=f32(cos), sin=f32(sin),
         k_before=f32(k_before), v_before=f32(v_before),
         k_new=f32(keys[0][rows, positions]), v_new=f32(values[0][rows, positions]),
         sdpa_q=f32(call["q"]), sdpa_mask=call["mask"][:, 0, 0].numpy(),
         out=f32(captured["out"]))


def encoder_attention(whisper, dtype: torch.dtype, tag: str) -> None:
    """``MultiHeadAttention.forward`` (unmasked encoder self-attention)."""
    module = whisper.MultiHeadAttention(384, 6)
    seeded_parameters(module, 2)
    module = module.to(dtype)
    x = seeded_normal((1, 136, 384), 12).to(dtype)
    with torch.no_grad(), SdpaRecorder() as rec:
        module(x)
    (call,) = rec.calls
    save(f"encoder_attention_{tag}", dict(dtype=str(dtype), site="whisper.py:108-110"),
         q=f32(call["q"]), k=f32(call["k"]), v=f32(call["v"]), out=f32(call["out"]))


def qwen3_varlen(qwen3, dtype: torch.dtype, tag: str) -> None:
    """``attend(q, k, v, segments, causal)`` (qwen3_asr.py:152-181) on its
    padded-SDPA path (``Segments.from_lengths(..., varlen=False)``) for the two
    call sites: causal grouped-query prefill (TextAttention.prefill: heads of
    128, two query heads per key-value head as in 16/8, kept to 2/1 here for
    size) and non-causal audio windows (AudioAttention, heads of 64). Ragged
    segments, one longer than two 128-row tiles."""
    cases = {
        "prefill": dict(lengths=[37, 130, 1, 290], heads=2, kv_heads=1, head_dim=128, causal=True,
                        seed=500),
        "audio": dict(lengths=[104, 104, 57], heads=2, kv_heads=2, head_dim=64, causal=False,
                      seed=510),
    }
    arrays = {}
    for name, case in cases.items():
        tokens = sum(case["lengths"])
        q = seeded_normal((tokens, case["heads"], case["head_dim"]), case["seed"]).to(dtype)
        k = seeded_normal((tokens, case["kv_heads"], case["head_dim"]), case["seed"] + 1).to(dtype)
        v = seeded_normal((tokens, case["kv_heads"], case["head_dim"]), case["seed"] + 2).to(dtype)
        segments = qwen3.Segments.from_lengths(case["lengths"], torch.device("cpu"), False)
        with torch.no_grad():
            out = qwen3.attend(q, k, v, segments, case["causal"])
        arrays.update({f"{name}_q": f32(q), f"{name}_k": f32(k), f"{name}_v": f32(v),
                       f"{name}_starts": segments.starts.numpy(), f"{name}_out": f32(out)})
    save(f"qwen3_varlen_{tag}",
         dict(dtype=str(dtype), site="qwen3_asr.py:152-181", cases=cases), **arrays)


WHISPER_PREFIX = [50258, 50259, 50359, 50363]  # SOT, <|en|>, <|transcribe|>, <|notimestamps|>


def whisper_tiny_decode(whisper) -> None:
    """Greedy decoder steps of the Whisper-tiny architecture (fp32, seed 0) over
    N(0,1) encoder states. Each row first takes its own prefix one token per
    step (batch-of-one views of its cache row), so the batched steps that follow
    run at ragged positions."""
    config = dict(d_model=384, encoder_attention_heads=6, decoder_attention_heads=6,
                  encoder_layers=4, decoder_layers=4, encoder_ffn_dim=1536, decoder_ffn_dim=1536,
                  num_mel_bins=80, max_source_positions=1500, max_target_positions=448,
                  vocab_size=51865)
    model = whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, 0)
    model.eval()
    batch, steps = 8, 48
    offsets = [4, 9, 17, 30, 5, 60, 12, 100]
    prompts = []
    for b, off in enumerate(offsets):
        extra = seeded_normal((off - 4,), 300 + b).abs().mul(7000).long().clamp(max=50256).tolist()
        prompts.append(WHISPER_PREFIX + extra)
    cache = model.allocate_cache(batch)
    with torch.no_grad():
        model.set_encoder_output(cache, seeded_normal((batch, 1500, 384), 21))
        for b, prompt in enumerate(prompts):
            row = cache.rows(b, b + 1)
            for p, token in enumerate(prompt):
                model.decode(torch.tensor([[token]]), torch.tensor([p]), row)
        positions = torch.tensor(offsets)
        tokens = torch.tensor([[p[-1]] for p in prompts])
        positions -= 1  # the prompt's last token is re-fed at its own position
        hidden_all, argmax_all, tokens_all, positions_all = [], [], [], []
        for _ in range(steps):
            hidden = model.decode(tokens, positions, cache)[:, -1]
            logits = model.logits(hidden).float()
            choice = logits.argmax(dim=-1)
            hidden_all.append(f32(hidden))
            argmax_all.append(choice.numpy())
            tokens_all.append(tokens[:, 0].numpy())
            positions_all.append(positions.numpy().copy())
            tokens = choice[:, None]
            positions = positions + 1
    save("whisper_tiny_decode",
         dict(config=config, seed=0, encoder_seed=21, prompts=prompts, steps=steps,
              site="whisper.py:942-960 (decode + logits + argmax)"),
         tokens=np.stack(tokens_all, 1), positions=np.stack(positions_all, 1),
         argmax=np.stack(argmax_all, 1), hidden=np.stack(hidden_all, 1))


def qwen3_small_decode(qwen3) -> None:
    """Greedy ``TextModel.step`` calls of a 2-layer Qwen3 text model (fp32,
    seed 3), rows prefilled one position per step to ragged lengths."""
    config = dict(vocab_size=4096, hidden_size=512, num_hidden_layers=2, num_attention_heads=16,
                  num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-6, intermediate_size=1024)
    model = qwen3.TextModel(config)
    lm_head = torch.nn.Linear(512, 4096, bias=False)
    seeded_parameters(model, 3)
    seeded_parameters(lm_head, 4)
    batch, steps, length = 4, 32, 1024
    offsets = [20, 45, 7, 90]
    prompts = [seeded_normal((off,), 400 + b).abs().mul(1500).long().clamp(max=4095).tolist()
               for b, off in enumerate(offsets)]
    inverse = 1.0 / (1e6 ** (torch.arange(0, 128, 2).float() / 128))
    angles = torch.arange(length).float()[:, None] * inverse[None, :]
    angles = torch.cat((angles, angles), dim=-1)
    cos, sin = angles.cos(), angles.sin()
    shape = (2, batch, length, 8, 128)
    cache = qwen3.KVCache(torch.zeros(shape), torch.zeros(shape))
    with torch.no_grad():
        for b, prompt in enumerate(prompts):
            row = qwen3.KVCache(cache.keys[:, b:b + 1], cache.values[:, b:b + 1])
            for p, token in enumerate(prompt[:-1]):
                model.step(torch.tensor([token]), torch.tensor([p]), row, cos, sin, varlen=False)
        tokens = torch.tensor([p[-1] for p in prompts])
        positions = torch.tensor(offsets) - 1
        hidden_all, argmax_all, tokens_all, positions_all = [], [], [], []
        for _ in range(steps):
            hidden = model.step(tokens, positions, cache, cos, sin, varlen=False)
            choice = lm_head(hidden).argmax(dim=-1)
            hidden_all.append(f32(hidden))
            argmax_all.append(choice.numpy())
            tokens_all.append(tokens.numpy())
            positions_all.append(positions.numpy().copy())
            tokens = choice
            positions = positions + 1
    save("qwen3_small_decode",
         dict(config=config, seed=3, lm_head_seed=4, prompts=prompts, steps=steps,
              rope_theta=1e6, site="qwen3_asr.py:494-524 (TextModel.step) + lm_head argmax"),
         tokens=np.stack(tokens_all, 1), positions=np.stack(positions_all, 1),
         argmax=np.stack(argmax_all, 1), hidden=np.stack(hidden_all, 1))


def cross_kv(whisper, dtype: torch.dtype, tag: str) -> None:
    """``set_encoder_output`` (``whisper.py:313-319``) of a 2-layer decoder,
    384 wide (6 heads), for 2 windows of 40 encoder frames into a 3-row cache
    (the third row stays as allocated)."""
    config = dict(d_model=384, encoder_attention_heads=6, decoder_attention_heads=6,
                  encoder_layers=1, decoder_layers=2, encoder_ffn_dim=64, decoder_ffn_dim=64,
                  num_mel_bins=80, max_source_positions=40, max_target_positions=48,
                  vocab_size=128)
    model = whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, 9)
    model = model.to(dtype)
    cache = model.allocate_cache(3)
    states = seeded_normal((2, 40, 384), 13).to(dtype)
    with torch.no_grad():
        model.set_encoder_output(cache, states)
    save(f"cross_kv_{tag}", dict(config=config, dtype=str(dtype), seed=9, site="whisper.py:313-319"),
         states=f32(states), cross_keys=f32(cache.cross_keys), cross_values=f32(cache.cross_values))


def _run_steps(step, stub, state, hiddens, fields) -> dict:
    """Runs the reference's ``_step(stub, state, None, None)`` once per hidden
    state, recording ``_choose``'s token and log-probability and the state
    fields after each step."""
    queue = list(hiddens)
    choose = stub._choose
    chosen = []

    def recording_choose(*args):
        token, logprob = choose(*args)
        chosen.append((token.clone(), logprob.clone()))
        return token, logprob

    stub._choose = recording_choose
    stub.next_hidden = lambda *args, **kwargs: queue.pop(0)
    after = {name: [] for name in fields}
    with torch.no_grad():
        for _ in hiddens:
            step(stub, state, None, None)
            for name in fields:
                after[name].append(getattr(state, name).clone().reshape(len(state.position), -1)
                                   .squeeze(1).numpy())
    out = {f"after_{name}": np.stack(values) for name, values in after.items()}
    out["token"] = np.stack([t.numpy() for t, _ in chosen])
    out["logprob"] = np.stack([lp.float().numpy() for _, lp in chosen])
    out["generated"] = state.generated.numpy()
    return out


def step_epilogue(whisper, qwen3, dtype: torch.dtype, tag: str) -> None:
    """Greedy ``_step`` calls of the reference's Transcriber classes
    (``whisper.py:942-960``, ``qwen3_asr.py:1180-1201``) on a stub engine whose
    decoder returns given hidden states: the logits, ``_choose`` and the state
    update are the reference's own. Weights come from ``seeded_parameters``
    (the embedding / ``lm_head`` seeds are in ``meta``), so the tests rebuild
    them without the reference."""
    import types as _types

    fields = ("tokens", "position", "finished", "sum_logprobs")
    arrays = {}
    # Whisper-tiny widths (config 1): tied embedding (51865, 384).
    config = dict(d_model=384, encoder_attention_heads=6, decoder_attention_heads=6,
                  encoder_layers=1, decoder_layers=1, encoder_ffn_dim=64, decoder_ffn_dim=64,
                  num_mel_bins=80, max_source_positions=40, max_target_positions=448,
                  vocab_size=51865)
    model = whisper.WhisperForConditionalGeneration(config)
    seeded_parameters(model.model.decoder, 7)
    model = model.to(dtype)
    batch, eos = 8, 50257
    weight = model.model.decoder.embed_tokens.weight
    suppress = torch.zeros(51865, dtype=torch.bool)
    suppress[50364:] = True                      # every timestamp token
    suppress[[1, 2, 7, 8, 9, 10, 14, 25, 26, 27, 28, 29, 31, 58, 59, 60, 61, 62, 63, 90, 91,
              92, 93, 220, 359, 503, 522, 542, 873, 893, 902, 918, 922, 931, 1350, 1853, 1982,
              2460, 2627, 3246, 3253, 3268, 3536, 3846, 3961, 4183, 4667, 6585, 6647, 7273,
              9061, 9383, 10428, 10929, 11938, 12033, 12331, 12562, 13793, 14157, 14635, 15265,
              15618, 16553, 16604, 18362, 18956, 20075, 21675, 22520, 26130, 26161, 26435,
              28279, 29464, 31650, 32302, 32470, 36865, 42863, 47425, 49870, 50254, 50258,
              50358, 50359, 50360, 50361, 50362]] = True
    hiddens = [seeded_normal((batch, 1, 384), 600 + i).to(dtype) for i in range(3)]
    # Row 3 is steered onto EOS at the first step.
    hiddens[0][3, 0] = (weight[eos].float() * 40.0).to(dtype)
    state = whisper._DecodeState.allocate(batch, 448, torch.device("cpu"))
    state.tokens[:, 0] = torch.tensor([50258, 11, 400, 7000, 13, 50363, 0, 220])
    state.position[:] = torch.tensor([3, 10, 50, 100, 200, 446, 0, 30])
    state.end[:] = torch.tensor([447, 447, 447, 447, 447, 447, 0, 31])
    state.finished[:] = torch.tensor([False] * 6 + [True, False])
    state.sum_logprobs[:] = seeded_normal((batch,), 610).abs().neg()
    state.generated[:, :4] = torch.tensor([50258, 50259, 50360, 50364])
    for name in fields + ("end",):
        arrays[f"whisper_{name}0"] = getattr(state, name).clone().reshape(batch, -1)[:, 0].numpy()
    arrays["whisper_generated0"] = state.generated.numpy().copy()
    stub = _types.SimpleNamespace(_suppress=suppress, _eos=eos)
    stub.model = _types.SimpleNamespace(
        decode=lambda tokens, position, cache: stub.next_hidden(), logits=model.logits)
    stub._choose = _types.MethodType(whisper.Transcriber._choose, stub)
    out = _run_steps(whisper.Transcriber._step, stub, state, hiddens, fields)
    arrays.update({f"whisper_{key}": value for key, value in out.items()})
    arrays["whisper_hidden"] = np.stack([f32(h[:, 0]) for h in hiddens])
    arrays["whisper_suppress"] = suppress.numpy()

    # Qwen3: lm_head (8192, 1024), several EOS ids, CACHE_LENGTH-wide generated.
    vocab, width, batch, eos_ids = 8192, 1024, 6, [8000, 8001]
    lm_head = torch.nn.Linear(width, vocab, bias=False)
    seeded_parameters(lm_head, 8)
    lm_head = lm_head.to(dtype)
    hiddens = [seeded_normal((batch, width), 620 + i).to(dtype) for i in range(3)]
    hiddens[1][1] = (lm_head.weight[8001].float() * 12.0).to(dtype)
    state = qwen3._DecodeState.allocate(batch, torch.device("cpu"))
    state.tokens[:] = torch.tensor([151, 9, 4000, 77, 1, 0])
    state.position[:] = torch.tensor([19, 100, 409, 1022, 5, 0])
    state.end[:] = torch.tensor([1023, 1023, 1023, 1023, 7, 0])
    state.finished[:] = torch.tensor([False] * 5 + [True])
    state.sum_logprobs[:] = seeded_normal((batch,), 630).abs().neg()
    for name in fields + ("end",):
        arrays[f"qwen3_{name}0"] = getattr(state, name).clone().numpy()
    arrays["qwen3_generated0"] = state.generated.numpy().copy()
    stub = _types.SimpleNamespace(_lm_head=lm_head, _eos_ids=torch.tensor(eos_ids), _cos=None,
                                  _sin=None, _varlen=False)
    stub._text = _types.SimpleNamespace(step=lambda *args: stub.next_hidden())
    stub._choose = _types.MethodType(qwen3.Qwen3ASRTranscriber._choose, stub)
    out = _run_steps(qwen3.Qwen3ASRTranscriber._step, stub, state, hiddens, fields)
    arrays.update({f"qwen3_{key}": value for key, value in out.items()})
    arrays["qwen3_hidden"] = np.stack([f32(h) for h in hiddens])
    save(f"step_epilogue_{tag}",
         dict(dtype=str(dtype), steps=3,
              whisper=dict(vocab=51865, width=384, batch=8, eos=[eos], seed=7,
                           weight="decoder embed_tokens.weight, N(0, 0.02)",
                           site="whisper.py:942-975"),
              qwen3=dict(vocab=vocab, width=width, batch=batch, eos=eos_ids, seed=8,
                         weight="lm_head weight, N(0, 1/width)", site="qwen3_asr.py:1180-1213")),
         **arrays)


def whisper_config1(ref) -> None:
    """BASELINE config 1 on the reference's own classes, unpatched, CPU fp32:
    the model-level run (encoder over the mel batch, ``set_encoder_output``,
    the prompt pass, 64 greedy ``Transcriber._step`` calls) and the engine run
    (the eight windows queued to a ``Transcriber`` loaded from a checkpoint
    directory of the same weights; its worker admits, prefills, steps and
    finishes them)."""
    import tempfile

    from tests import reference_models as rm

    model, mel = rm.whisper_config1(ref)
    out = rm.run_whisper_steps(ref, model, mel, rm.CONFIG1_STEPS, graph=False)
    save("whisper_config1_model",
         dict(config=rm.WHISPER_TINY, seed=0, steps=rm.CONFIG1_STEPS, prefix=rm.WHISPER_PREFIX,
              site="whisper.py:140-153 (encoder), :313-319, :828-878 (prompt pass), "
                   ":942-975 (_step)", encoder_sample="encoded[:, ::50]", hidden_every=4),
         **out)
    with tempfile.TemporaryDirectory() as tmp:
        directory = rm.write_whisper_model_dir(Path(tmp) / "whisper-config1", model)
        transcriber = ref.whisper.Transcriber(directory, device="cpu", dtype="float32",
                                              max_batch_size=8, batch_wait_ms=500.0,
                                              cuda_graphs=False)
        results = rm.submit_whisper_jobs(ref, transcriber, mel.numpy(), rm.CONFIG1_STEPS)
    width = max(len(r["tokens"]) for r in results)
    tokens = np.full((len(results), width), -1, np.int64)
    for i, r in enumerate(results):
        tokens[i, :len(r["tokens"])] = r["tokens"]
    save("whisper_config1_engine",
         dict(config=rm.WHISPER_TINY, seed=0, max_new_tokens=rm.CONFIG1_STEPS,
              jobs=rm.config1_jobs(), languages=[r["language"] for r in results],
              site="whisper.py:728-940 (Transcriber._serve/_admit/_prefill/_advance/_finish)"),
         tokens=tokens, lengths=np.array([len(r["tokens"]) for r in results]),
         avg_logprob=np.array([r["avg_logprob"] for r in results]),
         no_speech_prob=np.array([r["no_speech_prob"] for r in results]))


def qwen3_graph_decode(ref) -> None:
    """The reference's ``TextModel`` (Qwen3-1.7B widths, 4 layers) in bf16 on
    the CPU: packed prefill of four ragged prompts, then 16 greedy steps."""
    from tests import reference_models as rm

    model, lm_head = rm.qwen3_text_model(ref, torch.bfloat16, "cpu")
    out = rm.run_qwen3_steps(ref, model, lm_head, None, graph=False)
    save("qwen3_graph_decode_bf16",
         dict(config=rm.QWEN3_1_7B_4L, seed=3, lm_head_seed=4, prompts=rm.QWEN3_PROMPTS,
              steps=rm.QWEN3_STEPS, bucket=rm.QWEN3_BUCKET, rope_theta=1e6,
              site="qwen3_asr.py:463-524 (TextModel.prefill / step) + lm_head argmax"),
         **out)


def whisper_turbo_decode(ref) -> None:
    """The reference's Whisper decoder at large-v3-turbo widths (4 layers) in
    bf16 on the CPU: ``set_encoder_output``, the prompt pass, ragged rows, then
    24 greedy fixed-shape steps over the 64-position bucket view."""
    from tests import reference_models as rm

    model = rm.whisper_turbo_decoder(ref, torch.bfloat16, "cpu")
    out = rm.run_turbo_steps(ref, model, None, graph=False)
    save("whisper_turbo_decode_bf16",
         dict(config=rm.WHISPER_TURBO_4L, seed=1, encoder_seed=41, steps=rm.TURBO_STEPS,
              site="whisper.py:255-342 (decoder step, logits argmax), :313-319"),
         **out)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--reference", default=None,
                        help="checkout of sjjeong94/asrback (read-only); default: "
                             "$ASRBACK_REFERENCE, then baseline/_ref")
    parser.add_argument("--only", default=None, help="generate only the fixtures whose "
                        "generator function has this name")
    args = parser.parse_args()
    if args.reference:
        os.environ["ASRBACK_REFERENCE"] = args.reference
    ref = reference_env.load()
    whisper, qwen3 = ref.whisper, ref.qwen3_asr

    torch.set_num_threads(8)
    per_dtype = (whisper_step, whisper_prefix, qwen3_step, encoder_attention, qwen3_varlen)
    for dtype, tag in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
        for make in per_dtype:
            if args.only in (None, make.__name__):
                make(qwen3 if make.__name__.startswith("qwen3") else whisper, dtype, tag)
        if args.only in (None, "step_epilogue"):
            step_epilogue(whisper, qwen3, dtype, tag)
        if args.only in (None, "cross_kv"):
            cross_kv(whisper, dtype, tag)
    if args.only in (None, "whisper_tiny_decode"):
        whisper_tiny_decode(whisper)
    if args.only in (None, "qwen3_small_decode"):
        qwen3_small_decode(qwen3)
    if args.only in (None, "whisper_config1"):
        whisper_config1(ref)
    if args.only in (None, "qwen3_graph_decode"):
        qwen3_graph_decode(ref)
    if args.only in (None, "whisper_turbo_decode"):
        whisper_turbo_decode(ref)


if __name__ == "__main__":
    main()
