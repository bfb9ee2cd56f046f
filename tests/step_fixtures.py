"""The step-epilogue fixtures' weights, rebuilt from their seeds.

``tests/golden/make_golden.py`` (``step_epilogue``) filled the reference's
modules with ``asrback_b200.synthetic.seeded_parameters``; the same draws are
repeated here so that neither the fixture nor the GPU tests need the weights
stored.
"""

from __future__ import annotations

import math

import torch

from asrback_b200.synthetic import parameter_seed, seeded_normal

STATE_FIELDS = ("tokens", "position", "end", "finished", "sum_logprobs")


def step_weight(family: str, meta: dict, bf16: bool) -> torch.Tensor:
    """``(vocab, width)`` weight of the fixture's logits: Whisper's tied
    ``decoder.embed_tokens.weight`` or Qwen3's ``lm_head.weight``."""
    info = meta[family]
    vocab, width = info["vocab"], info["width"]
    if family == "whisper":
        weight = seeded_normal((vocab, width), parameter_seed(info["seed"], "embed_tokens.weight"),
                               0.02)
    else:
        weight = seeded_normal((vocab, width), parameter_seed(info["seed"], "weight"),
                               1.0 / math.sqrt(width))
    return weight.to(torch.bfloat16) if bf16 else weight


def initial_state(g: dict, family: str) -> dict:
    state = {name: g[f"{family}_{name}0"] for name in STATE_FIELDS}
    state["generated"] = g[f"{family}_generated0"]
    return state


def cross_kv_weights(config: dict, seed: int, bf16: bool) -> list[tuple]:
    """Each decoder layer's cross-attention ``(k_proj.weight, v_proj.weight,
    v_proj.bias)`` as float32 arrays, as ``seeded_parameters(model.model.decoder,
    seed)`` fills the reference's decoder (rounded through bf16 when ``bf16``)."""
    from asrback_b200.synthetic import seeded_parameter

    width = config["d_model"]
    layers = []
    for index in range(config["decoder_layers"]):
        prefix = f"layers.{index}.encoder_attn."
        tensors = (seeded_parameter(prefix + "k_proj.weight", (width, width), seed),
                   seeded_parameter(prefix + "v_proj.weight", (width, width), seed),
                   seeded_parameter(prefix + "v_proj.bias", (width,), seed))
        if bf16:
            tensors = tuple(t.to(torch.bfloat16).float() for t in tensors)
        layers.append(tuple(t.numpy() for t in tensors))
    return layers
