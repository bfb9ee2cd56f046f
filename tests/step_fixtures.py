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
