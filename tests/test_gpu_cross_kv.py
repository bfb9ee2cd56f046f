"""Cross-attention key/value projection on the GPU: asrback_whisper_cross_kv_projection
(through the C ABI) against the reference's recorded ``set_encoder_output``,
and at full size against the reference's own torch expression
(``_split_heads(k_proj(x))`` / ``v_proj``) on the same tensors.

Tolerances: max-abs 1e-4 for float32 outputs; bf16 outputs within one bf16
rounding step of the reference's (relative 2^-7 plus 1e-2 absolute).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from asrback_b200 import attention
from tests.golden import load
from tests.step_fixtures import cross_kv_weights

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True)
def clean_status():
    attention.read_status()
    yield


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_set_encoder_output_matches_reference(tag):
    """The op, one call per decoder layer into the ``(layers, rows, heads,
    frames, 64)`` cross cache, as ``set_encoder_output`` runs it, against the
    reference's recorded cache (two windows into a three-row cache: the third
    row stays zero)."""
    g = load(f"cross_kv_{tag}")
    dtype = torch.float32 if tag == "fp32" else torch.bfloat16
    config = g["meta"]["config"]
    heads, width = config["decoder_attention_heads"], config["d_model"]
    shape = (config["decoder_layers"], 3, heads, config["max_source_positions"], width // heads)
    cross_keys = torch.zeros(shape, dtype=dtype, device=DEV)
    cross_values = torch.zeros(shape, dtype=dtype, device=DEV)
    states = torch.from_numpy(g["states"]).to(DEV, dtype)
    batch = states.shape[0]
    for index, (k_weight, v_weight, v_bias) in enumerate(
            cross_kv_weights(config, g["meta"]["seed"], bf16=tag == "bf16")):
        attention.whisper_cross_kv_projection(
            states, *(torch.from_numpy(t).to(DEV, dtype) for t in (k_weight, v_weight, v_bias)),
            cross_keys[index, :batch], cross_values[index, :batch])
    tol = 1e-4 if tag == "fp32" else 2e-2
    np.testing.assert_allclose(cross_keys.float().cpu().numpy(), g["cross_keys"], atol=tol,
                               rtol=0)
    np.testing.assert_allclose(cross_values.float().cpu().numpy(), g["cross_values"],
                               atol=tol, rtol=0)
    assert attention.read_status() == 0


def _reference(x, wk, wv, bv, heads):
    def split(t):
        b, s, w = t.shape
        return t.view(b, s, heads, w // heads).transpose(1, 2)
    return split(F.linear(x, wk)), split(F.linear(x, wv, bv))


@pytest.mark.parametrize("dtype,width,tokens,length,batch", [
    (torch.bfloat16, 1280, 1500, 1500, 4),   # large-v3-turbo windows
    (torch.bfloat16, 1280, 1000, 1500, 3),   # fewer frames than the cache holds
    (torch.bfloat16, 384, 300, 320, 2),      # 128-feature tiles
    (torch.float32, 384, 300, 320, 2),
])
def test_matches_torch(dtype, width, tokens, length, batch):
    gen = torch.Generator(device=DEV).manual_seed(width + tokens)
    heads = width // 64
    x = torch.randn((batch, tokens, width), generator=gen, device=DEV).to(dtype)
    wk = (torch.randn((width, width), generator=gen, device=DEV) / width ** 0.5).to(dtype)
    wv = (torch.randn((width, width), generator=gen, device=DEV) / width ** 0.5).to(dtype)
    bv = (torch.randn((width,), generator=gen, device=DEV) * 0.1).to(dtype)
    # A 2-layer cache with room for one more window; layer 1, rows 0..batch-1.
    keys = torch.full((2, batch + 1, heads, length, 64), 7.0, device=DEV, dtype=dtype)
    values = torch.full_like(keys, 7.0)
    attention.whisper_cross_kv_projection(x, wk, wv, bv, keys[1, :batch], values[1, :batch])
    want_k, want_v = _reference(x, wk, wv, bv, heads)
    for got, want in ((keys, want_k), (values, want_v)):
        part = got[1, :batch, :, :tokens].float()
        if dtype == torch.float32:
            torch.testing.assert_close(part, want.float(), atol=1e-4, rtol=0)
        else:
            err = (part - want.float()).abs()
            assert torch.all(err <= want.float().abs() * 2.0 ** -7 + 1e-2), err.max()
        # Everything outside the written rows keeps its value.
        assert torch.all(got[0] == 7.0) and torch.all(got[1, batch:] == 7.0)
        assert torch.all(got[1, :batch, :, tokens:] == 7.0)
    assert attention.read_status() == 0
