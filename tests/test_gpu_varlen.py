"""Varlen attention parity on the GPU: asrback_varlen_attention (through the C
ABI) against the reference's recorded `attend` outputs and the CPU oracle.

Tolerances: max-abs 1e-4 for float32 outputs, 2e-2 for bfloat16.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from asrback_b200 import _native, attention
from oracle import attention as oracle
from tests.golden import load

pytestmark = pytest.mark.gpu

DEV = "cuda"
TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2}
DTYPES = {"fp32": torch.float32, "bf16": torch.bfloat16}


@pytest.fixture(autouse=True)
def clean_status():
    attention.read_status()
    yield


def dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("case", ["prefill", "audio"])
@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_varlen_matches_reference(tag, case):
    dtype = DTYPES[tag]
    g = load(f"qwen3_varlen_{tag}")
    meta = g["meta"]["cases"][case]
    starts = torch.from_numpy(g[f"{case}_starts"]).to(DEV, torch.int32)
    out = attention.varlen_attention(dev(g[f"{case}_q"], dtype), dev(g[f"{case}_k"], dtype),
                                     dev(g[f"{case}_v"], dtype), starts, max(meta["lengths"]),
                                     meta["causal"])
    np.testing.assert_allclose(host(out), g[f"{case}_out"], atol=TOL[dtype], rtol=0)
    assert attention.read_status() == 0


def _rand(gen, shape, dtype):
    return torch.randn(shape, generator=gen).to(dtype)


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
@pytest.mark.parametrize("lengths,heads,kv_heads,head_dim,causal", [
    ([410, 397, 423, 1, 128, 129, 255, 256, 257], 16, 8, 128, True),   # Qwen3 prompt prefill
    ([104, 104, 104, 57, 1], 16, 16, 64, False),                       # audio windows
    ([600, 33], 4, 1, 128, False),
    ([300, 5, 700], 8, 2, 64, True),
    # segments of at most one 128-row tile: two items per CTA in flight
    ([128, 1, 77, 128, 100, 0, 3], 16, 8, 128, True),
    ([104] * 60 + [57, 0, 1, 128, 90], 16, 16, 64, False),   # ~8 items per CTA
    ([100, 0, 0, 128, 5] * 12, 8, 2, 128, True),
])
def test_varlen_random(tag, lengths, heads, kv_heads, head_dim, causal):
    dtype = DTYPES[tag]
    gen = torch.Generator().manual_seed(sum(lengths) + heads + head_dim)
    tokens = sum(lengths)
    q = _rand(gen, (tokens, heads, head_dim), dtype)
    k = _rand(gen, (tokens, kv_heads, head_dim), dtype)
    v = _rand(gen, (tokens, kv_heads, head_dim), dtype)
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    out = attention.varlen_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                     torch.from_numpy(starts).to(DEV), max(lengths), causal)
    want = oracle.varlen_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                   starts, causal)
    np.testing.assert_allclose(host(out), want, atol=TOL[dtype], rtol=0)
    assert attention.read_status() == 0


@pytest.mark.parametrize("causal", [True, False])
def test_varlen_rescales_when_a_later_key_dominates(causal):
    """Keys in later tiles that score far above a row's running max (8 x the
    row's own query) move the max of some rows of a warp only: O is rescaled
    for those rows (the lazy rescale's j > 0 path), causal and not."""
    gen = torch.Generator().manual_seed(12)
    lengths, heads, kv_heads, head_dim = [410, 300], 16, 8, 128
    tokens = sum(lengths)
    q = _rand(gen, (tokens, heads, head_dim), torch.bfloat16)
    k = _rand(gen, (tokens, kv_heads, head_dim), torch.bfloat16)
    v = _rand(gen, (tokens, kv_heads, head_dim), torch.bfloat16)
    # (query row, key row) within the first segment, key before the row.
    for row, key in ((400, 300), (290, 200), (170, 130), (409, 390)):
        k[key, 0] = (q[row, 0].float() * 8).bfloat16()
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    out = attention.varlen_attention(q.to(DEV), k.to(DEV), v.to(DEV),
                                     torch.from_numpy(starts).to(DEV), max(lengths), causal)
    want = oracle.varlen_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                   starts, causal)
    np.testing.assert_allclose(host(out), want, atol=2e-2, rtol=0)
    assert attention.read_status() == 0


@pytest.mark.parametrize("contiguous_k", [False, True])
def test_varlen_strided_views_of_a_fused_projection(contiguous_k):
    """q, k, v as views into one (tokens, (16 + 8 + 8) * 128) projection, the
    layout TextAttention._project splits (qwen3_asr.py:366-372); with
    `contiguous_k`, q and k are new tensors (as after RMSNorm and RoPE) while v
    stays a view, so k and v have different strides."""
    gen = torch.Generator().manual_seed(3)
    lengths = [200, 61, 390]
    tokens = sum(lengths)
    qkv = _rand(gen, (tokens, 32 * 128), torch.bfloat16).to(DEV)
    q = qkv[:, : 16 * 128].view(tokens, 16, 128)
    k = qkv[:, 16 * 128 : 24 * 128].view(tokens, 8, 128)
    v = qkv[:, 24 * 128 :].view(tokens, 8, 128)
    if contiguous_k:
        q, k = q.contiguous(), k.contiguous()
        assert k.stride() != v.stride()
    starts = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    out = attention.varlen_attention(q, k, v, torch.from_numpy(starts).to(DEV), max(lengths), True)
    want = oracle.varlen_attention(host(q), host(k), host(v), starts, True)
    np.testing.assert_allclose(host(out), want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("longest", [150, 100])
def test_bad_segments_are_skipped_and_reported(longest):
    """A segment past the tensor, or longer than max_length, is not computed
    (its rows keep what the output held) and sets STATUS_SEGMENT; the other
    segments are still right. `longest` 100 takes the one-tile-per-segment
    schedule."""
    gen = torch.Generator().manual_seed(4)
    tokens = 300
    q = _rand(gen, (tokens, 4, 128), torch.bfloat16).to(DEV)
    k = _rand(gen, (tokens, 2, 128), torch.bfloat16).to(DEV)
    v = _rand(gen, (tokens, 2, 128), torch.bfloat16).to(DEV)
    for starts in ([0, 100, 400], [0, 100, 300]):
        cu = torch.tensor(starts, dtype=torch.int32, device=DEV)
        # the second segment (200 tokens) is longer than `longest`
        out = attention.varlen_attention(q, k, v, cu, longest, True)
        want = oracle.varlen_attention(host(q)[:100], host(k)[:100], host(v)[:100], [0, 100], True)
        np.testing.assert_allclose(host(out)[:100], want, atol=2e-2, rtol=0)
        torch.cuda.synchronize()
        assert attention.read_status() & _native.STATUS_SEGMENT


def test_graph_capture_replays_with_new_segments():
    from asrback_b200.transcription import CapturedGraph

    gen = torch.Generator().manual_seed(5)
    tokens = 512
    q = _rand(gen, (tokens, 16, 128), torch.bfloat16).to(DEV)
    k = _rand(gen, (tokens, 8, 128), torch.bfloat16).to(DEV)
    v = _rand(gen, (tokens, 8, 128), torch.bfloat16).to(DEV)
    cu = torch.tensor([0, 256, 512], dtype=torch.int32, device=DEV)
    result = {}

    def step():
        result["out"] = attention.varlen_attention(q, k, v, cu, 400, True)

    graph = CapturedGraph(step)
    cu.copy_(torch.tensor([0, 100, 500], dtype=torch.int32))
    graph.replay()
    torch.cuda.synchronize()
    got = host(result["out"])[:500]
    want = oracle.varlen_attention(host(q)[:500], host(k)[:500], host(v)[:500], [0, 100, 500], True)
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
