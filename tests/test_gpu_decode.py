"""Decode attention parity on the GPU: the sm_100a kernels (through the C ABI)
against the reference's recorded outputs and the CPU oracle.

Tolerances (from the build's target): max-abs 1e-4 for float32 outputs and
2e-2 for bfloat16 outputs; cache writes exact (float32, Whisper) or within one
bf16 rounding (Qwen3 bf16, whose keys pass RMSNorm and RoPE first).
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


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def host(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture(autouse=True)
def clean_status():
    attention.read_status()
    yield


# ---------------------------------------------------------------- golden ----

@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_whisper_self_step_matches_reference(tag):
    dtype = DTYPES[tag]
    g = load(f"whisper_step_{tag}")
    batch, heads, length, dim = g["self_k_before"].shape
    kc, vc = dev(g["self_k_before"], dtype), dev(g["self_v_before"], dtype)
    positions = dev(g["positions"], torch.int64)
    out = attention.whisper_self_attention_step(
        dev(g["self_q"], dtype), dev(g["self_k_new"], dtype), dev(g["self_v_new"], dtype),
        kc, vc, positions)
    np.testing.assert_allclose(host(out).reshape(batch, heads, dim), g["self_out"],
                               atol=TOL[dtype], rtol=0)
    rows = np.arange(batch)
    expected_k = g["self_k_before"].copy()
    expected_k[rows, :, g["positions"]] = g["self_k_new"]
    np.testing.assert_array_equal(host(kc), expected_k)
    expected_v = g["self_v_before"].copy()
    expected_v[rows, :, g["positions"]] = g["self_v_new"]
    np.testing.assert_array_equal(host(vc), expected_v)
    assert attention.read_status() == 0


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_whisper_cross_step_matches_reference(tag):
    dtype = DTYPES[tag]
    g = load(f"whisper_step_{tag}")
    batch, heads, _, dim = g["cross_k"].shape
    out = attention.whisper_cross_attention_step(dev(g["cross_q"], dtype), dev(g["cross_k"], dtype),
                                                 dev(g["cross_v"], dtype))
    np.testing.assert_allclose(host(out).reshape(batch, heads, dim), g["cross_out"],
                               atol=TOL[dtype], rtol=0)


def _heads_of(out, tokens, heads, dim):
    """``(B, P, H*D)`` op output as the reference's ``(B, H, P, D)``."""
    batch = out.shape[0]
    return host(out).reshape(batch, tokens, heads, dim).transpose(0, 2, 1, 3)


@pytest.mark.parametrize("name", ["detect", "prompt"])
@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_whisper_prefix_matches_reference(tag, name):
    """Prompt pass (P = 7) and language detection (P = 1): the caller writes
    the keys at 0..P-1; the kernel reads keys 0..t for token t of the cache
    cut to P positions, writes nothing; cross-attention of every token."""
    dtype = DTYPES[tag]
    g = load(f"whisper_prefix_{tag}")
    q, k, v = g[f"{name}_self_q"], g[f"{name}_self_k"], g[f"{name}_self_v"]
    batch, heads, tokens, dim = q.shape
    gen = torch.Generator().manual_seed(tokens)
    kc = _rand(gen, (batch, heads, 48, dim), dtype).to(DEV)
    vc = _rand(gen, (batch, heads, 48, dim), dtype).to(DEV)
    kc[:, :, :tokens] = dev(k, dtype)
    vc[:, :, :tokens] = dev(v, dtype)
    k_before, v_before = kc.clone(), vc.clone()
    out = attention.whisper_self_attention_prefix(dev(q, dtype), kc[:, :, :tokens], vc[:, :, :tokens])
    np.testing.assert_allclose(_heads_of(out, tokens, heads, dim), g[f"{name}_self_out"],
                               atol=TOL[dtype], rtol=0)
    assert torch.equal(kc, k_before) and torch.equal(vc, v_before)
    cross = attention.whisper_cross_attention_prefix(dev(g[f"{name}_cross_q"], dtype),
                                                     dev(g["cross_k"], dtype), dev(g["cross_v"], dtype))
    np.testing.assert_allclose(_heads_of(cross, tokens, heads, dim), g[f"{name}_cross_out"],
                               atol=TOL[dtype], rtol=0)
    assert attention.read_status() == 0


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_qwen3_step_matches_reference(tag):
    dtype = DTYPES[tag]
    g = load(f"qwen3_step_{tag}")
    keys, values = dev(g["k_before"], dtype), dev(g["v_before"], dtype)
    positions = dev(g["positions"], torch.int64)
    out = attention.qwen3_attention_step(
        dev(g["qkv"], dtype), dev(g["q_norm_weight"], dtype), dev(g["k_norm_weight"], dtype),
        float(g["eps"]), dev(g["cos"], dtype), dev(g["sin"], dtype), positions, keys, values, 16, 8)
    np.testing.assert_allclose(host(out), g["out"], atol=TOL[dtype], rtol=0)
    rows = np.arange(len(g["positions"]))
    written_k = host(keys)[rows, g["positions"]]
    np.testing.assert_allclose(written_k, g["k_new"], atol=TOL[dtype], rtol=0)
    if dtype == torch.bfloat16:
        assert np.mean(written_k == g["k_new"]) > 0.99
    np.testing.assert_array_equal(host(values)[rows, g["positions"]], g["v_new"])
    untouched = np.ones(g["k_before"].shape[:2], bool)
    untouched[rows, g["positions"]] = False
    np.testing.assert_array_equal(host(keys)[untouched], g["k_before"][untouched])


@pytest.mark.parametrize("tag", ["fp32", "bf16"])
def test_encoder_attention_matches_reference(tag):
    dtype = DTYPES[tag]
    g = load(f"encoder_attention_{tag}")
    b, h, s, d = g["q"].shape
    # The reference's layout: (B, S, H*D) projections viewed as (B, H, S, D).
    def proj(a):
        return dev(a.transpose(0, 2, 1, 3).reshape(b, s, h * d), dtype).view(b, s, h, d).transpose(1, 2)
    out = attention.whisper_encoder_attention(proj(g["q"]), proj(g["k"]), proj(g["v"]))
    got = host(out).reshape(b, s, h, d).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(got, g["out"], atol=TOL[dtype], rtol=0)


# ------------------------------------------------- seeded, against oracle ----

def _rand(gen, shape, dtype, scale=1.0):
    return (torch.randn(shape, generator=gen) * scale).to(dtype)


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
@pytest.mark.parametrize("batch,bucket", [(1, 448), (3, 64), (64, 448), (16, 256)])
def test_whisper_self_step_random(tag, batch, bucket):
    """Ragged positions (0 and bucket-1 included) in a bucket view of a larger
    cache: rows beyond the batch and positions beyond the bucket untouched."""
    dtype = DTYPES[tag]
    gen = torch.Generator().manual_seed(batch * 1000 + bucket)
    heads, dim, storage_rows = 20, 64, batch + 2
    k_store = _rand(gen, (storage_rows, heads, 448, dim), dtype)
    v_store = _rand(gen, (storage_rows, heads, 448, dim), dtype)
    q, k, v = (_rand(gen, (batch, heads, dim), dtype) for _ in range(3))
    positions = torch.randint(0, bucket, (batch,), generator=gen)
    positions[0] = bucket - 1
    if batch > 1:
        positions[1] = 0
    kc_dev, vc_dev = k_store.to(DEV), v_store.to(DEV)
    out = attention.whisper_self_attention_step(
        q.to(DEV), k.to(DEV), v.to(DEV), kc_dev[:batch, :, :bucket], vc_dev[:batch, :, :bucket],
        positions.to(DEV))
    want, k_after, v_after = oracle.whisper_self_attention_step(
        q.float().numpy(), k.float().numpy(), v.float().numpy(),
        k_store[:batch, :, :bucket].float().numpy(), v_store[:batch, :, :bucket].float().numpy(),
        positions.numpy())
    np.testing.assert_allclose(host(out).reshape(batch, heads, dim), want, atol=TOL[dtype], rtol=0)
    got_k = host(kc_dev)
    np.testing.assert_array_equal(got_k[:batch, :, :bucket], k_after)
    np.testing.assert_array_equal(got_k[batch:], k_store[batch:].float().numpy())
    np.testing.assert_array_equal(got_k[:, :, bucket:], k_store[:, :, bucket:].float().numpy())
    np.testing.assert_array_equal(host(vc_dev)[:batch, :, :bucket], v_after)
    assert attention.read_status() == 0


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
@pytest.mark.parametrize("batch,tokens,bucket", [(1, 1, 448), (5, 3, 448), (2, 5, 448), (1, 4, 448),
                                                 (64, 5, 64), (32, 4, 448), (2, 160, 448),
                                                 (3, 448, 448)])
def test_whisper_prefix_random(tag, batch, tokens, bucket):
    """Prompt passes of 1..448 tokens in a bucket view of a larger cache: the
    `_split_heads` query view (rows evenly spaced, heads interleaved), a cache
    view longer than the pass (keys past token t never read), nothing
    written; cross-attention over 1500 frames for the same rows (in bf16 from 4
    tokens up, 4 tokens per CTA: a last group with absent tokens, split and
    unsplit launches)."""
    dtype = DTYPES[tag]
    gen = torch.Generator().manual_seed(batch * 1000 + tokens)
    heads, dim = 20, 64
    kc = _rand(gen, (batch + 1, heads, 448, dim), dtype).to(DEV)
    vc = _rand(gen, (batch + 1, heads, 448, dim), dtype).to(DEV)
    x = _rand(gen, (batch, tokens, heads * dim), dtype).to(DEV)
    query = x.view(batch, tokens, heads, dim).transpose(1, 2)
    k_before = kc.clone()
    out = attention.whisper_self_attention_prefix(query, kc[:batch, :, :bucket], vc[:batch, :, :bucket])
    mask = np.arange(tokens)[None, :] <= np.arange(tokens)[:, None]
    want = oracle.sdpa(host(query), host(kc[:batch, :, :tokens]), host(vc[:batch, :, :tokens]), mask)
    np.testing.assert_allclose(_heads_of(out, tokens, heads, dim), want, atol=TOL[dtype], rtol=0)
    assert torch.equal(kc, k_before)
    if tokens <= 160:
        ck = _rand(gen, (batch, heads, 1500, dim), dtype).to(DEV)
        cv = _rand(gen, (batch, heads, 1500, dim), dtype).to(DEV)
        cross = attention.whisper_cross_attention_prefix(query, ck, cv)
        want = oracle.whisper_cross_attention_prefix(host(query), host(ck), host(cv))
        np.testing.assert_allclose(_heads_of(cross, tokens, heads, dim), want, atol=TOL[dtype], rtol=0)
    assert attention.read_status() == 0


@pytest.mark.parametrize("windows,tokens,length,plant",
                         [(1, 1, 1500, False), (3, 4, 1500, False), (2, 31, 1500, False),
                          (5, 32, 1500, False), (2, 33, 1500, False), (8, 100, 1500, False),
                          (2, 128, 1500, False), (4, 7, 200, False), (1, 4, 128, False),
                          (3, 2, 1500, False), (2, 12, 700, False), (6, 16, 1500, False),
                          (3, 3, 1500, False), (2, 5, 333, False), (4, 8, 1500, False),
                          (3, 9, 1500, False), (5, 64, 1500, False), (2, 6, 700, False),
                          (3, 4, 1500, True),
                          (2, 8, 1500, True), (3, 40, 1500, True)])
def test_whisper_cross_prefix_tensor_core(windows, tokens, length, plant, monkeypatch):
    """The tensor-core prompt-pass cross-attention (bf16, up to 128 tokens per
    window: one, two, three or four softmax warps; up to 8 tokens with a row
    shared by four lanes) against the oracle and the CUDA-core prefix kernel,
    over the whole cache, over a view of the first `length` frames of a longer
    one (keys past it never read), and with a last key tile that ends inside or
    at the tile. Up to 8 tokens over an even number of key tiles, an item's two
    halves run in the two slots and merge in the CTA. `plant` scales a few keys of later tiles up so that the running
    maximum moves by more than the rescale threshold after the first tile."""
    gen = torch.Generator().manual_seed(windows * 1000 + tokens + length)
    heads, dim, frames = 20, 64, 1500
    ck = _rand(gen, (windows, heads, frames, dim), torch.bfloat16)
    if plant:
        ck[:, :, 700:704] *= 12
        ck[:, :, 1300:1302] *= 24
    ck = ck.to(DEV)
    cv = _rand(gen, (windows, heads, frames, dim), torch.bfloat16).to(DEV)
    x = _rand(gen, (windows, tokens, heads * dim), torch.bfloat16).to(DEV)
    query = x.view(windows, tokens, heads, dim).transpose(1, 2)
    monkeypatch.setenv("ASRBACK_PREFIX_TC", "1")
    got = attention.whisper_cross_attention_prefix(query, ck[:, :, :length], cv[:, :, :length])
    monkeypatch.setenv("ASRBACK_PREFIX_TC", "0")
    old = attention.whisper_cross_attention_prefix(query, ck[:, :, :length], cv[:, :, :length])
    want = oracle.whisper_cross_attention_prefix(host(query), host(ck[:, :, :length]),
                                                 host(cv[:, :, :length]))
    np.testing.assert_allclose(_heads_of(got, tokens, heads, dim), want, atol=2e-2, rtol=0)
    np.testing.assert_allclose(host(got), host(old), atol=2e-2, rtol=0)
    assert attention.read_status() == 0


def test_whisper_prefix_rejects_bad_shapes():
    q = torch.zeros(2, 20, 4, 64, device=DEV, dtype=torch.bfloat16)
    kc = torch.zeros(2, 20, 448, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(_native.NativeError, match="exceed the cache length"):
        attention.whisper_self_attention_prefix(q, kc[:, :, :3], kc[:, :, :3])
    with pytest.raises(ValueError, match="head_dim"):
        attention.whisper_self_attention_prefix(q[:, :, :, 0], kc, kc)


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
@pytest.mark.parametrize("batch,length", [(1, 1500), (2, 1500), (64, 1500), (5, 77)])
def test_whisper_cross_step_random(tag, batch, length):
    dtype = DTYPES[tag]
    gen = torch.Generator().manual_seed(7 * batch + length)
    heads, dim = 20, 64
    q = _rand(gen, (batch, heads, dim), dtype)
    kc = _rand(gen, (batch + 1, heads, length, dim), dtype)
    vc = _rand(gen, (batch + 1, heads, length, dim), dtype)
    out = attention.whisper_cross_attention_step(q.to(DEV), kc.to(DEV)[:batch], vc.to(DEV)[:batch])
    want = oracle.whisper_cross_attention(q.float().numpy(), kc[:batch].float().numpy(),
                                          vc[:batch].float().numpy())
    np.testing.assert_allclose(host(out).reshape(batch, heads, dim), want, atol=TOL[dtype], rtol=0)


def _qwen3_inputs(gen, batch, bucket, heads, dtype, storage=1024):
    dim, kv_heads = 128, 8
    qkv = _rand(gen, (batch, (heads + 2 * kv_heads) * dim), dtype, 2.0)
    qn = (1.0 + 0.1 * torch.randn(dim, generator=gen)).to(dtype)
    kn = (1.0 + 0.1 * torch.randn(dim, generator=gen)).to(dtype)
    cos, sin = (torch.from_numpy(t) for t in oracle.rope_tables(1e6, dim, storage, bf16=False))
    cos, sin = cos.to(dtype), sin.to(dtype)
    k_store = _rand(gen, (batch + 1, storage, kv_heads, dim), dtype)
    v_store = _rand(gen, (batch + 1, storage, kv_heads, dim), dtype)
    positions = torch.randint(0, bucket, (batch,), generator=gen)
    positions[0] = bucket - 1
    if batch > 1:
        positions[1] = 0
    return qkv, qn, kn, cos, sin, k_store, v_store, positions


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
@pytest.mark.parametrize("batch,bucket,heads", [(1, 1024, 16), (5, 512, 16), (64, 1024, 16),
                                                (64, 128, 16), (9, 768, 8)])
def test_qwen3_step_random(tag, batch, bucket, heads):
    dtype = DTYPES[tag]
    gen = torch.Generator().manual_seed(batch * 31 + bucket + heads)
    qkv, qn, kn, cos, sin, k_store, v_store, positions = _qwen3_inputs(gen, batch, bucket, heads, dtype)
    kd, vd = k_store.to(DEV), v_store.to(DEV)
    out = attention.qwen3_attention_step(qkv.to(DEV), qn.to(DEV), kn.to(DEV), 1e-6, cos.to(DEV),
                                         sin.to(DEV), positions.to(DEV), kd[:batch, :bucket],
                                         vd[:batch, :bucket], heads, 8)
    want, k_after, v_after = oracle.qwen3_decode_attention(
        qkv.float().numpy(), qn.float().numpy(), kn.float().numpy(), 1e-6, cos.float().numpy(),
        sin.float().numpy(), positions.numpy(), k_store[:batch, :bucket].float().numpy(),
        v_store[:batch, :bucket].float().numpy(), heads, 8, bf16=dtype == torch.bfloat16)
    np.testing.assert_allclose(host(out), want, atol=TOL[dtype], rtol=0)
    got_k = host(kd)
    np.testing.assert_allclose(got_k[:batch, :bucket], k_after, atol=TOL[dtype], rtol=0)
    np.testing.assert_array_equal(got_k[batch:], k_store[batch:].float().numpy())
    np.testing.assert_array_equal(got_k[:, bucket:], k_store[:, bucket:].float().numpy())
    np.testing.assert_array_equal(host(vd)[:batch, :bucket], v_after)
    assert attention.read_status() == 0


@pytest.mark.parametrize("batch", [64, 32])
@pytest.mark.parametrize("tag", ["bf16", "fp32"])
def test_qwen3_split_clusters_match_the_workspace_merge(tag, batch, monkeypatch):
    """At 64 (32) rows every row is cut in 2 (4) splits, which run as one
    thread-block cluster handing the other splits' states to split 0 in its
    shared memory; with ASRBACK_SPLIT_PAIR=0 the same splits merge through the
    workspace. Both give the same outputs (to merge rounding) and the same
    cache writes, for rows that use one split or several."""
    dtype = DTYPES[tag]
    gen = torch.Generator().manual_seed(batch)
    bucket, heads = 1024, 16
    qkv, qn, kn, cos, sin, k_store, v_store, positions = _qwen3_inputs(gen, batch, bucket, heads, dtype)
    results = []
    for pair in ("1", "0"):
        monkeypatch.setenv("ASRBACK_SPLIT_PAIR", pair)
        kd, vd = k_store.to(DEV), v_store.to(DEV)
        out = attention.qwen3_attention_step(qkv.to(DEV), qn.to(DEV), kn.to(DEV), 1e-6, cos.to(DEV),
                                             sin.to(DEV), positions.to(DEV), kd[:batch, :bucket],
                                             vd[:batch, :bucket], heads, 8)
        results.append((host(out), host(kd), host(vd)))
    (o1, k1, v1), (o0, k0, v0) = results
    np.testing.assert_allclose(o1, o0, atol=TOL[dtype], rtol=0)
    np.testing.assert_array_equal(k1, k0)
    np.testing.assert_array_equal(v1, v0)
    assert attention.read_status() == 0


@pytest.mark.parametrize("batch,length", [(1, 1500), (2, 300)])
def test_encoder_attention_random(batch, length):
    gen = torch.Generator().manual_seed(length)
    heads, dim = 20, 64
    x = [_rand(gen, (batch, length, heads * dim), torch.bfloat16) for _ in range(3)]
    views = [t.to(DEV).view(batch, length, heads, dim).transpose(1, 2) for t in x]
    out = attention.whisper_encoder_attention(*views)
    q, k, v = (t.float().numpy().reshape(batch, length, heads, dim).transpose(0, 2, 1, 3) for t in x)
    want = oracle.encoder_attention(q, k, v)
    got = host(out).reshape(batch, length, heads, dim).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)


@pytest.mark.parametrize("length", [1, 95, 96, 97, 136, 257, 385])
def test_encoder_attention_ragged_tiles(length):
    """Lengths that end inside or exactly at a 96-key tile and leave a work
    item's three 128-row query tiles partly or wholly past the window."""
    gen = torch.Generator().manual_seed(1000 + length)
    batch, heads, dim = 2, 20, 64
    x = [_rand(gen, (batch, length, heads * dim), torch.bfloat16) for _ in range(3)]
    views = [t.to(DEV).view(batch, length, heads, dim).transpose(1, 2) for t in x]
    out = attention.whisper_encoder_attention(*views)
    q, k, v = (t.float().numpy().reshape(batch, length, heads, dim).transpose(0, 2, 1, 3) for t in x)
    want = oracle.encoder_attention(q, k, v)
    got = host(out).reshape(batch, length, heads, dim).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    assert attention.read_status() == 0


def test_encoder_attention_many_items_per_cta():
    """More work items than SMs (10 windows x 8 heads x 4 query-tile groups),
    so every persistent CTA runs several items through its Q buffers and K/V
    ring; against torch's float32 SDPA of the same bf16 inputs."""
    import torch.nn.functional as F

    gen = torch.Generator().manual_seed(77)
    batch, length, heads, dim = 10, 1500, 8, 64
    x = [_rand(gen, (batch, length, heads * dim), torch.bfloat16).to(DEV) for _ in range(3)]
    views = [t.view(batch, length, heads, dim).transpose(1, 2) for t in x]
    out = attention.whisper_encoder_attention(*views)
    want = F.scaled_dot_product_attention(*(t.float() for t in views))
    got = out.float().view(batch, length, heads, dim).transpose(1, 2)
    assert (got - want).abs().max().item() <= 2e-2
    assert attention.read_status() == 0


def test_encoder_attention_rescales_when_a_later_key_dominates():
    """Keys in later tiles that score far above a row's running max (8 x the
    row's own query) move the max of some rows of a warp and not others: O is
    rescaled for those rows only (the lazy rescale's j > 0 path)."""
    gen = torch.Generator().manual_seed(11)
    batch, length, heads, dim = 1, 1500, 4, 64
    x = [_rand(gen, (batch, length, heads * dim), torch.bfloat16) for _ in range(3)]
    q4, k4 = (t.view(batch, length, heads, dim) for t in x[:2])
    for row, key in ((0, 700), (37, 1400), (130, 300), (255, 129), (900, 1000)):
        k4[0, key] = (q4[0, row].float() * 8).bfloat16()
    views = [t.to(DEV).view(batch, length, heads, dim).transpose(1, 2) for t in x]
    out = attention.whisper_encoder_attention(*views)
    q, k, v = (t.float().numpy().reshape(batch, length, heads, dim).transpose(0, 2, 1, 3) for t in x)
    want = oracle.encoder_attention(q, k, v)
    got = host(out).reshape(batch, length, heads, dim).transpose(0, 2, 1, 3)
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=0)
    assert attention.read_status() == 0


# ------------------------------------------------------------ edge cases ----

def test_position_outside_cache_sets_status_and_skips_row():
    """A row whose position is past the cache view is not written or read: its
    output is zero and the status word says why (the kernel's own check)."""
    gen = torch.Generator().manual_seed(5)
    heads, dim, bucket = 20, 64, 64
    kc = _rand(gen, (3, heads, bucket, dim), torch.bfloat16).to(DEV)
    vc = kc.clone()
    before = kc.clone()
    q, k, v = (_rand(gen, (3, heads, dim), torch.bfloat16).to(DEV) for _ in range(3))
    positions = torch.tensor([5, bucket, 7], device=DEV)
    out = attention.whisper_self_attention_step(q, k, v, kc, vc, positions)
    torch.cuda.synchronize()
    assert attention.read_status() & _native.STATUS_POSITION
    assert torch.count_nonzero(out[1]) == 0
    assert torch.equal(kc[1], before[1])
    assert torch.count_nonzero(out[0]) > 0


@pytest.mark.parametrize("tag", ["bf16", "fp32"])
def test_ragged_rows_share_ctas_and_rearm(tag):
    """Rows of very different lengths, rows outside the view and a row at
    position 0 in one call: the long row is split over many CTAs while short
    rows take one. Three calls on the same workspace must each match the
    reference (the split-merge counters re-arm themselves)."""
    dtype = DTYPES[tag]
    gen = torch.Generator().manual_seed(11)
    dim, kv_heads, heads, bucket = 128, 8, 16, 1024
    qkv, qn, kn, cos, sin, k_store, v_store, _ = _qwen3_inputs(gen, 4, bucket, heads, dtype)
    kd, vd = k_store.to(DEV), v_store.to(DEV)
    for positions in ([bucket - 1, 0, bucket + 5, 3], [-1, 700, 1, bucket - 1], [17, 16, 15, 0]):
        positions = torch.tensor(positions)
        k_before, v_before = host(kd), host(vd)
        out = attention.qwen3_attention_step(qkv.to(DEV), qn.to(DEV), kn.to(DEV), 1e-6,
                                             cos.to(DEV), sin.to(DEV), positions.to(DEV),
                                             kd[:4, :bucket], vd[:4, :bucket], heads, kv_heads)
        valid = ((positions >= 0) & (positions < bucket)).numpy()
        safe = torch.where(torch.from_numpy(valid), positions, torch.zeros_like(positions))
        want, k_after, _ = oracle.qwen3_decode_attention(
            qkv.float().numpy(), qn.float().numpy(), kn.float().numpy(), 1e-6,
            cos.float().numpy(), sin.float().numpy(), safe.numpy(), k_before[:4, :bucket],
            v_before[:4, :bucket], heads, kv_heads, bf16=dtype == torch.bfloat16)
        got = host(out)
        np.testing.assert_allclose(got[valid], want[valid], atol=TOL[dtype], rtol=0)
        assert not got[~valid].any()
        got_k = host(kd)
        np.testing.assert_allclose(got_k[:4][valid, :bucket], k_after[valid], atol=TOL[dtype],
                                   rtol=0)
        np.testing.assert_array_equal(got_k[:4][~valid], k_before[:4][~valid])
        status = attention.read_status()
        assert bool(status & _native.STATUS_POSITION) == (not valid.all())
        assert not status & _native.STATUS_TIMEOUT


def test_graph_capture_replays_with_new_positions():
    from asrback_b200.transcription import CapturedGraph

    gen = torch.Generator().manual_seed(9)
    heads, dim, batch = 20, 64, 8
    kc = _rand(gen, (batch, heads, 448, dim), torch.bfloat16).to(DEV)
    vc = _rand(gen, (batch, heads, 448, dim), torch.bfloat16).to(DEV)
    xc = _rand(gen, (batch, heads, 1500, dim), torch.bfloat16).to(DEV)
    q, k, v = (_rand(gen, (batch, heads, dim), torch.bfloat16).to(DEV) for _ in range(3))
    positions = torch.zeros(batch, dtype=torch.int64, device=DEV)
    result = {}

    def step():
        result["self"] = attention.whisper_self_attention_step(q, k, v, kc, vc, positions)
        result["cross"] = attention.whisper_cross_attention_step(q, xc, xc)

    graph = CapturedGraph(step)
    new_positions = torch.randint(0, 448, (batch,), generator=gen)
    positions.copy_(new_positions)
    graph.replay()
    torch.cuda.synchronize()
    got_self, got_cross = result["self"].clone(), result["cross"].clone()
    step()
    torch.cuda.synchronize()
    assert torch.equal(got_self, result["self"])
    assert torch.equal(got_cross, result["cross"])


def test_graphs_of_earlier_buckets_survive_a_workspace_growth():
    """The reference captures one graph per batch bucket in ascending order;
    when a later bucket's warm-up needs a larger split workspace, the graphs
    captured before keep the buffer they baked in (it is never freed), so
    replaying them still matches an eager call."""
    from asrback_b200.transcription import CapturedGraph

    lib = _native.load()
    heads, dim, length = 20, 64, 1500
    need = {b: lib.asrback_decode_workspace_bytes(b, heads, dim, length) for b in range(1, 65)}
    small = 1
    large = next((b for b in range(2, 65) if need[b] > need[small]), None)
    assert large is not None, need
    gen = torch.Generator().manual_seed(21)
    xk = _rand(gen, (large, heads, length, dim), torch.bfloat16).to(DEV)
    xv = _rand(gen, (large, heads, length, dim), torch.bfloat16).to(DEV)
    q = _rand(gen, (large, heads, dim), torch.bfloat16).to(DEV)
    result = {}

    def step(batch):
        result[batch] = attention.whisper_cross_attention_step(q[:batch], xk[:batch], xv[:batch])

    graphs = {batch: CapturedGraph(lambda batch=batch: step(batch)) for batch in (small, large)}
    for _ in range(3):
        graphs[small].replay()
        graphs[large].replay()
    torch.cuda.synchronize()
    got = {batch: result[batch].clone() for batch in (small, large)}
    for batch in (small, large):
        step(batch)
    torch.cuda.synchronize()
    for batch in (small, large):
        assert torch.equal(got[batch], result[batch]), batch
    assert attention.read_status() == 0
