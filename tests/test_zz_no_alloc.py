"""The cross-attention step that allocates nothing, against the workspace one.

asrback_whisper_cross_attention_step_noalloc serves callers that cannot
allocate device memory (a host binding the C ABI from another language with no
device allocator, or a serving loop that must not call cudaMalloc because it
synchronizes the device). Its split-KV scratch is a static device array shared
by every call, so these tests call it twice in a row with different inputs and
compare each result with the existing entry point's, within the bf16/fp32
tolerances the decode tests use. The file is named to be collected last.
"""

from __future__ import annotations

import math
import os

import pytest
import torch

from asrback_b200 import _native, attention

pytestmark = pytest.mark.gpu

TOL = {torch.bfloat16: 2e-2, torch.float32: 1e-4}


def noalloc_cross(query, key_cache, value_cache, status):
    """Calls the no-allocation entry point through the C ABI."""
    batch, heads, head_dim = query.shape
    length = key_cache.shape[2]
    out = torch.empty((batch, 1, heads * head_dim), dtype=query.dtype, device=query.device)
    code = _native.BF16 if query.dtype == torch.bfloat16 else _native.F32
    _native.call(
        "asrback_whisper_cross_attention_step_noalloc",
        code, batch, heads, head_dim, length,
        query.data_ptr(), query.stride(0), query.stride(1),
        key_cache.data_ptr(), value_cache.data_ptr(), key_cache.stride(0), key_cache.stride(1),
        out.data_ptr(), heads * head_dim, head_dim, 1.0 / math.sqrt(head_dim),
        status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("batch,length", [(2, 1500), (1, 1500), (64, 1500), (3, 77)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, batch, length):
    device = torch.device("cuda", 0)
    heads, dim = 20, 64
    status = torch.zeros(1, dtype=torch.int32, device=device)
    for call in range(2):
        gen = torch.Generator(device=device).manual_seed(100 * call + batch)
        q = torch.randn((batch, heads, dim), generator=gen, device=device, dtype=dtype)
        kc = torch.randn((batch, heads, length, dim), generator=gen, device=device, dtype=dtype)
        vc = torch.randn((batch, heads, length, dim), generator=gen, device=device, dtype=dtype)
        want = attention.whisper_cross_attention_step(q, kc, vc)
        got = noalloc_cross(q, kc, vc, status)
        torch.cuda.synchronize()
        err = (got.float() - want.float()).abs().max().item()
        assert err <= TOL[dtype], (call, err)
    assert status.item() == 0


def test_noalloc_rejects_splits_beyond_its_scratch(monkeypatch):
    """Forcing 128-key splits of 256 keys over 5000 (row, head) units needs
    more than the static scratch (any tile size up to 128 keys splits them in
    two): the call is refused on the host, before any launch."""
    device = torch.device("cuda", 0)
    monkeypatch.setenv("ASRBACK_SPLIT_CHUNK", "128")
    q = torch.zeros((250, 20, 64), dtype=torch.bfloat16, device=device)
    kc = torch.zeros((250, 20, 256, 64), dtype=torch.bfloat16, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    with pytest.raises(_native.NativeError, match="no-allocation entry point holds"):
        noalloc_cross(q, kc, kc, status)
    assert os.environ["ASRBACK_SPLIT_CHUNK"] == "128"
