"""The C ABI library loads and exports what include/asrback_attn.h declares;
host-side argument checks reject bad calls before any launch (no GPU needed)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from asrback_b200 import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "asrback_attn.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"ASRBACK_API\s+[\w\s\*]+?\b(asrback_\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    return _native.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert "asrback_whisper_self_attention_step" in names
    assert "asrback_qwen3_attention_step" in names
    assert len(names) == len(set(names))


def test_every_declared_symbol_is_exported(lib):
    for name in declared_functions():
        assert hasattr(lib, name), name
    # ... and the binding types every one of them.
    assert set(declared_functions()) <= set(_native.SIGNATURES)


def test_abi_version(lib):
    assert lib.asrback_abi_version() >> 16 == _native.ABI_MAJOR


def test_workspace_size_is_host_only(lib):
    small = lib.asrback_decode_workspace_bytes(64, 20, 64, 448)
    assert small >= 256
    big = lib.asrback_decode_workspace_bytes(1, 20, 64, 1500)
    assert big > 256  # one row: keys split over many CTAs, partials needed
    assert lib.asrback_decode_workspace_bytes(0, 20, 64, 448) == 0


def _self_call(lib, **overrides):
    args = dict(dtype=_native.BF16, batch=2, heads=20, head_dim=64, length=448,
                q=16, k=16, v=16, kc=16, vc=16, pos=16, out=16)
    args.update(overrides)
    return lib.asrback_whisper_self_attention_step(
        args["dtype"], args["batch"], args["heads"], args["head_dim"], args["length"],
        args["q"], 1280, 64, args["k"], args["v"], 1280, 64,
        args["kc"], args["vc"], 20 * 448 * 64, 448 * 64, args["pos"],
        args["out"], 1280, 64, 0.125, None, 0, None, None)


@pytest.mark.parametrize("overrides,fragment", [
    (dict(head_dim=32), "head_dim must be 64"),
    (dict(dtype=7), "dtype"),
    (dict(batch=0), "positive"),
    (dict(q=0), "null"),
    (dict(q=8), "aligned"),
    (dict(pos=0), "positions"),
])
def test_invalid_arguments_are_rejected_on_the_host(lib, overrides, fragment):
    rc = _self_call(lib, **overrides)
    assert rc == _native.ERR_ARGUMENT
    assert fragment in lib.asrback_last_error().decode()


def test_missing_workspace_is_rejected(lib):
    # One row over 1500 keys splits, so a workspace is required.
    rc = lib.asrback_whisper_cross_attention_step(
        _native.BF16, 1, 20, 64, 1500, 16, 1280, 64, 16, 16, 20 * 1500 * 64, 1500 * 64,
        16, 1280, 64, 0.125, None, 0, None, None)
    assert rc == _native.ERR_WORKSPACE


def test_qwen3_shape_limits(lib):
    rc = lib.asrback_qwen3_attention_step(
        _native.BF16, 4, 16, 4, 128, 1024, 16, 4096, 16, 16, 1e-6, 16, 16, 128, 1024, 16,
        16, 16, 1024 * 1024, 16, 2048, 0.088, None, 0, None, None)
    assert rc == _native.ERR_ARGUMENT
    assert "8 key/value heads" in lib.asrback_last_error().decode()


def _varlen_call(lib, **overrides):
    args = dict(dtype=_native.BF16, tokens=512, heads=16, kv_heads=8, head_dim=128, q=16, k=16,
                v=16, cu=16, segments=2, max_length=256, out=16, q_tok=2048)
    args.update(overrides)
    return lib.asrback_varlen_attention(
        args["dtype"], args["tokens"], args["heads"], args["kv_heads"], args["head_dim"],
        args["q"], args["q_tok"], 128, args["k"], 1024, 128, args["v"], 4096, 128,
        args["cu"], args["segments"], args["max_length"], 1,
        args["out"], 2048, 128, 0.088, None, None)


@pytest.mark.parametrize("overrides,fragment", [
    (dict(head_dim=96), "head_dim must be 64 or 128"),
    (dict(heads=12), "multiple of kv_heads"),
    (dict(segments=0), "positive"),
    (dict(cu=0), "null"),
    (dict(k=8), "aligned"),
    (dict(q_tok=1000), "do not hold"),
])
def test_varlen_invalid_arguments_are_rejected_on_the_host(lib, overrides, fragment):
    rc = _varlen_call(lib, **overrides)
    assert rc == _native.ERR_ARGUMENT
    assert fragment in lib.asrback_last_error().decode()


def test_bounded_wait_selftest_checks_its_budget(lib):
    assert lib.asrback_selftest_bounded_wait(0, 16, None) == _native.ERR_ARGUMENT
    assert lib.asrback_selftest_bounded_wait(2_000_000_000, 16, None) == _native.ERR_ARGUMENT
    assert lib.asrback_selftest_bounded_wait(1000, None, None) == _native.ERR_ARGUMENT


def test_ops_refuse_cpu_tensors():
    """No CPU fallback: the product path raises on host tensors."""
    import torch

    from asrback_b200 import attention

    q = torch.zeros(2, 20, 64)
    cache = torch.zeros(2, 20, 1500, 64)
    with pytest.raises(ValueError, match="CUDA"):
        attention.whisper_cross_attention_step(q, cache, cache)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "_lib", None)
    monkeypatch.setenv("ASRBACK_LIBRARY", str(tmp_path / "absent.so"))
    with pytest.raises(_native.NativeError, match="no CPU or PyTorch fallback"):
        _native.load()


def test_ctypes_signatures_cover_argument_counts(lib):
    header = HEADER.read_text()
    for name, (argtypes, _) in _native.SIGNATURES.items():
        match = re.search(rf"ASRBACK_API[\w\s\*]+?\b{name}\s*\(([^;]*)\);", header)
        assert match, name
        params = [p for p in match.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(argtypes), name
        assert isinstance(getattr(lib, name), ctypes._CFuncPtr)


def _greedy_call(lib, **overrides):
    args = dict(dtype=_native.BF16, batch=64, vocab=51866, width=1280, hidden=16, h_stride=1280,
                weight=16, w_stride=1280, tokens=None, position=16, generated_cols=448,
                n_eos=1, workspace=16, workspace_bytes=1 << 20)
    args.update(overrides)
    eos = (ctypes.c_int64 * 1)(50257)
    return lib.asrback_greedy_step(
        args["dtype"], args["batch"], args["vocab"], args["width"], args["hidden"],
        args["h_stride"], args["weight"], args["w_stride"], None, None, None,
        args["tokens"], 1, args["position"], 16, 16, 16, 16, 448, args["generated_cols"],
        eos, args["n_eos"], args["workspace"], args["workspace_bytes"], None, None)


@pytest.mark.parametrize("overrides,fragment", [
    (dict(batch=0), "batch must be in [1, 128]"),
    (dict(batch=129), "batch must be in [1, 128]"),
    (dict(dtype=_native.F32, batch=65), "batch must be in [1, 64]"),
    (dict(width=1000, h_stride=1000, w_stride=1001), "16-byte boundaries"),
    (dict(weight=8), "16-byte boundaries"),
    (dict(h_stride=100), "at least hidden_dim"),
    (dict(n_eos=9), "n_eos"),
    (dict(tokens=16, position=None), "state update needs"),
    (dict(tokens=16, generated_cols=0), "state update needs"),
    (dict(workspace=None), "null workspace"),
    (dict(dtype=_native.F32, batch=1, width=65536, h_stride=65536, w_stride=65536), "200 KB"),
])
def test_greedy_step_invalid_arguments_are_rejected_on_the_host(lib, overrides, fragment):
    rc = _greedy_call(lib, **overrides)
    assert rc == _native.ERR_ARGUMENT
    assert fragment in lib.asrback_last_error().decode()


def test_greedy_step_workspace(lib):
    need = lib.asrback_greedy_step_workspace_bytes(64)
    assert need >= 256 + 64 * 16
    assert lib.asrback_greedy_step_workspace_bytes(128) > need
    assert lib.asrback_greedy_step_workspace_bytes(0) == 0
    assert _greedy_call(lib, workspace_bytes=need - 1) == _native.ERR_WORKSPACE


def _cross_kv_call(lib, **overrides):
    args = dict(dtype=_native.BF16, batch=32, tokens=1500, width=1280, x=16, x_sb=1500 * 1280,
                x_st=1280, wk=16, wv=16, w_stride=1280, keys=16, c_st=64)
    args.update(overrides)
    return lib.asrback_whisper_cross_kv_projection(
        args["dtype"], args["batch"], args["tokens"], args["width"], args["x"], args["x_sb"],
        args["x_st"], args["wk"], args["wv"], args["w_stride"], None, args["keys"], 16,
        20 * 1500 * 64, 1500 * 64, args["c_st"], None, None)


@pytest.mark.parametrize("overrides,fragment", [
    (dict(width=1000), "multiple of 128"),
    (dict(batch=0), "positive"),
    (dict(wk=None), "null"),
    (dict(x_st=1000), "(batch, tokens, width)"),
    (dict(c_st=32), "views with contiguous rows"),
    (dict(x=8), "16-byte aligned"),
])
def test_cross_kv_invalid_arguments_are_rejected_on_the_host(lib, overrides, fragment):
    rc = _cross_kv_call(lib, **overrides)
    assert rc == _native.ERR_ARGUMENT
    assert fragment in lib.asrback_last_error().decode()


def _prefix_call(lib, name, **overrides):
    args = dict(dtype=_native.BF16, windows=4, tokens=6, heads=20, head_dim=64, length=448,
                q=16, kc=16, vc=16, out=16, c_sh=448 * 64)
    args.update(overrides)
    return getattr(lib, name)(
        args["dtype"], args["windows"], args["tokens"], args["heads"], args["head_dim"],
        args["length"], args["q"], 1280, 64, args["kc"], args["vc"], 20 * args["c_sh"],
        args["c_sh"], args["out"], 1280, 64, 0.125, None, 0, None, None)


@pytest.mark.parametrize("name", ["asrback_whisper_self_attention_prefix",
                                  "asrback_whisper_cross_attention_prefix"])
@pytest.mark.parametrize("overrides,fragment", [
    (dict(windows=0), "windows"),
    (dict(windows=1000, tokens=100), "65535"),
    (dict(head_dim=32), "head_dim must be 64"),
    (dict(q=0), "null"),
    (dict(kc=8), "aligned"),
    (dict(c_sh=100 * 64), "cache strides"),
])
def test_prefix_invalid_arguments_are_rejected_on_the_host(lib, name, overrides, fragment):
    rc = _prefix_call(lib, name, **overrides)
    assert rc == _native.ERR_ARGUMENT
    assert fragment in lib.asrback_last_error().decode()


def test_self_prefix_tokens_fit_the_cache(lib):
    rc = _prefix_call(lib, "asrback_whisper_self_attention_prefix", tokens=8, length=7)
    assert rc == _native.ERR_ARGUMENT
    assert "exceed the cache length" in lib.asrback_last_error().decode()


def test_prefix_workspace_is_host_only(lib):
    # 32 windows of 4 tokens: 4 tokens per CTA, 640 (window, head) units split
    # in two over 1500 keys, so partials are needed.
    assert lib.asrback_whisper_prefix_workspace_bytes(32, 4, 20, 64, 1500) > 0
    assert lib.asrback_whisper_prefix_workspace_bytes(0, 4, 20, 64, 1500) == 0
    assert lib.asrback_whisper_prefix_workspace_bytes(32, 4, 20, 64, 0) == 0
