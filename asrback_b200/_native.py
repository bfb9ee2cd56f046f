"""ctypes binding of ``libasrback_attn.so`` (the C ABI in ``include/asrback_attn.h``).

The library is built in-tree by ``asrback_b200.build`` (or ``__graft_entry__.build``)
into ``asrback_b200/_lib``. There is no fallback: if it is missing or does not
load, every attention call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "_lib" / "libasrback_attn.so"

BF16 = 0
F32 = 1

OK = 0
ERR_ARGUMENT = 1
ERR_CUDA = 2
ERR_WORKSPACE = 3

STATUS_POSITION = 1
STATUS_TIMEOUT = 2
STATUS_SEGMENT = 4

ABI_MAJOR = 1

_c_int, _c_i64, _c_p, _c_f, _c_size = (
    ctypes.c_int,
    ctypes.c_int64,
    ctypes.c_void_p,
    ctypes.c_float,
    ctypes.c_size_t,
)

# Every exported function with its argument and return types, in header order.
SIGNATURES: dict[str, tuple[list, object]] = {
    "asrback_abi_version": ([], _c_int),
    "asrback_last_error": ([], ctypes.c_char_p),
    "asrback_device_sm_count": ([], _c_int),
    "asrback_decode_workspace_bytes": ([_c_int, _c_int, _c_int, _c_int], _c_size),
    "asrback_whisper_self_attention_step": (
        [_c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_p, _c_i64, _c_i64,
         _c_p, _c_p, _c_i64, _c_i64,
         _c_p,
         _c_p, _c_i64, _c_i64,
         _c_f, _c_p, _c_size, _c_p, _c_p],
        _c_int,
    ),
    "asrback_whisper_cross_attention_step": (
        [_c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64,
         _c_f, _c_p, _c_size, _c_p, _c_p],
        _c_int,
    ),
    "asrback_whisper_prefix_workspace_bytes": ([_c_int, _c_int, _c_int, _c_int, _c_int], _c_size),
    "asrback_whisper_self_attention_prefix": (
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64,
         _c_f, _c_p, _c_size, _c_p, _c_p],
        _c_int,
    ),
    "asrback_whisper_cross_attention_prefix": (
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64,
         _c_f, _c_p, _c_size, _c_p, _c_p],
        _c_int,
    ),
    "asrback_whisper_cross_attention_step_noalloc": (
        [_c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64,
         _c_f, _c_p, _c_p],
        _c_int,
    ),
    "asrback_qwen3_attention_step": (
        [_c_int, _c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64,
         _c_p, _c_p, _c_f,
         _c_p, _c_p, _c_i64, _c_int,
         _c_p,
         _c_p, _c_p, _c_i64,
         _c_p, _c_i64,
         _c_f, _c_p, _c_size, _c_p, _c_p],
        _c_int,
    ),
    "asrback_whisper_encoder_attention": (
        [_c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_p, _c_p, _c_p,
         _c_i64, _c_i64, _c_i64,
         _c_f, _c_p, _c_p],
        _c_int,
    ),
    "asrback_varlen_attention": (
        [_c_int, _c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_f, _c_p, _c_p],
        _c_int,
    ),
    "asrback_whisper_cross_kv_projection": (
        [_c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_p, _c_i64, _c_p,
         _c_p, _c_p,
         _c_i64, _c_i64, _c_i64,
         _c_p, _c_p],
        _c_int,
    ),
    "asrback_greedy_step_workspace_bytes": ([_c_int], _c_size),
    "asrback_greedy_step": (
        [_c_int, _c_int, _c_int, _c_int,
         _c_p, _c_i64,
         _c_p, _c_i64,
         _c_p,
         _c_p, _c_p,
         _c_p, _c_i64, _c_p, _c_p,
         _c_p, _c_p,
         _c_p, _c_i64, _c_i64,
         _c_p, _c_int,
         _c_p, _c_size, _c_p, _c_p],
        _c_int,
    ),
    "asrback_selftest_bounded_wait": ([_c_i64, _c_p, _c_p], _c_int),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class NativeError(RuntimeError):
    """A call into libasrback_attn failed (bad argument, CUDA error, ...)."""


def library_path() -> Path:
    override = os.environ.get("ASRBACK_LIBRARY")
    return Path(override) if override else LIBRARY


def load() -> ctypes.CDLL:
    """The loaded library with typed entry points; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = library_path()
        if not path.is_file():
            raise NativeError(
                f"{path} is missing: build it with `python -m asrback_b200.build` "
                "(asrback_b200 has no CPU or PyTorch fallback)"
            )
        lib = ctypes.CDLL(str(path))
        for name, (argtypes, restype) in SIGNATURES.items():
            function = getattr(lib, name)
            function.argtypes = argtypes
            function.restype = restype
        version = lib.asrback_abi_version()
        if version >> 16 != ABI_MAJOR:
            raise NativeError(f"{path} has ABI {version >> 16}.{version & 0xFFFF}, expected {ABI_MAJOR}.x")
        _lib = lib
        return lib


def call(name: str, *args) -> None:
    """Calls entry point ``name``; raises :class:`NativeError` with the
    library's message when it returns an error code."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != OK:
        message = lib.asrback_last_error().decode(errors="replace")
        kind = {ERR_ARGUMENT: "invalid argument", ERR_CUDA: "CUDA error",
                ERR_WORKSPACE: "workspace too small"}.get(rc, f"error {rc}")
        raise NativeError(f"{name}: {kind}: {message}")
