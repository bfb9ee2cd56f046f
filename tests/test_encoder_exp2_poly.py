"""The FMA-pipe exp2 of the encoder kernel (csrc/encoder_attention_tc.cu,
exp2_pair_fma) against its stated error bound, in float32 arithmetic.

2^x = 2^round(x) * q(f), f = x - round(x) in [-1/2, 1/2], q a cubic in Horner
form; round(x) comes from adding 1.5 * 2^23 and its low mantissa bits are
shifted into the exponent field. The constants are read from the kernel source
so the test checks what ships.
"""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np

SOURCE = Path(__file__).resolve().parents[1] / "asrback_b200" / "csrc" / "encoder_attention_tc.cu"


def _constants():
    text = SOURCE.read_text()
    found = {name: np.float32(float(value)) for name, value in
             re.findall(r"constexpr float (kPolyC\d|kRoundMagic) = ([0-9.eE+-]+)f;", text)}
    return [found[f"kPolyC{i}"] for i in range(4)], found["kRoundMagic"]


def _exp2_fma(x: np.ndarray) -> np.ndarray:
    """The kernel's steps, each rounded to float32 as the FMA pipe rounds them
    (an FMA rounds once; numpy's float32 a * b + c rounds twice, so the FMA
    steps are done in float64 and rounded once)."""
    (c0, c1, c2, c3), magic = _constants()
    f32 = np.float32
    x = np.maximum(x.astype(f32), f32(-126.0))
    y = (x + magic).astype(f32)
    r = (y - magic).astype(f32)
    f = (x.astype(np.float64) - r.astype(np.float64)).astype(f32)  # ffma(r, -1, x)
    p = (np.float64(c3) * f + np.float64(c2)).astype(f32)
    p = (p.astype(np.float64) * f + np.float64(c1)).astype(f32)
    p = (p.astype(np.float64) * f + np.float64(c0)).astype(f32)
    bits = p.view(np.int32).astype(np.int64) + (y.view(np.int32).astype(np.int64) << 23)
    return (bits & 0xFFFFFFFF).astype(np.uint32).view(np.int32).view(f32)


def test_cubic_relative_error_on_the_reduced_interval():
    (c0, c1, c2, c3), _ = _constants()
    f = np.linspace(-0.5, 0.5, 200001)
    q = ((c3 * f + c2) * f + c1) * f + c0
    rel = np.abs(q / np.exp2(f) - 1.0)
    assert rel.max() < 7.6e-5, rel.max()


def test_exp2_over_the_softmax_range():
    # Arguments the softmax produces: s * scale - m with the lazy max, so at
    # most +8, and anything below (down to -inf for keys past the window).
    # Results are normal floats from -125 up; below, the reconstruction reaches
    # the denormal range and only the absolute error (below 2^-124, nothing in
    # a bf16 P) is bounded.
    x = np.concatenate([np.linspace(-125.0, 8.0, 400001, dtype=np.float32),
                        np.float32([-0.5, 0.5, -1.5, 7.99, -124.9])])
    got = _exp2_fma(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    rel = np.abs(got / want - 1.0)
    assert rel.max() < 8e-5, (rel.max(), x[np.argmax(rel)])
    low = np.linspace(-126.0, -125.0, 1001, dtype=np.float32)
    err = np.abs(_exp2_fma(low).astype(np.float64) - np.exp2(low.astype(np.float64)))
    assert err.max() < 2.0 ** -124


def test_exp2_underflows_to_nearly_zero():
    x = np.float32([-126.5, -200.0, -1e30, -np.inf])
    got = _exp2_fma(x)
    assert np.all(np.isfinite(got)) and np.all(got >= 0) and np.all(got < 2.0 ** -125)
