"""Golden fixtures recorded from the reference's modules (see make_golden.py)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load(name: str) -> dict:
    """Fixture ``name`` as a dict of float32/int arrays plus ``meta``; bfloat16
    tensors (stored as raw bits) come back as float32."""
    with np.load(HERE / f"{name}.npz") as data:
        out = {}
        for key in data.files:
            value = data[key]
            if key == "meta":
                out["meta"] = json.loads(str(value))
            elif key.endswith("__bf16"):
                out[key[: -len("__bf16")]] = (value.astype(np.uint32) << 16).view(np.float32)
            else:
                out[key] = value
        return out
