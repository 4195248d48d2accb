"""Loading of the committed golden vectors (bf16 bit patterns -> float32)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def from_bits(a: np.ndarray) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype == np.uint16:
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def load(name: str) -> dict:
    with np.load(GOLDEN / name) as f:
        return {k: f[k] for k in f.files}


def ints() -> dict:
    return json.loads((GOLDEN / "int_helpers.json").read_text())
