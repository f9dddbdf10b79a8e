"""Runs the known-answer vectors of tests/golden/kats.json against an
implementation of the Backend surface (the CPU oracle or the CUDA backend).

An implementation is an object with the methods used below; errors are
reported as exception class names ("InvalidShape", ...).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

KATS = json.loads((Path(__file__).parent / "golden" / "kats.json").read_text())["kats"]


def f(values):
    return np.array([float(v) for v in values], dtype=np.float32)


def pack_rows(rows):
    """pack_ternary per row (row-aligned), ternary.rs:266-285."""
    out = []
    for r in rows:
        b = [0] * ((len(r) + 3) // 4)
        for i, v in enumerate(r):
            code = 0 if v == 1 else (1 if v == 0 else 2)
            b[i // 4] |= code << (2 * (i % 4))
        out += b
    return np.array(out, dtype=np.uint8)


def by_fn(*names):
    return [k for k in KATS if k["fn"] in names]
