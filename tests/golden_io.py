"""Load the golden fixtures written by tests/golden/make_golden.py."""

from __future__ import annotations

import json
import os
from functools import lru_cache

import numpy as np

GOLDEN_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def dec(arr: np.ndarray, dtype: str) -> np.ndarray:
    """Stored array -> float32 values (bfloat16 was stored as uint16 bits)."""
    if dtype == "bfloat16":
        return (arr.astype(np.uint32) << 16).view(np.float32)
    return arr


@lru_cache(maxsize=None)
def load(name: str) -> dict:
    """Return {case: {"params": dict, field: (array, dtype_str)}}."""
    z = np.load(os.path.join(GOLDEN_DIR, name))
    cases: dict = {}
    for key in z.files:
        case, field = key.split("/", 1)
        c = cases.setdefault(case, {})
        if field == "params":
            c["params"] = json.loads(str(z[key]))
    for key in z.files:
        case, field = key.split("/", 1)
        if field == "params" or field.endswith(".dtype"):
            continue
        dkey = f"{case}/{field}.dtype"
        dt = str(z[dkey]) if dkey in z.files else str(z[key].dtype)
        cases[case][field] = (dec(z[key], dt), dt)
    return cases


def cases(name: str, fn: str | None = None):
    for cname, c in sorted(load(name).items()):
        if fn is None or c["params"].get("fn") == fn:
            yield cname, c


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bitwise equality of float arrays (NaN payloads ignored, sign of zero kept)."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    if a.shape != b.shape:
        return False
    na, nb = np.isnan(a), np.isnan(b)
    if not np.array_equal(na, nb):
        return False
    return np.array_equal(a[~na].view(np.uint32), b[~nb].view(np.uint32))
