"""Shared test helpers: ulp distances, oracle inputs, library handles."""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def ulp_diff_f32(a, b):
    """Elementwise distance in units in the last place between two f32
    arrays (0 when bit-identical; NaN vs NaN counts as 0)."""
    a = np.ascontiguousarray(a, dtype=np.float32).view(np.int32).astype(np.int64)
    b = np.ascontiguousarray(b, dtype=np.float32).view(np.int32).astype(np.int64)
    # map the sign-magnitude float order onto the integers
    a = np.where(a < 0, -(a & 0x7FFFFFFF), a)
    b = np.where(b < 0, -(b & 0x7FFFFFFF), b)
    return np.abs(a - b)


def header_functions():
    """Every function the C ABI header declares."""
    with open(os.path.join(ROOT, "include", "zpucuda.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(zpucuda_[a-z0-9_]+)\s*\(", text)))


def rel_fro(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))
