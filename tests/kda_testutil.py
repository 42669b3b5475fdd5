"""Shared helpers for the KDA tests: golden fixtures and the relative-error metric."""
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# north-star tolerances (max |delta| / max |ref|, the reference's own error form,
# nope_gdn_mlx.py:4824-4825)
TOL_FP32 = 1e-4
TOL_BF16 = 2e-2

OUT_KEYS = ("o", "S_T", "dq", "dk", "dv", "dg", "dbeta", "dstate0")


def manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return json.load(f)


def golden(name):
    return dict(np.load(os.path.join(GOLDEN, f"{name}.npz")))


def rel_err(x, ref):
    x = np.asarray(x, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(x - ref).max() / max(den, 1e-30))
