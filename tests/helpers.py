"""Test helpers: golden fixtures, seeded inputs and tolerance checks."""

from __future__ import annotations

import glob
import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances of the north-star contract, written out where they are used:
#   fp32 kernel vs fp32 oracle: max|o - ref| / max|ref| <= 1e-4
#   bf16/f16 kernel vs fp32 oracle on the same rounded inputs: max|o - ref| <= 2e-2
FP32_REL_TOL = 1e-4
BF16_ABS_TOL = 2e-2


def golden_cases(kind="kernel"):
    out = []
    for path in sorted(glob.glob(os.path.join(GOLDEN, "*.npz"))):
        z = np.load(path)
        meta = json.loads(str(z["meta"]))
        if meta["kind"] == kind:
            out.append((os.path.basename(path)[:-4], z, meta))
    return out


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return z, json.loads(str(z["meta"]))


def seeded_inputs(B, H_q, H_k, T, d, L, seed, extra_rows=0, dtype=np.float32):
    rng = np.random.default_rng(seed)
    R = T * L + extra_rows
    Q = rng.standard_normal((B, H_q, T, d), dtype=np.float32)
    K = rng.standard_normal((B, H_k, T, d), dtype=np.float32)
    V = rng.standard_normal((B, H_k, T, d), dtype=np.float32)
    Kd = rng.standard_normal((B, H_k, R, d), dtype=np.float32)
    Vd = rng.standard_normal((B, H_k, R, d), dtype=np.float32)
    return [a.astype(dtype) for a in (Q, K, V, Kd, Vd)]


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def rel_err(o, ref):
    ref = np.asarray(ref, np.float64)
    den = float(np.max(np.abs(ref))) if ref.size else 1.0
    return max_abs(o, ref) / max(den, 1e-30)
