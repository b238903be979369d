"""Seeded random sweep: forward (and a third of the cases' backward) vs the oracle.

Shapes are drawn from a fixed generator, one test per case, across both kernels:
G in {1..128}, head_dim in {32, 64, 96, 128}, T in {1 .. 300} (ragged tiles, one
token, exact multiples of 128), L in {1 .. 100}, bf16 / f16 / fp32, with and without
chunk_size, and depth buffers with extra rows past T*L (which the kernels never read).
Tolerances as everywhere: fp32 1e-4 relative, bf16/f16 2e-2 absolute (forward);
gradients 1e-4 (fp32) / 3e-2 (16-bit) of the largest reference magnitude.
"""

import random

import numpy as np
import pytest
import torch

from moda.kernels import device_status, moda_attention_cuda
from oracle import moda_oracle as orc
from helpers import BF16_ABS_TOL, FP32_REL_TOL, max_abs, rel_err, seeded_inputs

pytestmark = pytest.mark.gpu


def _cases(n=80, seed=2024):
    rng = random.Random(seed)
    out = []
    while len(out) < n:
        G = rng.choice([1, 2, 4, 8, 16, 32, 64, 128])
        Hk = rng.choice([1, 2, 3]) if G <= 16 else 1
        d = rng.choice([64, 128, 64, 128, 32, 96])
        T = rng.choice([1, 2, 3, 17, 31, 64, 65, 127, 128, 129, 200, 255, 256, 257, 300])
        L = rng.choice([1, 2, 3, 5, 8, 12, 16, 24, 31, 32, 33, 48, 64, 100])
        B = rng.choice([1, 2])
        if G * Hk * T * (T + T * L) > 2e7:
            continue
        dtype = rng.choice(["bf16", "f16", "fp32"])
        chunk = rng.choice([None, 16, 64, 100])
        extra = rng.choice([0, 0, 7])
        grads = rng.random() < 0.35 and T <= 200 and not extra
        out.append((B, G * Hk, Hk, T, d, L, dtype, chunk, extra, grads))
    return out


CASES = _cases()
DT = {"bf16": torch.bfloat16, "f16": torch.float16, "fp32": torch.float32}


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert device_status() == 0, "a bounded device wait expired"


@pytest.mark.parametrize("idx", range(len(CASES)), ids=[f"{i}:" + "-".join(map(str, c)) for i, c in enumerate(CASES)])
def test_random_shape_matches_oracle(idx):
    B, Hq, Hk, T, d, L, dts, chunk, extra, grads = CASES[idx]
    dtype = DT[dts]
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=1000 + idx, extra_rows=extra)
    args = [torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype) for a in arrs]
    rin = [torch.from_numpy(np.ascontiguousarray(a)).to(dtype).double().numpy() for a in arrs]
    # the unchunked reference needs exactly T*L depth rows; the chunked one reads only those
    ref = orc.moda_attention_naive(*rin, L, chunk_size=(chunk or 64) if extra else chunk)
    out = moda_attention_cuda(*args, L, None, chunk)
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    if dtype == torch.float32:
        assert rel_err(o, ref) <= FP32_REL_TOL, rel_err(o, ref)
    else:
        assert max_abs(o, ref) <= BF16_ABS_TOL, max_abs(o, ref)
    if not grads:
        return
    ins = [a.clone().requires_grad_(True) for a in args]
    dO = np.random.RandomState(idx).standard_normal((B, Hq, T, d))
    dO_t = torch.from_numpy(dO).to("cuda", dtype)
    moda_attention_cuda(*ins, L, None, chunk).backward(dO_t)
    g = orc.moda_attention_grads(*rin, L, dO_t.double().cpu().numpy())
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    for t, k in zip(ins, ("dQ", "dK", "dV", "dK_depth", "dV_depth")):
        e = float(np.abs(t.grad.double().cpu().numpy() - g[k]).max()) / max(1.0, float(np.abs(g[k]).max()))
        assert e <= tol, (k, e)
