"""The oracle (oracle/moda_oracle.py) against the reference's own outputs.

The golden fixtures in tests/golden/ were produced by running the reference
implementation (moda_attention_naive, DepthKVCache) on CPU in fp32; see
tests/golden/make_golden.py. These tests pin the numpy restatement to them.
"""

import numpy as np
import pytest

from oracle import moda_oracle as orc
from helpers import golden_cases, load_golden, max_abs, seeded_inputs

KERNEL_CASES = golden_cases("kernel")


@pytest.mark.parametrize("name,z,meta", KERNEL_CASES, ids=[c[0] for c in KERNEL_CASES])
def test_oracle_matches_reference_outputs(name, z, meta):
    args = [z[k] for k in ("Q", "K", "V", "K_depth", "V_depth")]
    checked = 0
    for C in meta["chunk_sizes"]:
        key = "full" if C is None else f"c{C}"
        if "err_" + key in z.files:
            # the reference raised for this form; so does the restatement
            with pytest.raises(ValueError):
                orc.moda_attention_naive(*args, meta["L"], meta["scale"], C)
            continue
        ref = z["out_" + key]
        out = orc.moda_attention_naive(*args, meta["L"], meta["scale"], C)
        # reference ran in fp32; the oracle runs in fp64
        assert max_abs(out, ref) < 2e-5, (name, key, max_abs(out, ref))
        checked += 1
    assert checked >= 1


def test_golden_c1_is_the_seeded_benchmark_case():
    z, meta = load_golden("c1_b1_h4x2_t32_d64_l8")
    assert (meta["B"], meta["H_q"], meta["H_k"], meta["T"], meta["d"], meta["L"], meta["seed"]) == \
        (1, 4, 2, 32, 64, 8, 0)
    assert z["K_depth"].shape == (1, 2, 256, 64)


def test_oracle_fp32_mode_matches_fp64():
    args = seeded_inputs(1, 4, 2, 24, 32, 3, seed=5)
    a = orc.moda_attention_naive(*args, 3, chunk_size=8, dtype=np.float32)
    b = orc.moda_attention_naive(*args, 3, chunk_size=8)
    assert a.dtype == np.float32 and max_abs(a, b) < 1e-5


@pytest.mark.parametrize("C", [1, 3, 5, 16, 64])
def test_oracle_chunk_invariance(C):
    args = seeded_inputs(1, 2, 1, 13, 16, 4, seed=6)
    full = orc.moda_attention_naive(*args, 4)
    assert max_abs(orc.moda_attention_naive(*args, 4, chunk_size=C), full) < 1e-12


def test_oracle_rows_match_full():
    args = seeded_inputs(2, 4, 2, 19, 16, 5, seed=7)
    full = orc.moda_attention_naive(*args, 5)
    rows = [(0, 0, 0), (1, 3, 18), (0, 2, 7), (1, 1, 11)]
    got = orc.moda_rows(*args, 5, rows)
    for i, (b, h, t) in enumerate(rows):
        assert max_abs(got[i], full[b, h, t]) < 1e-12


def test_oracle_depth_rows_short_raises():
    # D1: a depth buffer with fewer than T*L rows is an error in the reference.
    Q, K, V, Kd, Vd = seeded_inputs(1, 2, 2, 8, 16, 3, seed=8)
    with pytest.raises(ValueError):
        orc.moda_attention_naive(Q, K, V, Kd[:, :, :20], Vd[:, :, :20], 3, chunk_size=4)


@pytest.mark.parametrize("shape", [(2, 4, 2, 0, 32, 3), (0, 4, 2, 5, 32, 3)], ids=["T0", "B0"])
@pytest.mark.parametrize("chunk", [None, 4])
def test_oracle_empty_inputs(shape, chunk):
    # moda_attention_naive on an empty sequence (T = 0) or batch (B = 0) returns an empty
    # O of Q's shape (torch's matmul / softmax of empty tensors), and autograd gives empty
    # gradients of the inputs' shapes; the oracle does the same.
    B, Hq, Hk, T, d, L = shape
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=10)
    assert orc.moda_attention_naive(*arrs, L, chunk_size=chunk).shape == (B, Hq, T, d)
    g = orc.moda_attention_grads(*arrs, L, np.zeros((B, Hq, T, d)))
    for k, a in zip(("dQ", "dK", "dV", "dK_depth", "dV_depth"), arrs):
        assert g[k].shape == a.shape, k


def test_oracle_causal_and_depth_isolation():
    # reference tests/test_kernel.py:32-59, restated on the oracle
    Q, K, V, Kd, Vd = seeded_inputs(1, 1, 1, 4, 8, 3, seed=9)
    out = orc.moda_attention_naive(Q, K, V, Kd, Vd, 3)
    K2 = K.copy(); K2[0, 0, 2] = 999.0
    Kd2 = Kd.copy(); Kd2[0, 0, 6:9] = 999.0
    assert max_abs(orc.moda_attention_naive(Q, K2, V, Kd, Vd, 3)[:, :, 0], out[:, :, 0]) == 0
    assert max_abs(orc.moda_attention_naive(Q, K, V, Kd2, Vd, 3)[:, :, 0], out[:, :, 0]) == 0


def test_depth_cache_write_restatement():
    z, meta = load_golden("cache_write")
    B, T, L, H, d = meta["B"], meta["T"], meta["L"], meta["H_k"], meta["d"]
    kc = np.zeros((B, H, T * L, d), np.float32)
    vc = np.zeros_like(kc)
    for layer in meta["order"]:
        orc.depth_cache_write(kc, vc, layer, z[f"k{layer}"], z[f"v{layer}"], L)
    assert max_abs(kc, z["k_cache"]) == 0 and max_abs(vc, z["v_cache"]) == 0
    assert tuple(z["partial_shape"]) == (B, H, 3 * L, d)


def test_roofline_formulas():
    # kernel-only benchmark configuration: B=4 H_q=32 H_k=8 T=8192 d=128 L=32 bf16
    f = orc.flops(4, 32, 8192, 128, 32)
    by = orc.hbm_bytes(4, 32, 8, 8192, 128, 32, 2)
    assert abs(f / 1e12 - 2.2165) < 1e-3
    assert abs(by / 1e9 - 4.966) < 1e-3


GRAD_CASES = golden_cases("grad")
GRAD_KEYS = ("O", "dQ", "dK", "dV", "dK_depth", "dV_depth")


@pytest.mark.parametrize("name,z,meta", GRAD_CASES, ids=[c[0] for c in GRAD_CASES])
def test_grad_oracle_matches_reference_autograd(name, z, meta):
    """The closed-form backward equals torch autograd through the reference (fp64)."""
    r = orc.moda_attention_grads(z["Q"], z["K"], z["V"], z["K_depth"], z["V_depth"], meta["L"],
                                 z["dO"], scale=meta["scale"])
    for k in GRAD_KEYS:
        ref = z[k].astype(np.float64)
        assert r[k].shape == ref.shape, k
        assert max_abs(r[k], ref) <= 1e-6 * max(1.0, float(np.max(np.abs(ref)))), k
    if meta["depth_rows"] > meta["T"] * meta["L"]:
        # rows past T*L are never read: zero gradient, as in the reference
        assert not np.any(z["dK_depth"][:, :, meta["T"] * meta["L"]:])


def test_grad_oracle_lse_matches_forward():
    z, meta = GRAD_CASES[0][1], GRAD_CASES[0][2]
    r = orc.moda_attention_grads(z["Q"], z["K"], z["V"], z["K_depth"], z["V_depth"], meta["L"],
                                 z["dO"], scale=meta["scale"])
    o = orc.moda_attention_naive(z["Q"], z["K"], z["V"], z["K_depth"], z["V_depth"], meta["L"],
                                 scale=meta["scale"])
    assert max_abs(r["O"], o) < 1e-12
    # lse row by row from the single-row form
    f64 = lambda a: np.asarray(a, np.float64)
    q, k, kd = f64(z["Q"][0, 1, 5]), f64(z["K"][0, 0, :6]), f64(z["K_depth"][0, 0, 5 * meta["L"]:6 * meta["L"]])
    s = np.concatenate([k @ q, kd @ q]) * z["Q"].shape[-1] ** -0.5
    assert abs(r["lse"][0, 1, 5] - (s.max() + np.log(np.exp(s - s.max()).sum()))) < 1e-9


def test_token_grads_match_reference_autograd_fixtures():
    # the per-token restatement used for full-size spot checks, against the reference's
    # own fp64 autograd (tests/golden/make_golden.py: grad_case)
    for name in ("grad_b1_h4x2_t32_d64_l8", "grad_b1_h8x2_t20_d64_l3_extra8"):
        z, meta = load_golden(name)
        L = meta["L"]
        G = z["Q"].shape[1] // z["K"].shape[1]
        scale = meta.get("scale") or z["Q"].shape[-1] ** -0.5
        for (b, hk, t) in [(0, 0, 0), (0, 1, 7), (0, 0, z["Q"].shape[2] - 1)]:
            heads = slice(hk * G, (hk + 1) * G)
            r = orc.moda_token_grads(z["Q"][b, heads, t], z["dO"][b, heads, t], z["K"][b, hk, :t + 1],
                                     z["V"][b, hk, :t + 1], z["K_depth"][b, hk, t * L:(t + 1) * L],
                                     z["V_depth"][b, hk, t * L:(t + 1) * L], scale)
            # the fixtures store the fp64 gradients as float32 (rounding ~1e-8 here)
            assert max_abs(r["dQ"], z["dQ"][b, heads, t]) < 1e-6
            assert max_abs(r["dK_depth"], z["dK_depth"][b, hk, t * L:(t + 1) * L]) < 1e-6
            assert max_abs(r["dV_depth"], z["dV_depth"][b, hk, t * L:(t + 1) * L]) < 1e-6
