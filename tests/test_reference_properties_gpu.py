"""The reference's own kernel and GQA tests, restated on the CUDA forward.

Each test names the reference test it mirrors (tests/test_kernel.py,
tests/test_gqa.py of the reference). Where the reference checks a shape or the
absence of NaN, the CUDA output is also compared with the oracle; where it checks a
relation (weights sum to one, GQA equals MHA on repeated K/V, shared KV heads), the
relation is checked on the CUDA output itself. Both kernels are exercised: the
tcgen05 kernel (16-bit, head_dim 64 / 128) and the CUDA-core kernel (fp32, any
head_dim).
"""

import numpy as np
import pytest
import torch

from moda.kernels import device_status, moda_attention_cuda, moda_plan
from oracle import moda_oracle as orc
from helpers import BF16_ABS_TOL, FP32_REL_TOL, max_abs, rel_err, seeded_inputs

pytestmark = pytest.mark.gpu

# (dtype, head_dim override): fp32 runs the CUDA-core kernel at the reference's
# head_dim; bf16 at head_dim 64 runs the tcgen05 kernel
PATHS = [(torch.float32, None), (torch.bfloat16, 64)]
PATH_IDS = ["fp32-simt", "bf16-tc"]


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert device_status() == 0, "a bounded device wait expired"


def _inputs(B, Hq, Hk, T, L, d, dtype, seed):
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=seed)
    return arrs, [torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype) for a in arrs]


def _check_vs_oracle(out, arrs, L, dtype):
    ref = orc.moda_attention_naive(
        *[torch.from_numpy(np.ascontiguousarray(a)).to(dtype).double().numpy() for a in arrs], L)
    o = out.float().cpu().numpy()
    if dtype == torch.float32:
        assert rel_err(o, ref) <= FP32_REL_TOL, rel_err(o, ref)
    else:
        assert max_abs(o, ref) <= BF16_ABS_TOL, max_abs(o, ref)


@pytest.mark.parametrize("dtype,dh", PATHS, ids=PATH_IDS)
def test_output_shape_and_no_nan(dtype, dh):
    """Reference test_kernel.py:19-30 (test_output_shape, test_no_nan)."""
    for (B, Hq, Hk, T, L, d) in [(2, 4, 2, 8, 3, 16), (1, 2, 2, 4, 2, 8)]:
        d = dh or d
        arrs, args = _inputs(B, Hq, Hk, T, L, d, dtype, seed=60)
        out = moda_attention_cuda(*args, num_layers=L)
        assert tuple(out.shape) == (B, Hq, T, d)
        assert torch.isfinite(out).all()
        _check_vs_oracle(out, arrs, L, dtype)


@pytest.mark.parametrize("dtype,dh", PATHS, ids=PATH_IDS)
def test_combined_softmax_sums_to_one(dtype, dh):
    """Reference test_kernel.py:61-83: the weights over the causal keys and the token's
    own depth rows sum to one. With every value row (V and V_depth) all ones, the output
    is therefore all ones, whatever Q, K and K_depth are."""
    B, H, T, L, d = 1, 1, 4, 2, dh or 8
    for (B, H, T, L) in [(B, H, T, L), (2, 4, 300, 32)]:
        arrs, args = _inputs(B, H, H, T, L, d, dtype, seed=61)
        args[2] = torch.ones_like(args[2])
        args[4] = torch.ones_like(args[4])
        out = moda_attention_cuda(*args, num_layers=L)
        err = float((out.float() - 1.0).abs().max())
        assert err <= (1e-5 if dtype == torch.float32 else 8e-3), err


@pytest.mark.parametrize("dtype,dh", PATHS, ids=PATH_IDS)
def test_single_head_and_gqa_shapes(dtype, dh):
    """Reference test_kernel.py:121-135 (test_single_head, test_gqa_output_shape) and
    test_gqa.py:11-49 (G = 1, 2, 4)."""
    for (B, Hq, Hk, T, L, d) in [(2, 1, 1, 6, 4, 32), (1, 8, 2, 4, 2, 8), (1, 4, 4, 8, 3, 16),
                                 (1, 4, 2, 6, 2, 8), (2, 8, 2, 4, 3, 16)]:
        d = dh or d
        arrs, args = _inputs(B, Hq, Hk, T, L, d, dtype, seed=62)
        out = moda_attention_cuda(*args, num_layers=L)
        assert tuple(out.shape) == (B, Hq, T, d) and torch.isfinite(out).all()
        _check_vs_oracle(out, arrs, L, dtype)


@pytest.mark.parametrize("dtype,dh", PATHS, ids=PATH_IDS)
def test_large_num_layers(dtype, dh):
    """Reference test_kernel.py:137-143: many depth layers (L = 32), plus L = 64."""
    for (T, L) in [(4, 32), (40, 64)]:
        arrs, args = _inputs(1, 1, 1, T, L, dh or 8, dtype, seed=63)
        out = moda_attention_cuda(*args, num_layers=L)
        assert torch.isfinite(out).all()
        _check_vs_oracle(out, arrs, L, dtype)


@pytest.mark.parametrize("dtype,dh", PATHS, ids=PATH_IDS)
def test_gqa_equals_mha_on_repeated_kv(dtype, dh):
    """Reference test_gqa.py:11-22 and moda_naive.py:51-56: grouped-query attention is
    multi-head attention on K/V heads repeated G times (repeat_interleave)."""
    B, Hq, Hk, T, L, d = 2, 8, 2, 150, 5, dh or 16
    arrs, args = _inputs(B, Hq, Hk, T, L, d, dtype, seed=64)
    G = Hq // Hk
    out = moda_attention_cuda(*args, num_layers=L)
    rep = [t.repeat_interleave(G, dim=1).contiguous() for t in args[1:]]
    out_mha = moda_attention_cuda(args[0], *rep, num_layers=L)
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert float((out.float() - out_mha.float()).abs().max()) <= tol


@pytest.mark.parametrize("dtype,dh", PATHS, ids=PATH_IDS)
def test_gqa_shared_kv_heads(dtype, dh):
    """Reference test_gqa.py:51-69: query heads of one KV group read the same K/V, so two
    equal query heads of a group give equal outputs."""
    B, Hq, Hk, T, L, d = 1, 4, 2, 70, 2, dh or 8
    _, args = _inputs(B, Hq, Hk, T, L, d, dtype, seed=65)
    args[0][:, 1] = args[0][:, 0]
    out = moda_attention_cuda(*args, num_layers=L)
    assert torch.equal(out[:, 0], out[:, 1])


def test_bf16_head_dim_64_runs_the_tensor_core_kernel():
    """The bf16 column of this file runs the tcgen05 kernel (and fp32 the CUDA-core one)."""
    _, args = _inputs(1, 4, 2, 8, 3, 64, torch.bfloat16, seed=66)
    assert moda_plan(*args, 3) == "tc"
    _, args = _inputs(1, 4, 2, 8, 3, 16, torch.float32, seed=66)
    assert moda_plan(*args, 3) == "simt"
