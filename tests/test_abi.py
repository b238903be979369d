"""C-ABI library: loads, exports what include/moda_b200.h declares, validates and
plans on the host. No kernel launches (these run without a GPU)."""

import os
import re

import pytest
import torch

from moda.kernels import _lib
from moda.kernels.moda_cuda import moda_plan

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "moda_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(moda_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    assert declared_functions() == sorted(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.moda_version() == 200
    assert lib.moda_last_error() == b""


def _t(shape, dtype=torch.bfloat16, strides=None):
    x = torch.empty(shape, dtype=dtype)
    return x if strides is None else x.as_strided(shape, strides)


def _plan(B, Hq, Hk, T, d, L, dtype=torch.bfloat16, extra=0, kernel="auto", q=None):
    Q = q if q is not None else _t((B, Hq, T, d), dtype)
    K, V = _t((B, Hk, T, d), dtype), _t((B, Hk, T, d), dtype)
    Kd, Vd = _t((B, Hk, T * L + extra, d), dtype), _t((B, Hk, T * L + extra, d), dtype)
    return moda_plan(Q, K, V, Kd, Vd, L, kernel=kernel)


@pytest.mark.parametrize("d,dtype,expect", [
    (128, torch.bfloat16, "tc"), (64, torch.bfloat16, "tc"), (64, torch.float16, "tc"),
    (128, torch.float32, "simt"), (32, torch.bfloat16, "simt"), (256, torch.bfloat16, "simt"),
])
def test_plan_by_dtype_and_head_dim(d, dtype, expect):
    assert _plan(1, 8, 2, 100, d, 4, dtype) == expect


# groups that do not divide 128 (3, 6, 12) run the tensor-core kernel as G launches with
# one query head per KV head; above 128 heads per group, the CUDA-core kernel
@pytest.mark.parametrize("G,expect", [(1, "tc"), (2, "tc"), (4, "tc"), (8, "tc"), (16, "tc"),
                                      (3, "tc"), (6, "tc"), (12, "tc"), (160, "simt")])
def test_plan_by_group_size(G, expect):
    assert _plan(1, 2 * G, 2, 64, 128, 2) == expect


def test_plan_strided_views_like_moda_attention():
    # MoDAAttention passes q_proj(x).view(B,T,H,d).transpose(1,2): strides (T*H*d, d, H*d, 1)
    B, T, H, d = 2, 40, 8, 64
    q = torch.empty(B, T, H, d, dtype=torch.bfloat16).transpose(1, 2)
    assert _plan(B, H, 4, T, d, 3, q=q) == "tc"
    # an innermost stride != 1 can only run on the CUDA-core kernel
    q2 = torch.empty(B, H, d, T, dtype=torch.bfloat16).transpose(2, 3)
    assert _plan(B, H, 4, T, d, 3, q=q2) == "simt"
    with pytest.raises(RuntimeError):
        _plan(B, H, 4, T, d, 3, q=q2, kernel="tc")


def test_plan_oversize_depth_buffer_is_accepted():
    assert _plan(1, 4, 2, 20, 64, 4, extra=16) == "tc"


def test_short_depth_buffer_is_rejected_before_launch():
    # D1: K_depth with 5 layers of rows but num_layers=6 (reference raises RuntimeError)
    B, H, Hk, T, d = 1, 8, 4, 64, 64
    Q = _t((B, H, T, d)); K = _t((B, Hk, T, d)); V = _t((B, Hk, T, d))
    Kd = _t((B, Hk, T * 5, d)); Vd = _t((B, Hk, T * 5, d))
    with pytest.raises(RuntimeError, match="rows"):
        moda_plan(Q, K, V, Kd, Vd, 6)
    with pytest.raises(ValueError):
        moda_plan(Q, K, V, Kd, Vd, 6)


@pytest.mark.parametrize("bad", ["heads", "head_dim", "batch", "kv_len"])
def test_shape_mismatches_raise(bad):
    B, Hq, Hk, T, d, L = 2, 8, 4, 16, 64, 2
    shapes = dict(Q=(B, Hq, T, d), K=(B, Hk, T, d), V=(B, Hk, T, d), Kd=(B, Hk, T * L, d))
    if bad == "heads":
        shapes["K"] = (B, 3, T, d)
    elif bad == "head_dim":
        shapes["V"] = (B, Hk, T, 32)
    elif bad == "batch":
        shapes["Kd"] = (1, Hk, T * L, d)
    else:
        shapes["K"] = (B, Hk, T + 1, d)
    with pytest.raises(_lib.MoDAShapeError):
        moda_plan(_t(shapes["Q"]), _t(shapes["K"]), _t(shapes["V"]), _t(shapes["Kd"]),
                  _t((B, Hk, T * L, d)), L)


def test_dtype_errors_are_type_and_runtime_errors():
    # torch raises RuntimeError inside moda_attention_naive for mixed dtypes; the drop-in's
    # dtype errors are both TypeError and RuntimeError, from the host checks and from the
    # C ABI's status code alike
    x = _t((1, 2, 8, 64))
    x64 = torch.zeros(1, 2, 8, 64, dtype=torch.float64)
    with pytest.raises(TypeError):
        moda_plan(x64, x64, x64, x64, x64, 1)
    with pytest.raises(RuntimeError):
        moda_plan(x64, x64, x64, x64, x64, 1)
    with pytest.raises(_lib.MoDADtypeError):
        _lib.check(_lib.MODA_ERR_DTYPE, "moda_fwd")
    assert issubclass(_lib.MoDADtypeError, TypeError) and issubclass(_lib.MoDADtypeError, RuntimeError)
    assert moda_plan(x, x, x, x, x, 1) in ("tc", "simt")


def test_negative_num_layers_rejected():
    x = _t((1, 2, 8, 64))
    with pytest.raises(ValueError):
        moda_plan(x, x, x, x, x, -1)


def test_cpu_tensors_are_refused_by_the_kernel_entry():
    from moda.kernels import moda_attention_cuda
    x = torch.zeros(1, 2, 4, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        moda_attention_cuda(x, x, x, torch.zeros(1, 2, 8, 16), torch.zeros(1, 2, 8, 16), 2)


def _bwd_args(B=1, Hq=4, Hk=2, T=8, d=16, L=2, R=None, dq_shape=None, work=1 << 20):
    """moda_bwd arguments over host tensors. Every call below fails validation, so
    nothing is launched (and no host pointer ever reaches a kernel)."""
    R = T * L if R is None else R
    Q, O, dO = _t((B, Hq, T, d)), _t((B, Hq, T, d)), _t((B, Hq, T, d))
    K, V = _t((B, Hk, T, d)), _t((B, Hk, T, d))
    Kd, Vd = _t((B, Hk, R, d)), _t((B, Hk, R, d))
    dQ = _t(dq_shape or (B, Hq, T, d))
    dK, dV, dKd, dVd = _t((B, Hk, T, d)), _t((B, Hk, T, d)), _t((B, Hk, R, d)), _t((B, Hk, R, d))
    lse = torch.empty(B, Hq, T)
    ws = torch.empty(work, dtype=torch.uint8)
    keep = (Q, O, dO, K, V, Kd, Vd, dQ, dK, dV, dKd, dVd, lse, ws)
    D = lambda x: _lib.describe(x.data_ptr(), x.shape, x.stride())
    args = [D(Q), D(K), D(V), D(Kd), D(Vd), D(O), D(dO), lse.data_ptr(), D(dQ), D(dK), D(dV),
            D(dKd), D(dVd), ws.data_ptr(), work, L, 0.0, _lib.MODA_BF16, None]
    return args, keep


def test_bwd_workspace_size():
    lib = _lib.load()
    assert lib.moda_bwd_workspace_size(2, 8, 100) == 2 * 8 * 100 * 4
    assert lib.moda_bwd_workspace_size(-1, 8, 100) == -1


@pytest.mark.parametrize("case", ["dq_shape", "short_depth", "small_workspace", "null_lse"])
def test_bwd_rejects_bad_arguments_before_launch(case):
    lib = _lib.load()
    if case == "dq_shape":
        args, keep = _bwd_args(dq_shape=(1, 4, 7, 16))
        expect = _lib.MODA_ERR_SHAPE
    elif case == "short_depth":
        args, keep = _bwd_args(R=10)
        expect = _lib.MODA_ERR_DEPTH_ROWS
    elif case == "small_workspace":
        args, keep = _bwd_args(work=4 * 4 * 8 - 4)
        expect = _lib.MODA_ERR_ARG
    else:
        args, keep = _bwd_args()
        args[7] = None
        expect = _lib.MODA_ERR_ARG
    assert lib.moda_bwd(*args) == expect
    assert lib.moda_last_error() != b""


@pytest.mark.parametrize("case", ["negative_rows", "k_heads", "o_shape"])
def test_zero_depth_rejects_bad_arguments_before_launch(case):
    lib = _lib.load()
    B, Hq, Hk, T, d = 1, 4, 2, 8, 64
    Q, O = _t((B, Hq, T, d)), _t((B, Hq, T, d) if case != "o_shape" else (B, Hq, T + 1, d))
    K, V = _t((B, Hk, T, d)), _t((B, Hk if case != "k_heads" else 3, T, d))
    D = lambda x: _lib.describe(x.data_ptr(), x.shape, x.stride())
    lse = torch.empty(B, Hq, T)
    rows = -1 if case == "negative_rows" else 4
    code = lib.moda_fwd_zero_depth(D(Q), D(K), D(V), D(O), lse.data_ptr(), rows, 0.0,
                                   _lib.MODA_BF16, _lib.KERNEL_AUTO, None)
    assert code == (_lib.MODA_ERR_ARG if case == "negative_rows" else _lib.MODA_ERR_SHAPE)
    assert lib.moda_last_error() != b""


@pytest.mark.parametrize("case", ["fp32", "w_rows", "short_cache", "slot"])
def test_depth_projection_rejects_before_launch(case):
    lib = _lib.load()
    dt = torch.float32 if case == "fp32" else torch.bfloat16
    B, T, D, Hk, d, L = 1, 8, 64, 2, 32, 3
    x = _t((B, 1, T, D), dt)
    w = _t((1, 1, 2 * Hk * d + (8 if case == "w_rows" else 0), D), dt)
    R = T * L - (1 if case == "short_cache" else 0)
    kc, vc = _t((B, Hk, R, d), dt), _t((B, Hk, R, d), dt)
    D_ = lambda t: _lib.describe(t.data_ptr(), t.shape, t.stride())
    code = lib.moda_depth_proj_append(D_(x), D_(w), D_(kc), D_(vc), L if case == "slot" else 1,
                                      L, T, _lib.MODA_F32 if case == "fp32" else _lib.MODA_BF16,
                                      None)
    expect = {"fp32": _lib.MODA_ERR_UNSUPPORTED, "w_rows": _lib.MODA_ERR_SHAPE,
              "short_cache": _lib.MODA_ERR_DEPTH_ROWS, "slot": _lib.MODA_ERR_ARG}[case]
    assert code == expect
    assert lib.moda_last_error() != b""


@pytest.mark.parametrize("case", ["w_rows", "kv_heads", "dtype", "x_heads"])
def test_qkv_projection_rejects_before_launch(case):
    """Shape and dtype errors of moda_qkv_proj are found on the host (no launch: the
    descriptors point at nothing)."""
    lib = _lib.load()
    B, T, D, Hq, Hk, d = 2, 16, 64, 4, 2, 32
    x = _lib.describe(256, (B, 1 if case != "x_heads" else 2, T, D), (T * D, T * D, D, 1))
    n = (Hq + 2 * Hk) * d + (32 if case == "w_rows" else 0)
    w = _lib.describe(256, (1, 1, n, D), (n * D, n * D, D, 1))
    q = _lib.describe(256, (B, Hq, T, d), (Hq * T * d, T * d, d, 1))
    hk_v = Hk + 1 if case == "kv_heads" else Hk
    k = _lib.describe(256, (B, Hk, T, d), (Hk * T * d, T * d, d, 1))
    v = _lib.describe(256, (B, hk_v, T, d), (hk_v * T * d, T * d, d, 1))
    dtype = 99 if case == "dtype" else _lib.MODA_BF16
    code = lib.moda_qkv_proj(x, w, q, k, v, dtype, None)
    assert code == (_lib.MODA_ERR_DTYPE if case == "dtype" else _lib.MODA_ERR_SHAPE)
