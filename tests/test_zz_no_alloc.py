"""moda_bwd_noalloc: the backward with the library's own fixed scratch (no workspace).

Some callers cannot allocate device memory when they call the backward: a caller that
runs inside a memory pool it does not own, one that has reserved all device memory up
front, or one that must not call into the allocator from its call site. This entry
point gives them the backward without a workspace argument; its rowsum(dO*O) scratch
is an array compiled into the library.

Collected last on purpose: it must pass on its own and after every other test
(the fixed scratch array is shared by all calls on a device).
"""

import numpy as np
import pytest
import torch

from moda.kernels import _lib
from moda.kernels.moda_cuda import _DTYPES, _desc, moda_backward, moda_forward_lse
from helpers import FP32_REL_TOL, golden_cases, rel_err

NAMES = ("Q", "K", "V", "K_depth", "V_depth")
GRADS = ("dQ", "dK", "dV", "dK_depth", "dV_depth")


def _noalloc_into(grads, dO, ins, O, lse, L, scale):
    code = _lib.load().moda_bwd_noalloc(*[_desc(t) for t in ins], _desc(O), _desc(dO),
                                        lse.data_ptr(), *[_desc(g) for g in grads], int(L),
                                        float(scale) if scale else 0.0, _DTYPES[ins[0].dtype],
                                        torch.cuda.current_stream().cuda_stream)
    _lib.check(code, "moda_bwd_noalloc")
    return grads


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_noalloc_backward_equals_workspace_backward(dtype):
    name, z, meta = golden_cases("grad")[0]
    ins = [torch.from_numpy(z[k]).to("cuda", dtype) for k in NAMES]
    dO = torch.from_numpy(z["dO"]).to("cuda", dtype)
    O, lse = moda_forward_lse(*ins, meta["L"], meta["scale"])
    ref = moda_backward(dO, *ins, O, lse, meta["L"], meta["scale"])
    grads = [torch.full_like(t, float("nan")) for t in ins]
    torch.cuda.synchronize()
    # two calls in a row: the second sees the scratch the first left behind
    for _ in range(2):
        before = torch.cuda.memory_allocated()
        got = _noalloc_into(grads, dO, ins, O, lse, meta["L"], meta["scale"])
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before  # the call allocated nothing
        for g, r, k in zip(got, ref, GRADS):
            assert torch.equal(g, r), k           # same kernels, same inputs: bit-identical
            if dtype == torch.float32:
                assert rel_err(g.double().cpu().numpy(), z[k]) <= FP32_REL_TOL, k


@pytest.mark.gpu
def test_noalloc_zero_rows():
    """T = 0: no query rows, no scratch needed; the call succeeds and launches nothing."""
    dev = torch.device("cuda")
    q = torch.empty(1, 4, 0, 64, device=dev, dtype=torch.bfloat16)
    kv = torch.empty(1, 2, 0, 64, device=dev, dtype=torch.bfloat16)
    ins = [q, kv, kv.clone(), kv.clone(), kv.clone()]
    lse = torch.empty(1, 4, 0, device=dev, dtype=torch.float32)
    grads = [torch.empty_like(t) for t in ins]
    _noalloc_into(grads, q.clone(), ins, q.clone(), lse, 4, None)
    torch.cuda.synchronize()


BAD_DTYPE = 99  # refused by the host-side validation, so nothing can ever launch


def _host_only_args(sizes_q):
    """Descriptors that point at nothing and an unknown dtype code: valid only for
    checks made on the host; a call that gets past the size check stops at the dtype
    check, before any launch."""
    strides = (sizes_q[1] * sizes_q[2] * 64, sizes_q[2] * 64, 64, 1)
    big = _lib.describe(256, sizes_q, strides)
    other = _lib.describe(256, (sizes_q[0], 1, sizes_q[2], 64), strides)
    return [big] + [other] * 6 + [256] + [other] * 5 + [1, 0.0, BAD_DTYPE, None]


def test_noalloc_rejects_more_rows_than_its_scratch():
    """B*H_q*T > MODA_NOALLOC_ROWS is refused before any descriptor is used or any
    CUDA call is made."""
    lib = _lib.load()
    rows = _lib.NOALLOC_ROWS // 8 + 1
    assert lib.moda_bwd_noalloc(*_host_only_args((8, 1, rows, 64))) == _lib.MODA_ERR_UNSUPPORTED
    assert b"query rows" in lib.moda_last_error()


@pytest.mark.parametrize("sizes", [(1 << 31, 1 << 31, 1 << 31, 64), (1 << 62, 4, 4, 64),
                                   (3, 1 << 21, 1, 64)])
def test_noalloc_rejects_sizes_whose_product_overflows(sizes):
    """Sizes whose product overflows int64 (or wraps below the limit) are refused by the
    size check itself."""
    lib = _lib.load()
    assert lib.moda_bwd_noalloc(*_host_only_args(sizes)) == _lib.MODA_ERR_UNSUPPORTED
    assert b"query rows" in lib.moda_last_error()


def test_noalloc_accepts_exactly_its_scratch_size():
    """B*H_q*T == MODA_NOALLOC_ROWS passes the size check: the call then stops at a
    later host-side check (no GPU here: resolving the scratch; with one: the dtype),
    not at the size refusal."""
    lib = _lib.load()
    code = lib.moda_bwd_noalloc(*_host_only_args((8, 1, _lib.NOALLOC_ROWS // 8, 64)))
    assert code != _lib.MODA_ERR_UNSUPPORTED
    assert b"query rows" not in lib.moda_last_error()
