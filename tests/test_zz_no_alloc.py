"""moda_bwd_noalloc: the backward with the library's own fixed scratch (no workspace).

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


def _noalloc(dO, ins, O, lse, L, scale):
    grads = [torch.empty_like(t) for t in ins]
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
    before = torch.cuda.memory_allocated()
    got = _noalloc(dO, ins, O, lse, meta["L"], meta["scale"])
    torch.cuda.synchronize()
    # the five outputs above are the only new device memory; the call itself took none
    assert torch.cuda.memory_allocated() - before == sum(g.numel() * g.element_size() for g in got)
    for g, r, k in zip(got, ref, GRADS):
        assert torch.equal(g, r), k           # same kernels, same inputs: bit-identical
        if dtype == torch.float32:
            assert rel_err(g.double().cpu().numpy(), z[k]) <= FP32_REL_TOL, k


def test_noalloc_rejects_more_rows_than_its_scratch():
    """B*H_q*T > MODA_NOALLOC_ROWS is refused before any descriptor is used or any
    CUDA call is made (the descriptors below point at nothing)."""
    lib = _lib.load()
    rows = _lib.NOALLOC_ROWS // 8 + 1
    big = _lib.describe(256, (8, 1, rows, 64), (rows * 64, rows * 64, 64, 1))
    other = _lib.describe(256, (8, 1, rows, 64), (rows * 64, rows * 64, 64, 1))
    args = [big] + [other] * 6 + [256] + [other] * 5 + [1, 0.0, _lib.MODA_BF16, None]
    assert lib.moda_bwd_noalloc(*args) == _lib.MODA_ERR_UNSUPPORTED
    assert b"query rows" in lib.moda_last_error()
