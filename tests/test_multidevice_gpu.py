"""Two devices driven from one process.

The kernels opt in to their dynamic shared memory once per device (function attributes
are per device), and the status word is read on the device asked for. Each device runs
the fused forward, its backward and the fused depth-write projection, checked against
the oracle; the first device runs again after the second.
"""

import numpy as np
import pytest
import torch

from moda.kernels import device_status, moda_attention_cuda, moda_backward, moda_forward_lse
from moda.kernels.moda_cuda import depth_proj_append
from oracle import moda_oracle as orc
from helpers import BF16_ABS_TOL, max_abs, seeded_inputs

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                       reason="needs two GPUs in this process"),
]


def test_forward_backward_projection_on_two_devices():
    L = 8
    arrs = seeded_inputs(1, 4, 2, 200, 128, L, seed=11)
    r16 = [torch.from_numpy(np.ascontiguousarray(a)).to(torch.bfloat16).double().numpy() for a in arrs]
    ref = orc.moda_attention_naive(*r16, L)
    do = np.random.default_rng(12).standard_normal(arrs[0].shape).astype(np.float32)
    do16 = torch.from_numpy(do).to(torch.bfloat16)
    gref = orc.moda_attention_grads(*r16, L, do16.double().numpy())
    for i in (0, 1, 0):
        dev = torch.device("cuda", i)
        a = [torch.from_numpy(np.ascontiguousarray(x)).to(dev, torch.bfloat16) for x in arrs]
        o = moda_attention_cuda(*a, L).float().cpu().numpy()
        assert max_abs(o, ref) <= BF16_ABS_TOL

        O, lse = moda_forward_lse(*a, L)
        grads = moda_backward(do16.to(dev), *a, O, lse, L)
        for g, k in zip(grads, ("dQ", "dK", "dV", "dK_depth", "dV_depth")):
            err = np.abs(g.float().cpu().numpy() - gref[k]).max() / max(1.0, np.abs(gref[k]).max())
            assert err <= BF16_ABS_TOL, (i, k, err)

        gen = torch.Generator(device=dev).manual_seed(3)
        x = torch.randn(2, 48, 256, device=dev, generator=gen).to(torch.bfloat16)
        w = (torch.randn(2 * 2 * 64, 256, device=dev, generator=gen) / 16).to(torch.bfloat16)
        kc = torch.zeros(2, 2, 48 * 6, 64, device=dev, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        depth_proj_append(x, w, kc, vc, 3, 6, 48)
        y = (x.double() @ w.double().t()).view(2, 48, 2, 2, 64)
        assert float((kc[:, :, 3::6].double() - y[:, :, 0].transpose(1, 2)).abs().max()) <= BF16_ABS_TOL
        assert float((vc[:, :, 3::6].double() - y[:, :, 1].transpose(1, 2)).abs().max()) <= BF16_ABS_TOL
        assert device_status(dev) == 0
