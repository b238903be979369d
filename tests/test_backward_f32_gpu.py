"""The backward in CUDA-core tiles (csrc/moda_bwd_f32.cu) against the oracle.

fp32 inputs with d a multiple of 4 up to 128, G <= 32 and 16-byte aligned rows take the
tiled kernels, and so do bf16 / f16 inputs of the shapes the tensor-core backward does
not take (head_dim outside {64, 128}, H_q / H_k not dividing 128); other layouts take
the row kernels (csrc/moda_bwd.cu). Both are
checked here: shapes across the tile edges (T around 64, head_dim 8 / 36 / 96 / 128, L
over one 32-row depth chunk, G = 1 .. 32, extra depth rows past T*L), the row-kernel
route through misaligned views, and at a medium size (B=1, H_q=32, H_k=8, T=2048,
d=128, L=32) the exact per-token gradients of sampled tokens plus two identities of the
full gradients per KV head: sum of dV over all key rows (sequence and depth) equals sum
of dO over the head group's query rows (each softmax row sums to one), and the sum of
dK over all key rows is zero (each row of dS sums to zero).
Tolerance: max|g - ref| / max|ref| <= 1e-4 for every gradient (FP32_REL_TOL); 16-bit
inputs against the fp64 oracle on the same rounded inputs: 3e-2 of max(1, max|ref|).
"""

import numpy as np
import pytest
import torch

from moda.kernels import device_status, moda_attention_cuda, moda_backward, moda_forward_lse
from oracle import moda_oracle as orc
from helpers import FP32_REL_TOL, rel_err, seeded_inputs

pytestmark = pytest.mark.gpu
GRADS = ("dQ", "dK", "dV", "dK_depth", "dV_depth")

# (B, H_q, H_k, T, d, L, extra depth rows)
CASES = [
    (1, 4, 2, 64, 64, 3, 0),      # one exact tile
    (2, 4, 4, 65, 128, 5, 0),     # ragged second tile, G = 1
    (1, 8, 2, 130, 32, 1, 0),     # head_dim 32, L = 1
    (1, 2, 1, 1, 128, 2, 0),      # one token
    (1, 32, 1, 70, 64, 4, 0),     # G = 32, the largest tiled group
    (2, 6, 2, 100, 96, 33, 0),    # head_dim 96, two depth chunks
    (1, 4, 2, 50, 36, 40, 0),     # head_dim 36: a partial column group
    (1, 4, 2, 90, 8, 3, 0),       # head_dim 8
    (1, 4, 2, 77, 64, 6, 11),     # depth rows past T*L get zero gradient
    (1, 3, 3, 129, 128, 32, 0),   # three query tiles, L = 32
    (1, 64, 1, 20, 32, 2, 0),     # G = 64: the row kernels
]


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert device_status() == 0, "a bounded device wait expired"


def _grads(args, L, dO):
    ins = [a.clone().requires_grad_(True) for a in args]
    moda_attention_cuda(*ins, L).backward(dO)
    return [t.grad.double().cpu().numpy() for t in ins]


@pytest.mark.parametrize("case", CASES, ids=["-".join(map(str, c)) for c in CASES])
def test_fp32_grads_match_oracle(case):
    B, Hq, Hk, T, d, L, extra = case
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=300 + T + d, extra_rows=extra)
    args = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]
    dO = np.random.default_rng(T * d).standard_normal((B, Hq, T, d)).astype(np.float32)
    got = _grads(args, L, torch.from_numpy(dO).cuda())
    ref = orc.moda_attention_grads(*[a.astype(np.float64) for a in arrs], L, dO.astype(np.float64))
    for k, g in zip(GRADS, got):
        assert g.shape == ref[k].shape, k
        assert rel_err(g, ref[k]) <= FP32_REL_TOL, (k, rel_err(g, ref[k]))
    if extra:
        assert not np.any(got[3][:, :, T * L:]) and not np.any(got[4][:, :, T * L:])


def test_row_kernel_route_agrees_with_tiled_route():
    # the same values in views whose rows start 4 bytes past a 16-byte boundary: the
    # tiled kernels refuse them and the row kernels run
    B, Hq, Hk, T, d, L = 1, 8, 2, 96, 64, 5
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=77)
    dense = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in arrs]

    bufs = []
    for t in dense:
        buf = torch.zeros(*t.shape[:-1], t.shape[-1] + 1, device="cuda")
        buf[..., 1:] = t
        bufs.append(buf.requires_grad_(True))
    views = [buf[..., 1:] for buf in bufs]  # the leaves are the padded buffers
    assert views[0].data_ptr() % 16 != 0 and views[0].stride(2) == d + 1
    dO = torch.from_numpy(np.random.default_rng(5).standard_normal((B, Hq, T, d)).astype(np.float32)).cuda()
    tiled = _grads(dense, L, dO)
    moda_attention_cuda(*views, L).backward(dO)
    rows = [buf.grad[..., 1:].double().cpu().numpy() for buf in bufs]
    ref = orc.moda_attention_grads(*[a.astype(np.float64) for a in arrs], L, dO.double().cpu().numpy())
    for k, a, b in zip(GRADS, tiled, rows):
        assert rel_err(a, ref[k]) <= FP32_REL_TOL and rel_err(b, ref[k]) <= FP32_REL_TOL, k
        assert rel_err(a, b) <= 1e-5, k


def test_fp32_medium_shape_tokens_and_identities():
    B, Hq, Hk, T, d, L = 1, 32, 8, 2048, 128, 32
    G = Hq // Hk
    g = torch.Generator(device="cuda").manual_seed(11)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g, dtype=torch.float32)
    Q, K, V, dO = mk(B, Hq, T, d), mk(B, Hk, T, d), mk(B, Hk, T, d), mk(B, Hq, T, d)
    Kd, Vd = mk(B, Hk, T * L, d), mk(B, Hk, T * L, d)
    O, lse = moda_forward_lse(Q, K, V, Kd, Vd, L)
    dQ, dK, dV, dKd, dVd = moda_backward(dO, Q, K, V, Kd, Vd, O, lse, L)
    torch.cuda.synchronize()
    h = lambda x: x.double().cpu().numpy()
    rng = np.random.default_rng(4)
    picks = [(0, 0), (Hk - 1, T - 1), (3, 1023), (5, 64)]
    picks += [(int(rng.integers(Hk)), int(rng.integers(T))) for _ in range(6)]
    for hk, t in picks:
        heads = slice(hk * G, (hk + 1) * G)
        rows = slice(t * L, (t + 1) * L)
        ref = orc.moda_token_grads(h(Q[0, heads, t]), h(dO[0, heads, t]), h(K[0, hk, :t + 1]),
                                   h(V[0, hk, :t + 1]), h(Kd[0, hk, rows]), h(Vd[0, hk, rows]), d ** -0.5)
        assert rel_err(h(dQ[0, heads, t]), ref["dQ"]) <= FP32_REL_TOL, ("dQ", hk, t)
        assert rel_err(h(dKd[0, hk, rows]), ref["dK_depth"]) <= FP32_REL_TOL, ("dK_depth", hk, t)
        assert rel_err(h(dVd[0, hk, rows]), ref["dV_depth"]) <= FP32_REL_TOL, ("dV_depth", hk, t)
    # the last key is read by the last token's G rows only: its dK and dV from their
    # full softmax rows (keys 0..T-1 and the token's depth rows), in fp64
    for hk in (0, Hk - 1):
        keys = np.concatenate([h(K[0, hk]), h(Kd[0, hk, (T - 1) * L:T * L])])
        vals = np.concatenate([h(V[0, hk]), h(Vd[0, hk, (T - 1) * L:T * L])])
        dk_ref, dv_ref = np.zeros(d), np.zeros(d)
        for q, do in zip(h(Q[0, hk * G:(hk + 1) * G, T - 1]), h(dO[0, hk * G:(hk + 1) * G, T - 1])):
            s = keys @ q * d ** -0.5
            w = np.exp(s - s.max())
            w /= w.sum()
            ds = w * (vals @ do - do @ (w @ vals))
            dk_ref += d ** -0.5 * ds[T - 1] * q
            dv_ref += w[T - 1] * do
        assert rel_err(h(dK[0, hk, T - 1]), dk_ref) <= FP32_REL_TOL, hk
        assert rel_err(h(dV[0, hk, T - 1]), dv_ref) <= FP32_REL_TOL, hk
    # per KV head: sum of dV over its key rows = sum of dO over its query rows; sum of dK = 0
    sum_dv = h(dV.sum(2)) + h(dVd.sum(2))                        # [B, Hk, d]
    sum_do = h(dO.reshape(B, Hk, G, T, d).sum((2, 3)))
    assert np.max(np.abs(sum_dv - sum_do)) <= 1e-4 * np.max(np.abs(sum_do)) + 1e-3
    sum_dk = h(dK.sum(2)) + h(dKd.sum(2))
    assert np.max(np.abs(sum_dk)) <= 1e-4 * float(h(dK.abs().sum(2)).max())


# 16-bit shapes the tensor-core backward does not take: (B, H_q, H_k, T, d, L, extra)
HALF_CASES = [
    (1, 6, 2, 70, 64, 3, 0),      # G = 3
    (1, 10, 2, 129, 128, 5, 0),   # G = 5, head_dim 128
    (2, 4, 2, 65, 32, 4, 0),      # head_dim 32
    (1, 6, 2, 100, 96, 33, 9),    # head_dim 96, G = 3, two depth chunks, extra depth rows
    (1, 4, 4, 50, 36, 2, 0),      # head_dim 36 (a partial 8-element copy per row)
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("case", HALF_CASES, ids=["-".join(map(str, c)) for c in HALF_CASES])
def test_half_grads_in_tiles_match_oracle(case, dtype):
    B, Hq, Hk, T, d, L, extra = case
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=500 + T + d, extra_rows=extra)
    args = [torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype) for a in arrs]
    rin = [t.double().cpu().numpy() for t in args]
    dO = torch.from_numpy(np.random.default_rng(T + d).standard_normal((B, Hq, T, d))).to("cuda", dtype)
    got = _grads(args, L, dO)
    ref = orc.moda_attention_grads(*rin, L, dO.double().cpu().numpy())
    for k, g in zip(GRADS, got):
        assert g.shape == ref[k].shape, k
        e = float(np.abs(g - ref[k]).max()) / max(1.0, float(np.abs(ref[k]).max()))
        assert e <= 3e-2, (k, e)
    if extra:
        assert not np.any(got[3][:, :, T * L:]) and not np.any(got[4][:, :, T * L:])
