"""Parity of the CUDA forward (libmoda_b200.so via its C ABI) with the oracle.

Tolerances:
  fp32 kernel vs fp32 reference: max|o - ref| / max|ref| <= 1e-4   (FP32_REL_TOL)
  bf16/f16 kernel vs fp64 oracle on the same rounded inputs: max|o - ref| <= 2e-2 (BF16_ABS_TOL)
"""

import numpy as np
import pytest
import torch

from moda.kernels import moda_attention_cuda, device_status, moda_plan
from oracle import moda_oracle as orc
from helpers import (BF16_ABS_TOL, FP32_REL_TOL, golden_cases, max_abs, rel_err,
                     seeded_inputs)

pytestmark = pytest.mark.gpu
KERNEL_CASES = golden_cases("kernel")


def dev(arrs, dtype):
    return [torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype) for a in arrs]


def rounded(arrs, dtype):
    """The inputs exactly as the kernel sees them, back in float64."""
    return [torch.from_numpy(np.ascontiguousarray(a)).to(dtype).double().numpy() for a in arrs]


def run(args, L, scale=None, chunk=None, kernel="auto"):
    out = moda_attention_cuda(*args, L, scale, chunk, kernel=kernel)
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert device_status() == 0, "a bounded device wait expired"


# ------------------------------------------------------------------ golden vectors
@pytest.mark.parametrize("name,z,meta", KERNEL_CASES, ids=[c[0] for c in KERNEL_CASES])
def test_golden_fp32(name, z, meta):
    arrs = [z[k] for k in ("Q", "K", "V", "K_depth", "V_depth")]
    out = run(dev(arrs, torch.float32), meta["L"], meta["scale"])
    ref_key = "out_full" if "out_full" in z.files else \
        [k for k in z.files if k.startswith("out_")][0]
    assert rel_err(out, z[ref_key]) <= FP32_REL_TOL, rel_err(out, z[ref_key])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("name,z,meta", KERNEL_CASES, ids=[c[0] for c in KERNEL_CASES])
def test_golden_half(name, z, meta, dtype):
    arrs = [z[k] for k in ("Q", "K", "V", "K_depth", "V_depth")]
    ref = orc.moda_attention_naive(*rounded(arrs, dtype), meta["L"], meta["scale"],
                                   chunk_size=meta["T"])
    for kernel in ("auto", "simt"):
        out = run(dev(arrs, dtype), meta["L"], meta["scale"], kernel=kernel)
        assert max_abs(out, ref) <= BF16_ABS_TOL, (kernel, max_abs(out, ref))


def test_golden_c1_runs_the_tensor_core_kernel_in_bf16():
    z = dict(np.load(__import__("helpers").GOLDEN + "/c1_b1_h4x2_t32_d64_l8.npz"))
    args = dev([z[k] for k in ("Q", "K", "V", "K_depth", "V_depth")], torch.bfloat16)
    assert moda_plan(*args, 8) == "tc"


# ------------------------------------------------------------------ seeded sweeps vs oracle
SHAPES = [
    # B, H_q, H_k, T, d, L
    (1, 4, 2, 32, 64, 8),
    (2, 8, 2, 300, 128, 32),
    (1, 4, 4, 129, 64, 1),
    (1, 16, 2, 257, 64, 48),
    (2, 4, 1, 1000, 128, 5),
    (1, 32, 8, 200, 128, 32),
    (1, 2, 2, 1, 128, 3),
    (1, 2, 1, 127, 64, 2),
    (1, 2, 1, 128, 64, 2),
    (1, 2, 2, 256, 128, 24),
    (1, 64, 8, 70, 128, 48),
    (1, 8, 8, 90, 64, 12),
    (1, 128, 1, 40, 64, 3),
    # L a multiple of 16 (or 32): depth windows are whole 16-column groups
    (1, 8, 2, 90, 128, 16),
    (2, 16, 2, 77, 64, 48),
    (1, 16, 2, 150, 64, 64),
    (1, 2, 2, 70, 128, 32),
    (1, 4, 2, 45, 64, 96),
    (1, 32, 2, 50, 128, 32),
    (1, 32, 1, 20, 64, 32),
    # L a multiple of 8 but not of 16: 8-column depth groups (windows straddle blocks)
    (1, 16, 4, 300, 128, 24),
    (2, 8, 2, 133, 64, 40),
    (1, 4, 4, 70, 128, 8),
    (1, 64, 8, 45, 64, 56),
]


EMPTY = [(2, 4, 2, 0, 128, 3), (0, 4, 2, 5, 128, 3), (2, 8, 2, 0, 64, 32)]


@pytest.mark.parametrize("shape", EMPTY, ids=[str(s) for s in EMPTY])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
@pytest.mark.parametrize("chunk", [None, 4])
def test_empty_inputs_give_empty_output(shape, dtype, chunk):
    """The reference returns an empty O of Q's shape for T = 0 or B = 0 (oracle too)."""
    B, Hq, Hk, T, d, L = shape
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=11)
    out = moda_attention_cuda(*dev(arrs, dtype), L, None, chunk)
    torch.cuda.synchronize()
    ref = orc.moda_attention_naive(*arrs, L, chunk_size=chunk)
    assert tuple(out.shape) == ref.shape == (B, Hq, T, d) and out.dtype == dtype


@pytest.mark.parametrize("shape", SHAPES, ids=[str(s) for s in SHAPES])
def test_tc_matches_oracle_bf16(shape):
    B, Hq, Hk, T, d, L = shape
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=hash(shape) % 1000)
    args = dev(arrs, torch.bfloat16)
    assert moda_plan(*args, L) == "tc"
    ref = orc.moda_attention_naive(*rounded(arrs, torch.bfloat16), L, chunk_size=64)
    out = run(args, L, kernel="tc")
    assert max_abs(out, ref) <= BF16_ABS_TOL, max_abs(out, ref)


@pytest.mark.parametrize("shape", [(1, 4, 2, 77, 64, 3), (2, 6, 3, 40, 32, 5), (1, 2, 1, 50, 256, 2),
                                   (1, 3, 1, 33, 16, 32)])
def test_simt_fp32_matches_oracle(shape):
    B, Hq, Hk, T, d, L = shape
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=11)
    ref = orc.moda_attention_naive(*arrs, L, chunk_size=16)
    out = run(dev(arrs, torch.float32), L)
    assert rel_err(out, ref) <= FP32_REL_TOL


# ------------------------------------------------------------------ relational properties
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_causal_invariance(dtype):
    # reference tests/test_kernel.py:32-44: a later key never changes an earlier row
    args = dev(seeded_inputs(1, 4, 2, 200, 64, 4, seed=3), dtype)
    out = moda_attention_cuda(*args, 4)
    K2 = args[1].clone()
    K2[:, :, 150] = 999.0
    out2 = moda_attention_cuda(args[0], K2, *args[2:], 4)
    assert torch.equal(out[:, :, :150], out2[:, :, :150])
    assert not torch.equal(out[:, :, 150:], out2[:, :, 150:])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_depth_isolation(dtype):
    # reference tests/test_kernel.py:46-59: token t reads only depth rows [t*L, (t+1)*L)
    L = 3
    args = dev(seeded_inputs(1, 4, 2, 100, 64, L, seed=4), dtype)
    out = moda_attention_cuda(*args, L)
    Kd2 = args[3].clone()
    Kd2[:, :, 40 * L:41 * L] = 999.0
    out2 = moda_attention_cuda(*args[:3], Kd2, args[4], L)
    changed = (out != out2).any(dim=-1).any(dim=0).any(dim=0)
    assert changed.nonzero().flatten().tolist() == [40]


def test_gqa_heads_share_kv():
    # reference tests/test_gqa.py:51-69
    args = dev(seeded_inputs(1, 8, 2, 64, 128, 4, seed=5), torch.bfloat16)
    Q = args[0].clone()
    Q[:, 1] = Q[:, 0]
    out = moda_attention_cuda(Q, *args[1:], 4)
    assert torch.equal(out[:, 0], out[:, 1])


@pytest.mark.parametrize("kernel", ["auto", "simt"])
def test_chunk_size_does_not_change_the_result(kernel):
    args = dev(seeded_inputs(1, 4, 2, 150, 64, 6, seed=6), torch.bfloat16)
    base = moda_attention_cuda(*args, 6, kernel=kernel)
    for C in (None, 1, 7, 64, 128, 4096):
        assert torch.equal(moda_attention_cuda(*args, 6, chunk_size=C, kernel=kernel), base)


def test_deterministic():
    args = dev(seeded_inputs(2, 8, 2, 333, 128, 32, seed=7), torch.bfloat16)
    a = moda_attention_cuda(*args, 32)
    assert all(torch.equal(a, moda_attention_cuda(*args, 32)) for _ in range(3))


def test_no_depth_is_causal_attention():
    B, Hq, Hk, T, d = 1, 8, 2, 200, 128
    arrs = seeded_inputs(B, Hq, Hk, T, d, 0, seed=8)
    args = dev(arrs, torch.bfloat16)
    ref = orc.moda_attention_naive(*rounded(arrs, torch.bfloat16), 0)
    assert max_abs(run(args, 0), ref) <= BF16_ABS_TOL


def test_strided_views_and_oversize_depth():
    # the layouts MoDAAttention and DepthKVCache.read() hand over (moda/attention.py:77-79,
    # moda/cache.py:85-88): transposed projections and a prefix view of a larger cache
    B, T, Hq, Hk, d, L, maxT = 2, 96, 8, 4, 64, 5, 130
    g = torch.Generator(device="cuda").manual_seed(9)
    Q = torch.randn(B, T, Hq, d, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)
    K = torch.randn(B, T, Hk, d, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)
    V = torch.randn(B, T, Hk, d, device="cuda", generator=g).to(torch.bfloat16).transpose(1, 2)
    kc = torch.randn(B, Hk, maxT * L, d, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(B, Hk, maxT * L, d, device="cuda", generator=g).to(torch.bfloat16)
    Kd, Vd = kc[:, :, :T * L], vc[:, :, :T * L]
    assert not Q.is_contiguous() and not Kd.is_contiguous()
    assert moda_plan(Q, K, V, Kd, Vd, L) == "tc"
    out = moda_attention_cuda(Q, K, V, Kd, Vd, L)
    # the whole cache (rows beyond T*L ignored) gives the same answer
    assert torch.equal(out, moda_attention_cuda(Q, K, V, kc, vc, L))
    ref = orc.moda_attention_naive(*[t.double().cpu().numpy() for t in (Q, K, V, Kd, Vd)], L)
    assert max_abs(out.float().cpu().numpy(), ref) <= BF16_ABS_TOL
    out_c = moda_attention_cuda(Q.contiguous(), K.contiguous(), V.contiguous(),
                                Kd.contiguous(), Vd.contiguous(), L)
    assert torch.equal(out, out_c)


def test_write_into_strided_output():
    from moda.kernels.moda_cuda import moda_forward_into
    arrs = seeded_inputs(1, 4, 2, 64, 64, 2, seed=10)
    args = dev(arrs, torch.bfloat16)
    ref = orc.moda_attention_naive(*rounded(arrs, torch.bfloat16), 2)
    O = torch.zeros(1, 64, 4, 64, dtype=torch.bfloat16, device="cuda").transpose(1, 2)
    moda_forward_into(O, *args, 2, kernel="simt")
    assert max_abs(O.float().cpu().numpy(), ref) <= BF16_ABS_TOL


def test_short_depth_buffer_raises_like_the_reference():
    args = dev(seeded_inputs(1, 8, 4, 64, 64, 5, seed=12), torch.bfloat16)
    with pytest.raises(RuntimeError):
        moda_attention_cuda(*args, 6)


# ------------------------------------------------------------------ full benchmark sizes
@pytest.mark.slow
def test_kernel_only_benchmark_config_sampled_rows():
    # B=4 H_q=32 H_k=8 T=8192 d=128 L=32 bf16: spot rows against the oracle
    B, Hq, Hk, T, d, L = 4, 32, 8, 8192, 128, 32
    g = torch.Generator(device="cuda").manual_seed(2)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g, dtype=torch.bfloat16)
    Q, K, V = mk(B, Hq, T, d), mk(B, Hk, T, d), mk(B, Hk, T, d)
    Kd, Vd = mk(B, Hk, T * L, d), mk(B, Hk, T * L, d)
    out = moda_attention_cuda(Q, K, V, Kd, Vd, L, chunk_size=64)
    assert torch.isfinite(out).all()
    rng = np.random.default_rng(0)
    rows = [(0, 0, 0), (B - 1, Hq - 1, T - 1), (1, 5, 4095), (2, 17, 128), (3, 31, 127)]
    rows += [(int(rng.integers(B)), int(rng.integers(Hq)), int(rng.integers(T))) for _ in range(27)]
    G = Hq // Hk
    for (b, h, t) in rows:
        hk = h // G
        ref = orc.moda_row(Q[b, h, t].cpu().double().numpy(), K[b, hk, :t + 1].cpu().double().numpy(),
                           V[b, hk, :t + 1].cpu().double().numpy(),
                           Kd[b, hk, t * L:(t + 1) * L].cpu().double().numpy(),
                           Vd[b, hk, t * L:(t + 1) * L].cpu().double().numpy(), d ** -0.5)
        assert max_abs(out[b, h, t].float().cpu().numpy(), ref) <= BF16_ABS_TOL, (b, h, t)


@pytest.mark.slow
def test_scaling_config_one_batch_sampled_rows():
    # one batch of the multi-GPU configuration (H_q=64, H_k=8: G=8, T=16384, d=128, L=48),
    # bf16: the G=8 tiling, 48 depth rows per token and the longest sequences
    B, Hq, Hk, T, d, L = 1, 64, 8, 16384, 128, 48
    g = torch.Generator(device="cuda").manual_seed(4)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g, dtype=torch.bfloat16)
    Q, K, V = mk(B, Hq, T, d), mk(B, Hk, T, d), mk(B, Hk, T, d)
    Kd, Vd = mk(B, Hk, T * L, d), mk(B, Hk, T * L, d)
    out = moda_attention_cuda(Q, K, V, Kd, Vd, L, chunk_size=128)
    assert torch.isfinite(out).all()
    rng = np.random.default_rng(1)
    rows = [(0, 0, 0), (0, Hq - 1, T - 1), (0, 9, 8191), (0, 40, 16)]
    rows += [(0, int(rng.integers(Hq)), int(rng.integers(T))) for _ in range(12)]
    G = Hq // Hk
    for (b, h, t) in rows:
        hk = h // G
        ref = orc.moda_row(Q[b, h, t].cpu().double().numpy(), K[b, hk, :t + 1].cpu().double().numpy(),
                           V[b, hk, :t + 1].cpu().double().numpy(),
                           Kd[b, hk, t * L:(t + 1) * L].cpu().double().numpy(),
                           Vd[b, hk, t * L:(t + 1) * L].cpu().double().numpy(), d ** -0.5)
        assert max_abs(out[b, h, t].float().cpu().numpy(), ref) <= BF16_ABS_TOL, (b, h, t)


def _boundary_rows(B, Hq, T, G, L, seed, n_random=16):
    """First/last tokens, query-tile edges (128/G tokens per tile), 16k-1 tokens, tokens
    whose depth window [t*L, (t+1)*L) straddles a 128-row block, and seeded random rows."""
    n_tok = 128 // G
    toks = {0, T - 1, n_tok - 1, n_tok, 2 * n_tok - 1, 2 * n_tok, 15, 16 * 7 - 1, 16 * 64 - 1}
    toks |= {t for t in range(0, min(T, 600)) if (t * L) // 128 != ((t + 1) * L - 1) // 128}
    toks = sorted(t for t in toks if 0 <= t < T)
    rng = np.random.default_rng(seed)
    rows = [(int(rng.integers(B)), int(rng.integers(Hq)), t) for t in toks]
    rows += [(B - 1, Hq - 1, T - 1), (0, 0, 0)]
    rows += [(int(rng.integers(B)), int(rng.integers(Hq)), int(rng.integers(T)))
             for _ in range(n_random)]
    return rows


def _check_sampled(out, Q, K, V, Kd, Vd, L, rows):
    G = Q.shape[1] // K.shape[1]
    d = Q.shape[3]
    for (b, h, t) in rows:
        hk = h // G
        ref = orc.moda_row(Q[b, h, t].cpu().double().numpy(), K[b, hk, :t + 1].cpu().double().numpy(),
                           V[b, hk, :t + 1].cpu().double().numpy(),
                           Kd[b, hk, t * L:(t + 1) * L].cpu().double().numpy(),
                           Vd[b, hk, t * L:(t + 1) * L].cpu().double().numpy(), d ** -0.5)
        assert max_abs(out[b, h, t].float().cpu().numpy(), ref) <= BF16_ABS_TOL, (b, h, t)


@pytest.mark.slow
def test_module_config_kernel_shape_sampled_rows():
    """The module configuration's kernel call at full size: B=8, H_q=8, H_k=4, T=2048,
    d=64, L=5 (L not a multiple of 16: the per-score depth mask), Q/K/V as the module
    passes them (transposed views of [B, T, H, d] projections), depth [8, 4, 10240, 64]."""
    B, Hq, Hk, T, d, L = 8, 8, 4, 2048, 64, 5
    g = torch.Generator(device="cuda").manual_seed(1)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g, dtype=torch.bfloat16)
    Q = mk(B, T, Hq, d).transpose(1, 2)
    K, V = mk(B, T, Hk, d).transpose(1, 2), mk(B, T, Hk, d).transpose(1, 2)
    Kd, Vd = mk(B, Hk, T * L, d), mk(B, Hk, T * L, d)
    assert moda_plan(Q, K, V, Kd, Vd, L) == "tc"
    out = moda_attention_cuda(Q, K, V, Kd, Vd, L, chunk_size=64)
    assert torch.isfinite(out).all()
    _check_sampled(out, Q, K, V, Kd, Vd, L, _boundary_rows(B, Hq, T, Hq // Hk, L, seed=3))


@pytest.mark.slow
def test_model_config_kernel_shape_through_depth_cache_sampled_rows():
    """The model configuration's per-layer kernel call at full size: B=8, H_q=16, H_k=4,
    T=4096, d=128, read through a real DepthKVCache of 2N = 48 slots per token with
    num_layers = N = 24, as MoDAModel addresses it (token t reads rows [24t, 24t+24) of
    the 48-slot buffer). L = 24 is not a multiple of 16: the per-score depth mask, and
    windows that straddle 128-row blocks."""
    from moda import DepthKVCache
    B, Hq, Hk, T, d, N = 8, 16, 4, 4096, 128, 24
    g = torch.Generator(device="cuda").manual_seed(3)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g, dtype=torch.bfloat16)
    cache = DepthKVCache(B, T, 2 * N, Hk, d, device="cuda", dtype=torch.bfloat16)
    for slot in range(2 * N):  # every slot written, as after a full forward
        k = mk(B, T, Hk, d).transpose(1, 2)
        v = mk(B, T, Hk, d).transpose(1, 2)
        cache.write(slot, k, v, T)
    Kd, Vd = cache.read(T)
    assert Kd.shape[2] == T * 2 * N
    Q = mk(B, T, Hq, d).transpose(1, 2)
    K, V = mk(B, T, Hk, d).transpose(1, 2), mk(B, T, Hk, d).transpose(1, 2)
    assert moda_plan(Q, K, V, Kd, Vd, N) == "tc"
    out = moda_attention_cuda(Q, K, V, Kd, Vd, N, chunk_size=64)
    assert torch.isfinite(out).all()
    _check_sampled(out, Q, K, V, Kd, Vd, N, _boundary_rows(B, Hq, T, Hq // Hk, N, seed=4))


# query-head groups that do not divide 128 (H_q / H_k = 3, 5, 6, 12): the tcgen05 kernel
# runs them as G problems with one query head per KV head
ODD_G = [(1, 6, 2, 130, 64, 3), (2, 15, 3, 77, 128, 5), (1, 12, 2, 64, 64, 32), (1, 12, 1, 200, 128, 2)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("shape", ODD_G, ids=[str(s) for s in ODD_G])
def test_tc_odd_group_sizes_match_oracle(shape, dtype):
    from moda.kernels.moda_cuda import moda_forward_into, moda_forward_lse
    B, Hq, Hk, T, d, L = shape
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=T + Hq)
    args = dev(arrs, dtype)
    assert moda_plan(*args, L) == "tc"
    rin = rounded(arrs, dtype)
    ref = orc.moda_attention_naive(*rin, L)
    assert max_abs(run(args, L, kernel="tc"), ref) <= BF16_ABS_TOL
    # the row log-sum-exp lands at each head's own rows
    O, lse = moda_forward_lse(*args, L)
    lse_ref = orc.moda_attention_grads(*rin, L, np.zeros((B, Hq, T, d)))["lse"]
    assert max_abs(O.float().cpu().numpy(), ref) <= BF16_ABS_TOL
    assert max_abs(lse.cpu().numpy(), lse_ref) <= 1e-2 * max(1.0, float(np.abs(lse_ref).max()))
    # into a [B, T, H_q, d] buffer seen as [B, H_q, T, d]
    Ot = torch.zeros(B, T, Hq, d, dtype=dtype, device="cuda").transpose(1, 2)
    moda_forward_into(Ot, *args, L, kernel="tc")
    assert max_abs(Ot.float().cpu().numpy(), ref) <= BF16_ABS_TOL


def test_tc_odd_group_gradients_match_oracle():
    # the backward reads the forward's log-sum-exp rows, so this also checks where the
    # G launches put them
    B, Hq, Hk, T, d, L = 1, 6, 2, 70, 64, 3
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=5)
    ins = [t.requires_grad_(True) for t in dev(arrs, torch.bfloat16)]
    dO = np.random.default_rng(6).standard_normal((B, Hq, T, d))
    moda_attention_cuda(*ins, L).backward(torch.from_numpy(dO).to("cuda", torch.bfloat16))
    g = orc.moda_attention_grads(*rounded(arrs, torch.bfloat16), L,
                                 torch.from_numpy(dO).to(torch.bfloat16).double().numpy())
    for t, k in zip(ins, ("dQ", "dK", "dV", "dK_depth", "dV_depth")):
        e = float(np.abs(t.grad.double().cpu().numpy() - g[k]).max()) / max(1.0, float(np.abs(g[k]).max()))
        assert e <= 3e-2, (k, e)


# 16-bit on the tiled CUDA-core kernel: head dims the tensor-core kernel does not take,
# and head_dim 64 / 128 with the CUDA-core kernel forced
HALF_TILED = [(1, 4, 2, 130, 8, 3, "auto"), (2, 6, 3, 77, 36, 5, "auto"), (1, 4, 2, 200, 96, 33, "auto"),
              (1, 8, 2, 129, 64, 4, "simt"), (1, 4, 4, 64, 128, 2, "simt")]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("case", HALF_TILED, ids=[str(c) for c in HALF_TILED])
def test_half_inputs_on_the_tiled_cuda_core_kernel(case, dtype):
    B, Hq, Hk, T, d, L, kernel = case
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=T + d)
    args = dev(arrs, dtype)
    if kernel == "auto":
        assert moda_plan(*args, L) == "simt"
    ref = orc.moda_attention_naive(*rounded(arrs, dtype), L)
    assert max_abs(run(args, L, kernel=kernel), ref) <= BF16_ABS_TOL
