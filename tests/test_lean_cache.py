"""Opt-in lean depth-cache lifecycle of MoDAModel (config.lean_depth_cache).

CPU: the row-liveness rule against enumeration, a row-level replay of the cache
lifecycle (every row any layer reads is the same with and without the lean
flag, and the first layer reads only zeros), and the whole model on CPU with the
CUDA calls swapped for the oracle, lean and default, against the reference's own
model outputs (golden files made by running the reference).
GPU: the implicit-zero-row kernel against explicit zero depth rows (values, lse,
gradients) and the lean model against the default one and the golden outputs.
"""

import numpy as np
import pytest
import torch

import moda.attention as moda_attention_mod
import moda.cache as moda_cache_mod
from moda import MoDAConfig, MoDAModel
from moda.model import live_write_tokens
from helpers import BF16_ABS_TOL, FP32_REL_TOL, load_golden, max_abs, rel_err, seeded_inputs
from oracle.moda_oracle import moda_attention_naive


# ---------------------------------------------------------------- CPU: host logic

@pytest.mark.parametrize("T", [0, 1, 2, 3, 7, 16, 33])
@pytest.mark.parametrize("n_read,slots", [(1, 2), (3, 6), (4, 8), (5, 10), (2, 7)])
def test_live_write_tokens_matches_enumeration(T, n_read, slots):
    for slot in range(slots):
        live = [t for t in range(T) if t * slots + slot < T * n_read]
        assert live == list(range(len(live)))  # always a prefix
        assert live_write_tokens(T, n_read, slots, slot) == len(live)


def _replay(T, N, lean):
    """Row tags of the cache as each layer reads it: 0 = zero, -1 = never initialised,
    else a unique id of the (layer slot, token) that wrote the row."""
    slots = 2 * N
    rows = np.full(T * slots, -1 if lean else 0, np.int64)
    if lean:
        rows[:T * N] = 0
    reads, written = [], False
    for i in range(N):
        reads.append((rows[:T * N].copy(), lean and not written))
        for slot in (2 * i, 2 * i + 1):
            n = T
            if lean:
                n = 0 if i == N - 1 else live_write_tokens(T, N, slots, slot)
            for t in range(n):
                rows[t * slots + slot] = 1 + slot * T + t
            written = written or n > 0
    return reads


@pytest.mark.parametrize("T,N", [(1, 1), (5, 1), (8, 2), (7, 3), (16, 4), (9, 6), (12, 24)])
def test_lean_lifecycle_reads_what_the_default_reads(T, N):
    default, lean = _replay(T, N, False), _replay(T, N, True)
    for i, ((rows_d, _), (rows_l, implicit_zero)) in enumerate(zip(default, lean)):
        if implicit_zero:  # the lean first layer reads nothing: it must be all zeros
            assert i == 0 and not rows_d.any()
        else:
            assert (rows_l >= 0).all(), f"layer {i} would read an uninitialised row"
            assert (rows_l == rows_d).all(), f"layer {i} reads different rows"


def _oracle_attention(Q, K, V, K_depth, V_depth, num_layers, scale=None, chunk_size=None,
                      out=None, **_):
    np_ = [t.detach().cpu().numpy() for t in (Q, K, V, K_depth, V_depth)]
    o = torch.from_numpy(moda_attention_naive(*np_, num_layers, scale=scale,
                                              chunk_size=chunk_size)).to(Q.dtype)
    return o if out is None else out.copy_(o)


def _oracle_zero_depth(Q, K, V, zero_rows, scale=None, out=None, **_):
    B, H_k, T, d = K.shape
    zeros = torch.zeros(B, H_k, T * zero_rows, d, dtype=Q.dtype)
    return _oracle_attention(Q, K, V, zeros, zeros, zero_rows, scale=scale, out=out)


def _torch_append(k_cache, v_cache, layer_idx, k, v, num_layers, seq_len):
    L = num_layers
    k_cache[:, :, layer_idx:seq_len * L:L] = k[:, :, :seq_len]
    v_cache[:, :, layer_idx:seq_len * L:L] = v[:, :, :seq_len]


class _NaNEmpty:
    """torch with ``empty`` returning NaN-filled tensors: any read of a cache row the
    lean lifecycle left uninitialised poisons the output."""

    def __getattr__(self, name):
        return getattr(torch, name)

    @staticmethod
    def empty(*size, **kw):
        return torch.full(size[0] if len(size) == 1 else size, float("nan"), **kw)


@pytest.fixture
def oracle_stand_ins(monkeypatch):
    monkeypatch.setattr(moda_attention_mod, "moda_attention_cuda", _oracle_attention)
    monkeypatch.setattr(moda_attention_mod, "moda_attention_zero_depth", _oracle_zero_depth)
    monkeypatch.setattr(moda_cache_mod, "depth_append", _torch_append)
    monkeypatch.setattr(moda_cache_mod, "torch", _NaNEmpty())


def _golden_model(name, lean):
    z, meta = load_golden(name)
    model = MoDAModel(MoDAConfig(**meta["config"], lean_depth_cache=lean))
    model.load_state_dict({k[2:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("w.")})
    return model.eval(), torch.from_numpy(z["x"]), z["out"]


@pytest.mark.parametrize("name", ["model_postnorm", "model_prenorm"])
def test_lean_model_host_logic_matches_reference_on_cpu(oracle_stand_ins, name):
    outs = []
    for lean in (False, True):
        model, x, ref = _golden_model(name, lean)
        with torch.no_grad():
            out = model(x).numpy()
        assert np.isfinite(out).all()
        assert rel_err(out, ref) <= FP32_REL_TOL
        outs.append(out)
    assert max_abs(outs[0], outs[1]) <= 1e-5


# ---------------------------------------------------------------- GPU

@pytest.fixture
def _gpu_status():
    yield
    from moda.kernels import device_status
    assert device_status() == 0


def _cuda(arrs, dtype):
    return [torch.from_numpy(a).to(device="cuda", dtype=dtype) for a in arrs]


ZERO_CASES = [  # B, H_q, H_k, T, d, Z
    (1, 4, 2, 37, 64, 3),
    (2, 8, 2, 300, 128, 32),
    (1, 16, 4, 129, 128, 24),
    (1, 2, 2, 5, 32, 1),
]


@pytest.mark.gpu
@pytest.mark.parametrize("kernel", ["tc", "simt"])
@pytest.mark.parametrize("case", ZERO_CASES, ids=[str(c) for c in ZERO_CASES])
def test_zero_depth_kernel_equals_explicit_zero_rows(_gpu_status, case, kernel):
    from moda.kernels import moda_forward_lse
    from moda.kernels.moda_cuda import moda_forward_zero_depth
    B, Hq, Hk, T, d, Z = case
    dtype = torch.bfloat16 if kernel == "tc" else torch.float32
    if kernel == "tc" and d not in (64, 128):
        pytest.skip("tensor-core path needs d in {64, 128}")
    Q, K, V, _, _ = seeded_inputs(B, Hq, Hk, T, d, 0, seed=11)
    q, k, v = _cuda((Q, K, V), dtype)
    zeros = torch.zeros(B, Hk, T * Z, d, device="cuda", dtype=dtype)
    o_imp, lse_imp = moda_forward_zero_depth(q, k, v, Z, kernel=kernel)
    o_exp, lse_exp = moda_forward_lse(q, k, v, zeros, zeros, Z, kernel=kernel)
    ref = moda_attention_naive(*(t.float().cpu().numpy() for t in (q, k, v, zeros, zeros)), Z)
    torch.cuda.synchronize()
    tol = BF16_ABS_TOL if dtype == torch.bfloat16 else 1e-5
    assert max_abs(o_imp.float().cpu().numpy(), ref) <= tol
    assert max_abs(o_imp.float().cpu().numpy(), o_exp.float().cpu().numpy()) <= tol
    assert max_abs(lse_imp.cpu().numpy(), lse_exp.cpu().numpy()) <= 1e-4


@pytest.mark.gpu
def test_zero_depth_gradients_equal_explicit_zero_rows(_gpu_status):
    from moda.kernels import moda_attention_cuda, moda_attention_zero_depth
    B, Hq, Hk, T, d, Z = 1, 8, 2, 96, 128, 6
    Q, K, V, _, _ = seeded_inputs(B, Hq, Hk, T, d, 0, seed=12)
    dO = torch.randn(B, Hq, T, d, generator=torch.Generator().manual_seed(5)).cuda().float()
    grads = []
    for implicit in (True, False):
        q, k, v = (t.requires_grad_() for t in _cuda((Q, K, V), torch.float32))
        if implicit:
            o = moda_attention_zero_depth(q, k, v, Z)
        else:
            zeros = torch.zeros(B, Hk, T * Z, d, device="cuda")
            o = moda_attention_cuda(q, k, v, zeros, zeros, Z)
        o.backward(dO)
        grads.append([t.grad.cpu().numpy() for t in (q, k, v)])
    for g_imp, g_exp in zip(*grads):
        assert rel_err(g_imp, g_exp) <= 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["model_postnorm", "model_prenorm"])
def test_lean_model_matches_default_and_reference(_gpu_status, name):
    outs = []
    for lean in (False, True):
        model, x, ref = _golden_model(name, lean)
        with torch.no_grad():
            out = model.cuda()(x.cuda()).cpu().numpy()
        assert rel_err(out, ref) <= FP32_REL_TOL
        outs.append(out)
    assert rel_err(outs[1], outs[0]) <= 1e-5


@pytest.mark.gpu
def test_lean_model_bf16_tensor_core_path_matches_default(_gpu_status):
    cfg = dict(d_model=512, num_heads=8, num_kv_heads=2, head_dim=128, num_layers=4,
               max_seq_len=256, post_norm=True)
    x = torch.randn(2, 256, 512, generator=torch.Generator().manual_seed(3))
    outs = []
    for lean in (False, True):
        torch.manual_seed(7)
        model = MoDAModel(MoDAConfig(**cfg, lean_depth_cache=lean)).cuda().to(torch.bfloat16)
        with torch.no_grad():
            outs.append(model(x.cuda().to(torch.bfloat16)).float().cpu().numpy())
    # post-norm outputs are O(1); layer 0's softmax sum is rounded differently
    assert max_abs(outs[0], outs[1]) <= 0.1
    assert np.mean(np.abs(outs[0] - outs[1])) <= 5e-3
