"""Parity of the CUDA backward (moda_bwd via the C ABI) with the reference's gradients.

The golden gradient fixtures hold torch autograd through the reference's
moda_attention_naive (fp64, tests/golden/make_golden.py); the oracle's closed
form (oracle/moda_oracle.py: moda_attention_grads) is pinned to them on CPU.

Tolerances:
  fp32 inputs: max|g - ref| / max|ref| <= 1e-4 for every gradient   (FP32_REL_TOL)
  bf16/f16 inputs (gradients stored in that dtype), against the fp64 oracle on the
  same rounded inputs: max|g - ref| <= 2e-2 * max(1, max|ref|)       (BF16_ABS_TOL)
"""

import numpy as np
import pytest
import torch

from moda.kernels import device_status, moda_attention_cuda, moda_backward, moda_forward_lse
from oracle import moda_oracle as orc
from helpers import BF16_ABS_TOL, FP32_REL_TOL, golden_cases, rel_err, seeded_inputs

pytestmark = pytest.mark.gpu
GRAD_CASES = golden_cases("grad")
NAMES = ("Q", "K", "V", "K_depth", "V_depth")
GRADS = ("dQ", "dK", "dV", "dK_depth", "dV_depth")


def dev(arrs, dtype):
    return [torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype) for a in arrs]


def rounded(arrs, dtype):
    return [torch.from_numpy(np.ascontiguousarray(a)).to(dtype).double().numpy() for a in arrs]


def host(t):
    return t.double().cpu().numpy()


def half_ok(g, ref):
    return float(np.max(np.abs(g - ref))) <= BF16_ABS_TOL * max(1.0, float(np.max(np.abs(ref))))


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert device_status() == 0, "a bounded device wait expired"


@pytest.mark.parametrize("name,z,meta", GRAD_CASES, ids=[c[0] for c in GRAD_CASES])
def test_golden_grads_fp32(name, z, meta):
    ins = dev([z[k] for k in NAMES], torch.float32)
    O, lse = moda_forward_lse(*ins, meta["L"], meta["scale"])
    dO = dev([z["dO"]], torch.float32)[0]
    grads = moda_backward(dO, *ins, O, lse, meta["L"], meta["scale"])
    torch.cuda.synchronize()
    assert rel_err(host(O), z["O"]) <= FP32_REL_TOL
    ref = orc.moda_attention_grads(*[z[k] for k in NAMES], meta["L"], z["dO"], scale=meta["scale"])
    assert float(np.max(np.abs(host(lse) - ref["lse"]))) <= 1e-4
    for g, k in zip(grads, GRADS):
        assert g.shape == ins[GRADS.index(k)].shape and g.dtype == torch.float32
        assert rel_err(host(g), z[k]) <= FP32_REL_TOL, (k, rel_err(host(g), z[k]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("name,z,meta", GRAD_CASES, ids=[c[0] for c in GRAD_CASES])
def test_golden_grads_half(name, z, meta, dtype):
    arrs = [z[k] for k in NAMES]
    rin = rounded(arrs + [z["dO"]], dtype)
    ref = orc.moda_attention_grads(*rin[:5], meta["L"], rin[5], scale=meta["scale"])
    ins = dev(arrs, dtype)
    dO = dev([z["dO"]], dtype)[0]
    for kernel in ("auto", "simt"):   # forward on the tcgen05 kernel where it tiles
        O, lse = moda_forward_lse(*ins, meta["L"], meta["scale"], kernel=kernel)
        grads = moda_backward(dO, *ins, O, lse, meta["L"], meta["scale"])
        torch.cuda.synchronize()
        assert float(np.max(np.abs(host(lse) - ref["lse"]))) <= 1e-2, kernel
        for g, k in zip(grads, GRADS):
            assert g.dtype == dtype
            assert half_ok(host(g), ref[k]), (kernel, k, float(np.max(np.abs(host(g) - ref[k]))))


def test_medium_shape_bf16():
    """B=1, H_q=8, H_k=2 (GQA 4), T=256, d=128, L=4: the tcgen05 forward's tiling and
    several causal blocks, against the oracle."""
    L = 4
    arrs = seeded_inputs(1, 8, 2, 256, 128, L, seed=50)
    dO = np.random.default_rng(51).standard_normal((1, 8, 256, 128)).astype(np.float32)
    rin = rounded(arrs + [dO], torch.bfloat16)
    ref = orc.moda_attention_grads(*rin[:5], L, rin[5])
    ins = dev(arrs, torch.bfloat16)
    O, lse = moda_forward_lse(*ins, L, kernel="tc")
    grads = moda_backward(dev([dO], torch.bfloat16)[0], *ins, O, lse, L)
    torch.cuda.synchronize()
    for g, k in zip(grads, GRADS):
        assert half_ok(host(g), ref[k]), (k, float(np.max(np.abs(host(g) - ref[k]))))


def test_autograd_through_moda_attention_cuda():
    """Reference tests/test_kernel.py:106-119: out.sum().backward() gives finite
    gradients for all five inputs (dO is then a zero-stride expanded tensor)."""
    B, H, T, L, d = 1, 2, 4, 2, 8
    arrs = seeded_inputs(B, H, H, T, d, L, seed=52)
    ins = [t.requires_grad_(True) for t in dev(arrs, torch.float32)]
    out = moda_attention_cuda(*ins, num_layers=L)
    out.sum().backward()
    ref = orc.moda_attention_grads(*arrs, L, np.ones((B, H, T, d)))
    for t, k in zip(ins, GRADS):
        assert t.grad is not None and torch.isfinite(t.grad).all(), k
        assert rel_err(host(t.grad), ref[k]) <= FP32_REL_TOL, k


@pytest.mark.parametrize("shape", [(2, 4, 2, 0, 64, 3), (0, 4, 2, 5, 128, 3)], ids=["T0", "B0"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_autograd_on_empty_inputs(shape, dtype):
    """Empty sequence or batch: the reference's autograd gives empty gradients of the
    inputs' shapes (oracle too); so does the CUDA backward."""
    B, H_q, H_k, T, d, L = shape
    arrs = seeded_inputs(B, H_q, H_k, T, d, L, seed=53)
    ins = [t.requires_grad_(True) for t in dev(arrs, dtype)]
    out = moda_attention_cuda(*ins, num_layers=L)
    out.sum().backward()
    torch.cuda.synchronize()
    ref = orc.moda_attention_grads(*arrs, L, np.ones((B, H_q, T, d)))
    for t, k in zip(ins, GRADS):
        assert t.grad is not None and tuple(t.grad.shape) == ref[k].shape == tuple(t.shape), k


def test_double_backward_raises():
    """Second derivatives are not implemented: differentiating a gradient of the CUDA
    attention raises (the backward is once-differentiable) rather than returning values
    that miss the backward's dependence on its inputs."""
    B, H, T, L, d = 1, 2, 6, 2, 16
    arrs = seeded_inputs(B, H, H, T, d, L, seed=54)
    ins = [t.requires_grad_(True) for t in dev(arrs, torch.float32)]
    out = moda_attention_cuda(*ins, num_layers=L)
    (gq,) = torch.autograd.grad(out.square().sum(), ins[0], create_graph=True)
    with pytest.raises(RuntimeError):
        gq.sum().backward()


def test_autograd_matches_direct_backward_with_strided_views():
    """MoDAAttention hands the kernel transposed views; gradients flow back into them."""
    B, Hq, Hk, T, d, L = 2, 4, 2, 24, 64, 3
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=53)
    q_bthd = torch.from_numpy(np.ascontiguousarray(arrs[0].transpose(0, 2, 1, 3))).cuda().bfloat16()
    q_bthd.requires_grad_(True)
    rest = [t.requires_grad_(True) for t in dev(arrs[1:], torch.bfloat16)]
    Q = q_bthd.transpose(1, 2)                       # strides (T*H*d, d, H*d, 1)
    out = moda_attention_cuda(Q, *rest, num_layers=L)
    W = torch.randn(out.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(54))
    (out.float() * W).sum().backward()
    rin = rounded(arrs, torch.bfloat16)
    ref = orc.moda_attention_grads(*rin, L, W.double().cpu().numpy())
    assert half_ok(host(q_bthd.grad.transpose(1, 2)), ref["dQ"])
    for t, k in zip(rest, GRADS[1:]):
        assert half_ok(host(t.grad), ref[k]), k


def test_module_gradient_through_depth():
    """Reference tests/test_attention.py:57-71 on CUDA: gradients reach x, K_depth, V_depth."""
    from moda.config import MoDAConfig
    from moda.attention import MoDAAttention
    torch.manual_seed(55)
    cfg = MoDAConfig(d_model=64, num_heads=4, num_kv_heads=2, num_layers=3)
    attn = MoDAAttention(cfg).cuda()
    B, T, L = 1, 4, 3
    x = torch.randn(B, T, cfg.d_model, device="cuda", requires_grad=True)
    Kd = torch.randn(B, cfg.num_kv_heads, T * L, cfg.head_dim, device="cuda", requires_grad=True)
    Vd = torch.randn(B, cfg.num_kv_heads, T * L, cfg.head_dim, device="cuda", requires_grad=True)
    out, _, _ = attn(x, Kd, Vd)
    out.sum().backward()
    for t in (x, Kd, Vd):
        assert t.grad is not None and torch.isfinite(t.grad).all()
        assert float(t.grad.abs().max()) > 0


@pytest.mark.parametrize("lean", [False, True])
@pytest.mark.parametrize("name", ["model_grad_postnorm", "model_grad_prenorm"])
def test_model_gradients_match_reference(name, lean):
    # 3-layer MoDAModel trained through the depth cache: gradients reach every depth
    # projection whose rows a later layer reads (through the in-place cache writes), and
    # every attention sees the cache as it was when it read it. Reference: fp64 autograd.
    from helpers import load_golden
    from moda import MoDAConfig, MoDAModel
    z, meta = load_golden(name)
    model = MoDAModel(MoDAConfig(**meta["config"], lean_depth_cache=lean))
    model.load_state_dict({k[2:]: torch.from_numpy(z[k]) for k in z.files if k.startswith("w.")})
    model = model.cuda()
    x = torch.from_numpy(z["x"]).cuda().requires_grad_()
    out = model(x)
    (out * torch.from_numpy(z["loss_weight"]).cuda()).sum().backward()
    assert rel_err(out.detach().cpu().numpy(), z["out"]) <= FP32_REL_TOL
    assert rel_err(x.grad.cpu().numpy(), z["x_grad"]) <= FP32_REL_TOL
    for pname, p in model.named_parameters():
        if pname in meta["no_grad_params"]:
            assert p.grad is None or not p.grad.any(), pname
        else:
            assert p.grad is not None, pname
            assert rel_err(p.grad.cpu().numpy(), z["g." + pname]) <= FP32_REL_TOL, pname


DEPTH_MMA_CASES = [  # B, H_q, H_k, T, d, L: the tensor-core depth backward's range
    (1, 8, 2, 37, 128, 32),   # G = 4, L at its maximum, T ends inside a 16-row block
    (1, 16, 2, 20, 64, 17),   # G = 8, L not a multiple of 8
    (2, 16, 1, 9, 128, 5),    # G = 16: one token per block
    (1, 2, 2, 33, 64, 32),    # G = 1: sixteen tokens per block
    (1, 8, 2, 21, 128, 48),   # two key chunks per token, the second partial
    (1, 4, 1, 10, 64, 70),    # three key chunks
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("case", DEPTH_MMA_CASES, ids=[str(c) for c in DEPTH_MMA_CASES])
def test_depth_backward_tensor_core_range(case, dtype):
    B, Hq, Hk, T, d, L = case
    arrs = seeded_inputs(B, Hq, Hk, T, d, L, seed=60 + T)
    dO = np.random.default_rng(61 + T).standard_normal((B, Hq, T, d)).astype(np.float32)
    rin = rounded(arrs + [dO], dtype)
    ref = orc.moda_attention_grads(*rin[:5], L, rin[5])
    ins = dev(arrs, dtype)
    O, lse = moda_forward_lse(*ins, L)
    grads = moda_backward(dev([dO], dtype)[0], *ins, O, lse, L)
    torch.cuda.synchronize()
    for g, k in zip(grads, GRADS):
        assert half_ok(host(g), ref[k]), (k, float(np.max(np.abs(host(g) - ref[k]))))


@pytest.mark.slow
def test_kernel_only_config_backward_sampled_tokens():
    # B=1 of the kernel-only configuration (H_q=32, H_k=8, T=8192, d=128, L=32), bf16:
    # dQ rows and the depth rows' gradients of sampled tokens, exactly per token in fp64
    B, Hq, Hk, T, d, L = 1, 32, 8, 8192, 128, 32
    G = Hq // Hk
    g = torch.Generator(device="cuda").manual_seed(9)
    mk = lambda *s: torch.randn(*s, device="cuda", generator=g, dtype=torch.bfloat16)
    Q, K, V, dO = mk(B, Hq, T, d), mk(B, Hk, T, d), mk(B, Hk, T, d), mk(B, Hq, T, d)
    Kd, Vd = mk(B, Hk, T * L, d), mk(B, Hk, T * L, d)
    O, lse = moda_forward_lse(Q, K, V, Kd, Vd, L)
    dQ, dK, dV, dKd, dVd = moda_backward(dO, Q, K, V, Kd, Vd, O, lse, L)
    torch.cuda.synchronize()
    for t_ in (dQ, dK, dV, dKd, dVd):
        assert torch.isfinite(t_).all()
    h = lambda x: x.float().cpu().numpy()
    rng = np.random.default_rng(3)
    picks = [(0, 0), (Hk - 1, T - 1), (3, 4095), (5, 128)]
    picks += [(int(rng.integers(Hk)), int(rng.integers(T))) for _ in range(8)]
    for hk, t in picks:
        heads = slice(hk * G, (hk + 1) * G)
        rows = slice(t * L, (t + 1) * L)
        ref = orc.moda_token_grads(h(Q[0, heads, t]), h(dO[0, heads, t]), h(K[0, hk, :t + 1]),
                                   h(V[0, hk, :t + 1]), h(Kd[0, hk, rows]), h(Vd[0, hk, rows]), d ** -0.5)
        assert half_ok(h(dQ[0, heads, t]), ref["dQ"]), ("dQ", hk, t)
        assert half_ok(h(dKd[0, hk, rows]), ref["dK_depth"]), ("dK_depth", hk, t)
        assert half_ok(h(dVd[0, hk, rows]), ref["dV_depth"]), ("dV_depth", hk, t)
