"""Depth-write projection with the cache append fused (moda_depth_proj_append) on GPU.

Reference behaviour: the two depth projections (nn.Linear, moda/attention.py:81-82 and
moda/model.py:78-81) followed by DepthKVCache.write (moda/cache.py:52-74). The fused
kernel must write exactly the rows t*L + slot for t < seq_len, with the projection
computed in fp32 from the 16-bit inputs (checked against a float32 torch product of
the same rounded tensors, tolerance 2e-2 absolute on outputs of unit scale), and leave
every other cache row untouched.
"""

import pytest
import torch

from moda.kernels import device_status
from moda.kernels._lib import MoDAUnsupported
from moda.kernels.moda_cuda import depth_append, depth_proj_append

pytestmark = pytest.mark.gpu

TOL = 2e-2


@pytest.fixture(autouse=True)
def _no_device_timeouts():
    yield
    assert device_status() == 0


def _case(B, T, D, Hk, d, L, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, T, D, device="cuda", generator=g).to(dtype)
    w = (torch.randn(2 * Hk * d, D, device="cuda", generator=g) / D ** 0.5).to(dtype)
    R = T * L
    kc = torch.full((B, Hk, R, d), 7.0, device="cuda", dtype=dtype)  # sentinel
    vc = torch.full((B, Hk, R, d), -7.0, device="cuda", dtype=dtype)
    return x, w, kc, vc


def _expected(x, w, kc, vc, slot, L, n):
    B, T, D = x.shape
    Hk, d = kc.shape[1], kc.shape[3]
    y = (x.float() @ w.float().t()).view(B, T, 2, Hk, d)
    ek, ev = kc.clone().float(), vc.clone().float()
    ek[:, :, slot:n * L:L] = y[:, :n, 0].transpose(1, 2)
    ev[:, :, slot:n * L:L] = y[:, :n, 1].transpose(1, 2)
    return ek, ev


CASES = [  # B, T, D, H_k, d, L, slot, n_write
    (2, 300, 256, 2, 64, 6, 3, 300),       # ragged T (last tile partly out of range)
    (1, 512, 2048, 4, 128, 48, 47, 512),   # the model configuration's head layout
    (2, 257, 200, 1, 64, 4, 0, 131),       # K tail (D % 64 != 0), N = 128 < tile, n < T
    (1, 96, 128, 3, 96, 2, 1, 96),         # d = 96: N = 576, chunks straddle tiles
    (3, 64, 64, 2, 32, 3, 2, 0),           # nothing to write
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", CASES, ids=[str(c) for c in CASES])
def test_fused_depth_projection_writes_the_cache_rows(case, dtype):
    B, T, D, Hk, d, L, slot, n = case
    x, w, kc, vc = _case(B, T, D, Hk, d, L, dtype)
    ek, ev = _expected(x, w, kc, vc, slot, L, n)
    depth_proj_append(x, w, kc, vc, slot, L, n)
    torch.cuda.synchronize()
    assert (kc.float() - ek).abs().max().item() <= TOL
    assert (vc.float() - ev).abs().max().item() <= TOL
    # rows not addressed by (t < n, slot) keep their sentinel exactly
    mask = torch.ones(kc.shape[2], dtype=torch.bool, device="cuda")
    mask[slot:n * L:L] = False
    assert (kc[:, :, mask] == 7.0).all() and (vc[:, :, mask] == -7.0).all()


def test_fused_equals_linear_plus_append_module_path():
    # what MoDATransformerBlock does without the fused kernel: two nn.Linear + the append
    torch.manual_seed(0)
    B, T, D, Hk, d, L, slot = 2, 200, 512, 2, 128, 8, 5
    dtype = torch.bfloat16
    kl = torch.nn.Linear(D, Hk * d, bias=False).cuda().to(dtype)
    vl = torch.nn.Linear(D, Hk * d, bias=False).cuda().to(dtype)
    x = torch.randn(B, T, D, device="cuda", dtype=dtype)
    kc1 = torch.zeros(B, Hk, T * L, d, device="cuda", dtype=dtype)
    vc1, kc2, vc2 = kc1.clone(), kc1.clone(), kc1.clone()
    with torch.no_grad():
        k = kl(x).view(B, T, Hk, d).transpose(1, 2)
        v = vl(x).view(B, T, Hk, d).transpose(1, 2)
        depth_append(kc1, vc1, slot, k, v, L, T)
        depth_proj_append(x, torch.cat([kl.weight, vl.weight]), kc2, vc2, slot, L, T)
    torch.cuda.synchronize()
    # both round an fp32 accumulation to bf16; they differ by accumulation order only
    assert (kc1.float() - kc2.float()).abs().max().item() <= TOL
    assert (vc1.float() - vc2.float()).abs().max().item() <= TOL


def test_fp32_is_refused_before_launch():
    x, w, kc, vc = _case(1, 8, 64, 1, 32, 2, torch.float32)
    with pytest.raises(MoDAUnsupported):
        depth_proj_append(x, w, kc, vc, 0, 2, 8)


# ---------------------------------------------------------------- fused Q/K/V projection
from moda.kernels.moda_cuda import qkv_proj  # noqa: E402

QKV_CASES = [  # B, T, D, H_q, H_k, d
    (2, 300, 256, 4, 2, 64),       # ragged T
    (1, 512, 2048, 16, 4, 128),    # the model configuration's heads (N = 3072)
    (2, 257, 200, 2, 1, 64),       # K tail (D % 64 != 0), N = 256
    (1, 96, 128, 6, 3, 96),        # d = 96: segment ends inside column tiles
    (1, 64, 512, 8, 4, 64),        # the module configuration's heads
]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("case", QKV_CASES, ids=[str(c) for c in QKV_CASES])
def test_fused_qkv_projection(case, dtype):
    """One GEMM over cat(W_q, W_k, W_v) writes Q, K, V head-major; each equals the
    float32 product of the same rounded inputs within the 16-bit output tolerance."""
    B, T, D, Hq, Hk, d = case
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(B, T, D, device="cuda", generator=g).to(dtype)
    w = (torch.randn((Hq + 2 * Hk) * d, D, device="cuda", generator=g) / D ** 0.5).to(dtype)
    Q, K, V = qkv_proj(x, w, Hq, Hk, d)
    torch.cuda.synchronize()
    y = x.float() @ w.float().t()
    eq = y[..., :Hq * d].view(B, T, Hq, d).transpose(1, 2)
    ek = y[..., Hq * d:(Hq + Hk) * d].view(B, T, Hk, d).transpose(1, 2)
    ev = y[..., (Hq + Hk) * d:].view(B, T, Hk, d).transpose(1, 2)
    for got, exp in ((Q, eq), (K, ek), (V, ev)):
        assert got.shape == exp.shape and got.is_contiguous()
        assert (got.float() - exp).abs().max().item() <= TOL


def test_module_uses_fused_qkv_without_autograd():
    """MoDAAttention under no_grad (fused QKV GEMM) and with autograd (three nn.Linear)
    give the same output within the 16-bit tolerance; the cached concatenated weight
    follows an in-place weight update."""
    from moda import MoDAAttention, MoDAConfig
    torch.manual_seed(0)
    cfg = MoDAConfig(d_model=256, num_heads=4, num_kv_heads=2, head_dim=64, num_layers=3)
    attn = MoDAAttention(cfg).cuda().to(torch.bfloat16)
    x = torch.randn(2, 96, 256, device="cuda", dtype=torch.bfloat16)
    Kd = torch.randn(2, 2, 96 * 3, 64, device="cuda", dtype=torch.bfloat16)
    Vd = torch.randn_like(Kd)
    for _ in range(2):
        with torch.no_grad():
            fast = attn(x, Kd, Vd)[0]
        ref = attn(x, Kd, Vd)[0].detach()
        assert (fast.float() - ref.float()).abs().max().item() <= TOL
        with torch.no_grad():
            attn.k_proj.weight.mul_(0.5)  # bumps the version: the fused weight is rebuilt


def test_module_falls_back_to_library_gemms_for_shapes_the_fused_kernel_refuses():
    """head_dim 16 (not a multiple of 32): the fused Q/K/V kernel refuses on the host, the
    module remembers it and uses the three nn.Linear; output as with autograd."""
    from moda import MoDAAttention, MoDAConfig
    torch.manual_seed(1)
    cfg = MoDAConfig(d_model=64, num_heads=4, num_kv_heads=2, head_dim=16, num_layers=2)
    attn = MoDAAttention(cfg).cuda().to(torch.bfloat16)
    x = torch.randn(1, 40, 64, device="cuda", dtype=torch.bfloat16)
    Kd = torch.randn(1, 2, 80, 16, device="cuda", dtype=torch.bfloat16)
    Vd = torch.randn_like(Kd)
    for _ in range(2):
        with torch.no_grad():
            fast = attn(x, Kd, Vd)[0]
        assert attn._qkv_fused_ok is False
    ref = attn(x, Kd, Vd)[0].detach()
    assert (fast.float() - ref.float()).abs().max().item() <= TOL
