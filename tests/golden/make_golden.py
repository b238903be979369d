"""Generate the golden fixtures in this folder by running the reference itself.

Run (in a container that has the reference checkout), giving the checkout's path
either as an argument or in the MODA_REFERENCE environment variable:

    python tests/golden/make_golden.py --reference <path to the reference checkout>

It imports ``moda`` from the reference checkout (pure Python/PyTorch, CPU,
fp32) and records seeded inputs and the reference's outputs as ``.npz`` files.
The GPU box never runs this script; the tests only read the ``.npz`` files.

Cases follow the reference's own tests (tests/test_kernel.py, tests/test_gqa.py,
tests/test_cache.py, tests/test_attention.py, tests/test_model.py) plus the
smallest benchmark configuration (B=1, H_q=4, H_k=2, T=32, d=64, L=8, seed 0).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _randn(gen_shape_list, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(*s, generator=g) for s in gen_shape_list]


def kernel_case(name, B, H_q, H_k, T, d, L, seed, chunk_sizes, extra_rows=0, scale=None):
    from moda.kernels.moda_naive import moda_attention_naive
    R = T * L + extra_rows
    Q, K, V, Kd, Vd = _randn([(B, H_q, T, d), (B, H_k, T, d), (B, H_k, T, d),
                              (B, H_k, R, d), (B, H_k, R, d)], seed)
    arrays = dict(Q=Q.numpy(), K=K.numpy(), V=V.numpy(), K_depth=Kd.numpy(), V_depth=Vd.numpy())
    outs = {}
    for C in chunk_sizes:
        try:
            o = moda_attention_naive(Q, K, V, Kd, Vd, num_layers=L, scale=scale, chunk_size=C)
            outs["out_" + ("full" if C is None else f"c{C}")] = o.numpy()
        except RuntimeError as e:          # recorded: the reference refuses this form
            outs["err_" + ("full" if C is None else f"c{C}")] = np.array(str(e).split("\n")[0])
    meta = dict(kind="kernel", B=B, H_q=H_q, H_k=H_k, T=T, d=d, L=L, seed=seed,
                scale=scale, depth_rows=R, chunk_sizes=[c for c in chunk_sizes])
    return name, arrays | outs, meta


def grad_case(name, B, H_q, H_k, T, d, L, seed, chunk_size, extra_rows=0, scale=None):
    """The reference's gradients: moda_attention_naive under torch autograd (CPU, fp64)."""
    from moda.kernels.moda_naive import moda_attention_naive
    R = T * L + extra_rows
    g = torch.Generator().manual_seed(seed)
    shapes = [(B, H_q, T, d), (B, H_k, T, d), (B, H_k, T, d), (B, H_k, R, d), (B, H_k, R, d),
              (B, H_q, T, d)]
    # fp32 inputs (stored exactly), fp64 arithmetic, results stored rounded to fp32
    Q, K, V, Kd, Vd, dO = [torch.randn(*s, generator=g) for s in shapes]
    leaves = [t.double().requires_grad_(True) for t in (Q, K, V, Kd, Vd)]
    O = moda_attention_naive(*leaves, num_layers=L, scale=scale, chunk_size=chunk_size)
    O.backward(dO.double())
    names = ["Q", "K", "V", "K_depth", "V_depth"]
    arrays = {n: t.numpy() for n, t in zip(names, (Q, K, V, Kd, Vd))}
    arrays |= {"dO": dO.numpy(), "O": O.detach().float().numpy()}
    arrays |= {"d" + n: t.grad.float().numpy() for n, t in zip(names, leaves)}
    meta = dict(kind="grad", B=B, H_q=H_q, H_k=H_k, T=T, d=d, L=L, seed=seed, scale=scale,
                depth_rows=R, chunk_size=chunk_size)
    return name, arrays, meta


def module_case():
    from moda.config import MoDAConfig
    from moda.attention import MoDAAttention
    torch.manual_seed(1)
    cfg = MoDAConfig(d_model=64, num_heads=4, num_kv_heads=2, num_layers=3)
    attn = MoDAAttention(cfg).eval()
    B, T, L = 2, 8, 3
    g = torch.Generator().manual_seed(11)
    x = torch.randn(B, T, cfg.d_model, generator=g)
    Kd = torch.randn(B, cfg.num_kv_heads, T * L, cfg.head_dim, generator=g)
    Vd = torch.randn(B, cfg.num_kv_heads, T * L, cfg.head_dim, generator=g)
    with torch.no_grad():
        out, kw, vw = attn(x, Kd, Vd)
    arrays = {f"w.{k}": v.numpy() for k, v in attn.state_dict().items()}
    arrays |= dict(x=x.numpy(), K_depth=Kd.numpy(), V_depth=Vd.numpy(),
                   out=out.numpy(), k_write=kw.numpy(), v_write=vw.numpy())
    meta = dict(kind="module", config=dict(d_model=64, num_heads=4, num_kv_heads=2, num_layers=3),
                B=B, T=T, L=L)
    return "module_attention", arrays, meta


def model_case(post_norm):
    from moda.config import MoDAConfig
    from moda.model import MoDAModel
    torch.manual_seed(3)
    cfg = MoDAConfig(d_model=64, num_heads=4, num_kv_heads=2, num_layers=2, max_seq_len=16,
                     post_norm=post_norm)
    model = MoDAModel(cfg).eval()
    g = torch.Generator().manual_seed(13)
    x = torch.randn(2, 8, cfg.d_model, generator=g)
    with torch.no_grad():
        out = model(x)
    arrays = {f"w.{k}": v.numpy() for k, v in model.state_dict().items()}
    arrays |= dict(x=x.numpy(), out=out.numpy())
    meta = dict(kind="model", config=dict(d_model=64, num_heads=4, num_kv_heads=2, num_layers=2,
                                          max_seq_len=16, post_norm=post_norm))
    return f"model_{'post' if post_norm else 'pre'}norm", arrays, meta


def model_grad_case(post_norm):
    """Parameter and input gradients of a 3-layer reference MoDAModel (fp64 autograd).

    With 3 layers, later layers write cache rows that earlier layers read (the 2N-slot
    cache addressed with L = N), so the gradients cover the autograd path through the
    in-place cache writes (moda/cache.py:73-74) as well as the attention."""
    from moda.config import MoDAConfig
    from moda.model import MoDAModel
    torch.manual_seed(5)
    conf = dict(d_model=32, num_heads=4, num_kv_heads=2, num_layers=3, max_seq_len=16,
                post_norm=post_norm)
    model = MoDAModel(MoDAConfig(**conf)).double()
    g = torch.Generator().manual_seed(19)
    # fp32-representable inputs, so the fp32 fixture holds them exactly
    x = torch.randn(2, 9, 32, generator=g).double().requires_grad_()
    w = torch.randn(2, 9, 32, generator=g).double()
    out = model(x)
    (out * w).sum().backward()
    f32 = lambda t: t.detach().float().numpy()  # weights start as fp32; fp32 keeps 1e-7
    arrays = {f"w.{k}": f32(v) for k, v in model.state_dict().items()}
    arrays |= {f"g.{k}": f32(p.grad) for k, p in model.named_parameters() if p.grad is not None}
    arrays |= dict(x=f32(x), loss_weight=f32(w), out=f32(out), x_grad=f32(x.grad))
    meta = dict(kind="model_grad", config=conf,
                no_grad_params=[k for k, p in model.named_parameters() if p.grad is None])
    return f"model_grad_{'post' if post_norm else 'pre'}norm", arrays, meta


def cache_case():
    from moda.cache import DepthKVCache
    B, T, L, H_k, d = 2, 5, 3, 2, 8
    cache = DepthKVCache(B, T, L, H_k, d)
    g = torch.Generator().manual_seed(17)
    arrays = {}
    for layer in (0, 2, 1):
        k = torch.randn(B, H_k, T, d, generator=g)
        v = torch.randn(B, H_k, T, d, generator=g)
        cache.write(layer, k, v)
        arrays[f"k{layer}"] = k.numpy()
        arrays[f"v{layer}"] = v.numpy()
    K, V = cache.read(seq_len=T)
    arrays |= dict(k_cache=K.numpy(), v_cache=V.numpy())
    Kp, _ = cache.read(seq_len=3)
    arrays["partial_shape"] = np.array(Kp.shape)
    meta = dict(kind="cache", B=B, T=T, L=L, H_k=H_k, d=d, order=[0, 2, 1])
    return "cache_write", arrays, meta


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MODA_REFERENCE"),
                    help="path of the reference checkout (default: $MODA_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set MODA_REFERENCE")
    sys.path.insert(0, args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    cases = [
        # smallest benchmark configuration: B=1 H_q=4 H_k=2 T=32 d=64 L=8, N(0,1) seed 0
        kernel_case("c1_b1_h4x2_t32_d64_l8", 1, 4, 2, 32, 64, 8, 0, [None, 8, 64]),
        # reference tests/test_kernel.py:159-185 shapes
        kernel_case("t_b1_h1_t8_d16_l4", 1, 1, 1, 8, 16, 4, 21, [None, 3]),
        kernel_case("t_b1_h4x2_t8_d16_l3", 1, 4, 2, 8, 16, 3, 22, [None, 4]),
        kernel_case("t_b4_h2_t16_d32_l4", 4, 2, 2, 16, 32, 4, 23, [None, 16]),
        # tests/test_kernel.py:137-143 (L=32) and :95-104 (T=7, ragged chunks)
        kernel_case("t_b1_h1_t4_d8_l32", 1, 1, 1, 4, 8, 32, 24, [None, 2]),
        kernel_case("t_b1_h1_t7_d8_l2", 1, 1, 1, 7, 8, 2, 25, [None, 1, 2, 3, 4, 7, 16]),
        # GQA G=4, ragged T, d=64 / d=128, several L
        kernel_case("g_b1_h8x2_t37_d64_l3", 1, 8, 2, 37, 64, 3, 26, [None, 16]),
        kernel_case("g_b1_h2x2_t45_d128_l5", 1, 2, 2, 45, 128, 5, 27, [None, 64]),
        kernel_case("g_b1_h8x1_t24_d128_l12", 1, 8, 1, 24, 128, 12, 28, [None, 64]),
        kernel_case("g_b1_h16x2_t12_d64_l48", 1, 16, 2, 12, 64, 48, 29, [None, 8]),
        # custom scale
        kernel_case("s_b1_h4x4_t19_d32_l2_scale", 1, 4, 4, 19, 32, 2, 30, [None, 5], scale=0.3),
        # oversize depth buffer: only rows [0, T*L) are addressed; unchunked form raises
        kernel_case("o_b1_h4x2_t20_d64_l4_extra16", 1, 4, 2, 20, 64, 4, 31, [None, 8], extra_rows=16),
        # gradients (torch autograd through the reference, fp64)
        grad_case("grad_b1_h4x2_t32_d64_l8", 1, 4, 2, 32, 64, 8, 40, 8),
        grad_case("grad_b2_h2x2_t16_d32_l4", 2, 2, 2, 16, 32, 4, 41, None),
        grad_case("grad_b1_h8x2_t20_d64_l3_extra8", 1, 8, 2, 20, 64, 3, 42, 16, extra_rows=8),
        grad_case("grad_b1_h16x2_t12_d64_l48", 1, 16, 2, 12, 64, 48, 43, None),
        grad_case("grad_b1_h4x1_t9_d16_l5_scale", 1, 4, 1, 9, 16, 5, 44, 4, scale=0.4),
        module_case(),
        model_case(True),
        model_case(False),
        model_grad_case(True),
        model_grad_case(False),
        cache_case(),
    ]
    for name, arrays, meta in cases:
        meta["torch"] = torch.__version__
        meta["source"] = ("reference moda (sahilmalik27/mixture-of-depth-attention), CPU "
                          + ("fp64 autograd" if meta["kind"] in ("grad", "model_grad") else "fp32"))
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, meta=np.array(json.dumps(meta)), **arrays)
        print(f"{name}: {os.path.getsize(path)} bytes, keys={sorted(arrays)[:8]}...")


if __name__ == "__main__":
    main()
