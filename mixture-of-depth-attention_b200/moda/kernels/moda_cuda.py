"""B200 CUDA MoDA attention behind the reference kernel signature.

``moda_attention_cuda(Q, K, V, K_depth, V_depth, num_layers, scale=None,
chunk_size=None)`` keeps the positional/keyword order of
``moda_attention_naive`` (moda/kernels/moda_naive.py:13-22) and
``moda_attention_triton`` (moda/kernels/moda_triton.py:218-227) and computes the
same function: one softmax over the causal sequence keys and the token's own L
depth rows. The forward always runs in libmoda_b200.so (tcgen05 kernel for
bf16/f16 with d in {64,128}, CUDA-core kernel otherwise), and so does the
backward (``moda_bwd``, through ``torch.autograd``); CPU tensors raise.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor
from torch.autograd.function import once_differentiable

from . import _lib

_DTYPES = {torch.float32: _lib.MODA_F32, torch.bfloat16: _lib.MODA_BF16,
           torch.float16: _lib.MODA_F16}
_KERNELS = {"auto": _lib.KERNEL_AUTO, "tc": _lib.KERNEL_TC, "simt": _lib.KERNEL_SIMT}


def _desc(t: Tensor) -> _lib.ModaTensor:
    return _lib.describe(t.data_ptr(), t.shape, t.stride())


def _check_inputs(Q, K, V, K_depth, V_depth):
    ts = (Q, K, V, K_depth, V_depth)
    names = ("Q", "K", "V", "K_depth", "V_depth")
    for n, t in zip(names, ts):
        if not isinstance(t, Tensor):
            raise TypeError(f"{n} must be a torch.Tensor")
        if t.dim() != 4:
            raise _lib.MoDAShapeError(f"{n} must be 4-D [B, H, rows, d], got shape {tuple(t.shape)}")
        if t.device.type != "cuda":
            raise RuntimeError(
                f"moda_attention_cuda runs on CUDA tensors only ({n} is on {t.device}); "
                "there is no CPU path")
        if t.dtype not in _DTYPES:
            raise _lib.MoDADtypeError(f"{n} has unsupported dtype {t.dtype} (float32, bfloat16, float16)")
    dev, dt = Q.device, Q.dtype
    for n, t in zip(names, ts):
        if t.device != dev:
            raise RuntimeError(f"{n} is on {t.device}, Q on {dev}")
        if t.dtype != dt:
            raise _lib.MoDADtypeError(f"{n} has dtype {t.dtype}, Q has {dt}")


def _check_out(out: Tensor, Q: Tensor) -> Tensor:
    if not isinstance(out, Tensor) or out.shape != Q.shape or out.dtype != Q.dtype or \
            out.device != Q.device:
        raise _lib.MoDAShapeError("out must be a tensor with Q's shape, dtype and device")
    return out


def moda_forward_into(O: Tensor, Q: Tensor, K: Tensor, V: Tensor, K_depth: Tensor,
                      V_depth: Tensor, num_layers: int, scale: Optional[float] = None,
                      chunk_size: Optional[int] = None, kernel: str = "auto") -> Tensor:
    """Run the forward into a preallocated O [B,H_q,T,d] (any strides). Returns O."""
    _check_inputs(Q, K, V, K_depth, V_depth)
    if O.device != Q.device or O.dtype != Q.dtype or O.dim() != 4:
        raise _lib.MoDAShapeError("O must be a 4-D tensor on Q's device with Q's dtype")
    lib = _lib.load()
    stream = torch.cuda.current_stream(Q.device).cuda_stream
    with torch.cuda.device(Q.device):
        code = lib.moda_fwd_ex(_desc(Q), _desc(K), _desc(V), _desc(K_depth), _desc(V_depth),
                               _desc(O), int(num_layers), float(scale) if scale else 0.0,
                               int(chunk_size or 0), _DTYPES[Q.dtype], _KERNELS[kernel],
                               stream)
    _lib.check(code, "moda_fwd")
    return O


def moda_plan(Q, K, V, K_depth, V_depth, num_layers: int, kernel: str = "auto") -> str:
    """Which kernel a call would launch ("tc" or "simt"). Host-only; works on any device."""
    if Q.dtype not in _DTYPES:
        raise _lib.MoDADtypeError(f"Q has unsupported dtype {Q.dtype} (float32, bfloat16, float16)")
    O_shape = (Q.shape[0], Q.shape[1], Q.shape[2], Q.shape[3])
    o = _lib.describe(Q.data_ptr(), O_shape, Q.stride())
    code = _lib.load().moda_fwd_plan(_desc(Q), _desc(K), _desc(V), _desc(K_depth),
                                     _desc(V_depth), o, int(num_layers), _DTYPES[Q.dtype],
                                     _KERNELS[kernel])
    _lib.check(code, "moda_fwd_plan")
    return {_lib.KERNEL_TC: "tc", _lib.KERNEL_SIMT: "simt"}[code]


def moda_forward_lse(Q: Tensor, K: Tensor, V: Tensor, K_depth: Tensor, V_depth: Tensor,
                     num_layers: int, scale: Optional[float] = None,
                     chunk_size: Optional[int] = None, kernel: str = "auto"):
    """Forward that also returns the row log-sum-exp: (O [B,H_q,T,d], lse [B,H_q,T] fp32).

    lse[b,h,t] = log(sum over the row's keys of exp(scale * q.k)), natural log; the
    backward pass needs it.
    """
    _check_inputs(Q, K, V, K_depth, V_depth)
    O = torch.empty(Q.shape, dtype=Q.dtype, device=Q.device)
    lse = torch.empty(Q.shape[:3], dtype=torch.float32, device=Q.device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(Q.device).cuda_stream
    with torch.cuda.device(Q.device):
        code = lib.moda_fwd_lse(_desc(Q), _desc(K), _desc(V), _desc(K_depth), _desc(V_depth),
                                _desc(O), lse.data_ptr(), int(num_layers),
                                float(scale) if scale else 0.0, int(chunk_size or 0),
                                _DTYPES[Q.dtype], _KERNELS[kernel], stream)
    _lib.check(code, "moda_fwd_lse")
    return O, lse


def moda_backward(dO: Tensor, Q: Tensor, K: Tensor, V: Tensor, K_depth: Tensor,
                  V_depth: Tensor, O: Tensor, lse: Tensor, num_layers: int,
                  scale: Optional[float] = None):
    """Gradients (dQ, dK, dV, dK_depth, dV_depth) of the forward for upstream dO.

    Runs the backward kernels of libmoda_b200.so (moda_bwd); every gradient has the
    shape and dtype of its input; depth rows the forward never reads get zero.
    """
    _check_inputs(Q, K, V, K_depth, V_depth)
    for n, t in (("dO", dO), ("O", O)):
        if t.shape != Q.shape or t.dtype != Q.dtype or t.device != Q.device:
            raise _lib.MoDAShapeError(f"{n} must have Q's shape, dtype and device")
    if lse.dtype != torch.float32 or lse.shape != Q.shape[:3] or not lse.is_contiguous():
        raise _lib.MoDAShapeError("lse must be a contiguous float32 [B, H_q, T] tensor")
    # autograd may hand over an expanded (zero-stride) dO; the tensor-core path loads
    # it with TMA, which needs real 16-byte strides
    dO = dO.contiguous()
    grads = [torch.empty(t.shape, dtype=t.dtype, device=t.device) for t in (Q, K, V, K_depth, V_depth)]
    lib = _lib.load()
    nbytes = lib.moda_bwd_workspace_size(Q.shape[0], Q.shape[1], Q.shape[2])
    work = torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=Q.device)
    stream = torch.cuda.current_stream(Q.device).cuda_stream
    with torch.cuda.device(Q.device):
        code = lib.moda_bwd(_desc(Q), _desc(K), _desc(V), _desc(K_depth), _desc(V_depth),
                            _desc(O), _desc(dO), lse.data_ptr(), *[_desc(g) for g in grads],
                            work.data_ptr(), int(nbytes), int(num_layers),
                            float(scale) if scale else 0.0, _DTYPES[Q.dtype], stream)
    _lib.check(code, "moda_bwd")
    return tuple(grads)


class _MoDAFunction(torch.autograd.Function):
    """Forward and backward both run in libmoda_b200.so: the forward saves O and the
    row log-sum-exp; the backward kernels recompute the attention weights from them.
    First derivatives only: differentiating the gradients (double backward, which torch
    autograd gives the reference's moda_attention_naive) raises instead of returning
    gradients that ignore the backward's own dependence on the inputs."""

    @staticmethod
    def forward(ctx, Q, K, V, K_depth, V_depth, num_layers, scale, chunk_size, kernel):
        O, lse = moda_forward_lse(Q, K, V, K_depth, V_depth, num_layers, scale, chunk_size,
                                  kernel)
        ctx.save_for_backward(Q, K, V, K_depth, V_depth, O, lse)
        ctx.num_layers = num_layers
        ctx.scale = scale
        return O

    @staticmethod
    @once_differentiable
    def backward(ctx, dO):
        Q, K, V, Kd, Vd, O, lse = ctx.saved_tensors
        grads = moda_backward(dO, Q, K, V, Kd, Vd, O, lse, ctx.num_layers, ctx.scale)
        return (*grads, None, None, None, None)


def moda_attention_cuda(Q: Tensor, K: Tensor, V: Tensor, K_depth: Tensor, V_depth: Tensor,
                        num_layers: int, scale: Optional[float] = None,
                        chunk_size: Optional[int] = None, *, kernel: str = "auto",
                        out: Optional[Tensor] = None) -> Tensor:
    """MoDA attention: fused sequence + depth attention with one combined softmax.

    Args:
        Q: [B, H_q, T, d] queries. K, V: [B, H_k, T, d]. K_depth, V_depth:
            [B, H_k, R, d] with R >= T*num_layers; token t's depth rows are
            [t*L, (t+1)*L) (DepthKVCache layout, moda/cache.py:8-20).
        num_layers: L, depth rows per token (0 = plain causal attention).
        scale: softmax scale, default d**-0.5 (moda_naive.py:48-49).
        chunk_size: accepted for signature parity; the result does not depend on it.
        kernel: "auto" (default), "tc" or "simt" to force a kernel.
        out: keyword-only, not in the reference. Destination [B, H_q, T, d] of Q's
            dtype and device, any strides (e.g. the transposed view of a
            [B, T, H_q, d] buffer, the layout the output projection reads). Only
            without autograd.

    Returns:
        [B, H_q, T, d] tensor of Q's dtype: ``out``, or a new contiguous tensor.
    """
    if kernel not in _KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}")
    if num_layers is None or int(num_layers) < 0:
        raise ValueError(f"num_layers must be a non-negative int, got {num_layers}")
    _check_inputs(Q, K, V, K_depth, V_depth)
    needs_grad = torch.is_grad_enabled() and any(
        t.requires_grad for t in (Q, K, V, K_depth, V_depth))
    if needs_grad:
        if out is not None:
            raise ValueError("out= is only supported when no gradient is needed")
        return _MoDAFunction.apply(Q, K, V, K_depth, V_depth, int(num_layers), scale,
                                   chunk_size, kernel)
    O = torch.empty(Q.shape, dtype=Q.dtype, device=Q.device) if out is None else _check_out(out, Q)
    return moda_forward_into(O, Q, K, V, K_depth, V_depth, int(num_layers), scale, chunk_size,
                             kernel)


def moda_forward_zero_depth(Q: Tensor, K: Tensor, V: Tensor, zero_rows: int,
                            scale: Optional[float] = None, kernel: str = "auto",
                            out: Optional[Tensor] = None):
    """Forward whose depth part is ``zero_rows`` all-zero rows per token, none read.

    Equals ``moda_forward_lse`` with K_depth = V_depth = zeros [B,H_k,T*zero_rows,d]
    and num_layers = zero_rows, up to rounding. Returns (O, lse); O is ``out`` (any
    strides) when given.
    """
    empty = Q.new_empty(Q.shape[0], K.shape[1], 0, Q.shape[3])
    _check_inputs(Q, K, V, empty, empty)
    if int(zero_rows) < 0:
        raise ValueError(f"zero_rows must be >= 0, got {zero_rows}")
    O = torch.empty(Q.shape, dtype=Q.dtype, device=Q.device) if out is None else _check_out(out, Q)
    lse = torch.empty(Q.shape[:3], dtype=torch.float32, device=Q.device)
    lib = _lib.load()
    stream = torch.cuda.current_stream(Q.device).cuda_stream
    with torch.cuda.device(Q.device):
        code = lib.moda_fwd_zero_depth(_desc(Q), _desc(K), _desc(V), _desc(O), lse.data_ptr(),
                                       int(zero_rows), float(scale) if scale else 0.0,
                                       _DTYPES[Q.dtype], _KERNELS[kernel], stream)
    _lib.check(code, "moda_fwd_zero_depth")
    return O, lse


class _ZeroDepthFunction(torch.autograd.Function):
    """Autograd for the implicit-zero depth forward. The zero rows have no tensor and
    contribute nothing to dQ (their keys are 0), so the backward is the L = 0 backward
    with this forward's log-sum-exp, which already counts them."""

    @staticmethod
    def forward(ctx, Q, K, V, zero_rows, scale, kernel):
        O, lse = moda_forward_zero_depth(Q, K, V, zero_rows, scale, kernel)
        ctx.save_for_backward(Q, K, V, O, lse)
        ctx.scale = scale
        return O

    @staticmethod
    @once_differentiable
    def backward(ctx, dO):
        Q, K, V, O, lse = ctx.saved_tensors
        empty = Q.new_empty(Q.shape[0], K.shape[1], 0, Q.shape[3])
        dQ, dK, dV, _, _ = moda_backward(dO, Q, K, V, empty, empty, O, lse, 0, ctx.scale)
        return dQ, dK, dV, None, None, None


def moda_attention_zero_depth(Q: Tensor, K: Tensor, V: Tensor, zero_rows: int,
                              scale: Optional[float] = None, *, kernel: str = "auto",
                              out: Optional[Tensor] = None) -> Tensor:
    """``moda_attention_cuda`` over an all-zero depth part of ``zero_rows`` rows per
    token, without the depth tensors: each row's softmax also holds ``zero_rows`` keys
    of score 0 with value 0. What the first layer of ``MoDAModel`` computes from its
    freshly zero-filled cache (moda/model.py:143-151, moda/cache.py:40-47).
    ``out`` as in ``moda_attention_cuda``."""
    if kernel not in _KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}")
    needs_grad = torch.is_grad_enabled() and any(t.requires_grad for t in (Q, K, V))
    if needs_grad:
        if out is not None:
            raise ValueError("out= is only supported when no gradient is needed")
        return _ZeroDepthFunction.apply(Q, K, V, int(zero_rows), scale, kernel)
    return moda_forward_zero_depth(Q, K, V, zero_rows, scale, kernel, out)[0]


def depth_append(k_cache: Tensor, v_cache: Tensor, layer_idx: int, k: Tensor, v: Tensor,
                 num_layers: int, seq_len: int) -> None:
    """k_cache[:, :, t*L + layer_idx] = k[:, :, t] for t < seq_len (and v); one CUDA launch."""
    for n, t in (("k_cache", k_cache), ("v_cache", v_cache), ("k", k), ("v", v)):
        if t.device.type != "cuda":
            raise RuntimeError(f"depth append runs on CUDA tensors only ({n} is on {t.device})")
        if t.dim() != 4:
            raise _lib.MoDAShapeError(f"{n} must be 4-D")
        if t.dtype != k_cache.dtype:
            raise _lib.MoDADtypeError(f"{n} has dtype {t.dtype}, cache has {k_cache.dtype}")
        if t.device != k_cache.device:
            raise RuntimeError(f"{n} is on {t.device}, cache on {k_cache.device}")
    if k_cache.dtype not in _DTYPES:
        raise _lib.MoDADtypeError(f"unsupported cache dtype {k_cache.dtype}")
    lib = _lib.load()
    stream = torch.cuda.current_stream(k_cache.device).cuda_stream
    with torch.cuda.device(k_cache.device):
        code = lib.moda_depth_append(_desc(k), _desc(v), _desc(k_cache), _desc(v_cache),
                                     int(layer_idx), int(num_layers), int(seq_len),
                                     _DTYPES[k_cache.dtype], stream)
    _lib.check(code, "moda_depth_append")


def depth_proj_append(x: Tensor, w_kv: Tensor, k_cache: Tensor, v_cache: Tensor, layer_idx: int,
                      num_layers: int, seq_len: int) -> None:
    """k/v depth projections of ``x`` stored straight into the cache rows (one kernel).

    x [B, T, D]; w_kv [2*H_k*d, D] = cat(W_k_depth, W_v_depth); caches [B, H_k, R, d].
    For t < seq_len: k_cache[:, h, t*L + layer_idx] = (x[:, t] @ W_k_depth.T)[h*d:(h+1)*d],
    and the same for v. No autograd. Raises ``MoDAUnsupported`` (before any launch) for
    fp32, d not a multiple of 32, D not a multiple of 8 or unaligned layouts.
    """
    for n, t in (("x", x), ("w_kv", w_kv), ("k_cache", k_cache), ("v_cache", v_cache)):
        if t.device.type != "cuda":
            raise RuntimeError(f"depth projection runs on CUDA tensors only ({n} is on {t.device})")
        if t.device != x.device:
            raise RuntimeError(f"{n} is on {t.device}, x on {x.device}")
        if t.dtype != x.dtype:
            raise _lib.MoDADtypeError(f"{n} has dtype {t.dtype}, x has {x.dtype}")
    if x.dim() != 3 or w_kv.dim() != 2:
        raise _lib.MoDAShapeError("x must be [B, T, D] and w_kv [2*H_k*d, D]")
    if x.dtype not in _DTYPES:
        raise _lib.MoDADtypeError(f"unsupported dtype {x.dtype}")
    lib = _lib.load()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        code = lib.moda_depth_proj_append(_desc(x.unsqueeze(1)), _desc(w_kv[None, None]),
                                          _desc(k_cache), _desc(v_cache), int(layer_idx),
                                          int(num_layers), int(seq_len), _DTYPES[x.dtype],
                                          stream)
    _lib.check(code, "moda_depth_proj_append")


def qkv_proj(x: Tensor, w_qkv: Tensor, num_heads: int, num_kv_heads: int,
             head_dim: int) -> tuple[Tensor, Tensor, Tensor]:
    """The attention's three input projections as one kernel (moda/attention.py:77-79).

    x [B, T, D]; w_qkv [(H_q + 2*H_k)*d, D] = cat(W_q, W_k, W_v). Returns Q [B, H_q, T, d],
    K, V [B, H_k, T, d], contiguous (the layout the attention kernel reads; the
    reference's transposed views hold the same values). No autograd. Raises
    ``MoDAUnsupported`` (before any launch) for fp32, d not a multiple of 32, D not a
    multiple of 8 or unaligned layouts.
    """
    for n, t in (("x", x), ("w_qkv", w_qkv)):
        if t.device.type != "cuda":
            raise RuntimeError(f"QKV projection runs on CUDA tensors only ({n} is on {t.device})")
        if t.device != x.device:
            raise RuntimeError(f"{n} is on {t.device}, x on {x.device}")
        if t.dtype != x.dtype:
            raise _lib.MoDADtypeError(f"{n} has dtype {t.dtype}, x has {x.dtype}")
    if x.dim() != 3 or w_qkv.dim() != 2:
        raise _lib.MoDAShapeError("x must be [B, T, D] and w_qkv [(H_q+2*H_k)*d, D]")
    if x.dtype not in _DTYPES:
        raise _lib.MoDADtypeError(f"unsupported dtype {x.dtype}")
    B, T, _ = x.shape
    Q = x.new_empty(B, num_heads, T, head_dim)
    K = x.new_empty(B, num_kv_heads, T, head_dim)
    V = x.new_empty(B, num_kv_heads, T, head_dim)
    lib = _lib.load()
    stream = torch.cuda.current_stream(x.device).cuda_stream
    with torch.cuda.device(x.device):
        code = lib.moda_qkv_proj(_desc(x.unsqueeze(1)), _desc(w_qkv[None, None]), _desc(Q),
                                 _desc(K), _desc(V), _DTYPES[x.dtype], stream)
    _lib.check(code, "moda_qkv_proj")
    return Q, K, V


class _DepthAppendFunction(torch.autograd.Function):
    """In-place depth append that autograd sees, like the reference's strided slice
    assignment into the cache (moda/cache.py:73-74, recorded by torch as a copy into
    slices): the rows written get their gradient from the cache's gradient, and the
    cache's earlier content gets the rest. The forward is the CUDA append kernel."""

    @staticmethod
    def forward(ctx, k_cache, v_cache, k, v, layer_idx, num_layers, seq_len):
        depth_append(k_cache, v_cache, layer_idx, k, v, num_layers, seq_len)
        ctx.mark_dirty(k_cache, v_cache)
        ctx.meta = (layer_idx, num_layers, seq_len, k.shape, v.shape)
        return k_cache, v_cache

    @staticmethod
    def backward(ctx, g_kc, g_vc):
        slot, L, T, k_shape, v_shape = ctx.meta

        def split(g, src_shape):
            if g is None:
                return None, None
            g_src = g.new_zeros(src_shape)
            g_src[:, :, :T] = g[:, :, slot:T * L:L]
            g_prev = g.clone()
            g_prev[:, :, slot:T * L:L] = 0  # overwritten rows: nothing flows further back
            return g_prev, g_src

        gk_prev, gk = split(g_kc, k_shape)
        gv_prev, gv = split(g_vc, v_shape)
        return gk_prev, gv_prev, gk, gv, None, None, None


def depth_append_autograd(k_cache: Tensor, v_cache: Tensor, layer_idx: int, k: Tensor,
                          v: Tensor, num_layers: int, seq_len: int):
    """``depth_append`` recorded by autograd; returns the (same, now dirty) caches."""
    return _DepthAppendFunction.apply(k_cache, v_cache, k, v, int(layer_idx), int(num_layers),
                                      int(seq_len))


def device_status(device=None) -> int:
    """Read and clear the kernels' timeout status word of ``device`` (default: the current
    device); 0 = no bounded wait expired."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    stream = torch.cuda.current_stream(device).cuda_stream
    with torch.cuda.device(device):
        code = _lib.load().moda_device_status(stream)
    _lib.check(code, "moda_device_status")
    return code
