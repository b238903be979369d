"""MoDAAttention with the B200 fused kernel (reference: moda/attention.py:16-116).

Same parameters (q_proj, k_proj, v_proj, o_proj, k_depth_proj, v_depth_proj),
same forward signature and outputs. Every attention call -- with depth
(attention.py:85-93) or without (attention.py:94-96, 104-116) -- runs
``moda_attention_cuda``; without depth it is the same kernel with L = 0, i.e.
plain causal attention with in-kernel GQA.
"""

from typing import Optional

import torch
import torch.nn as nn
from torch import Tensor

from .config import MoDAConfig
from .kernels._lib import MoDAUnsupported
from .kernels.moda_cuda import moda_attention_cuda, moda_attention_zero_depth, qkv_proj


class MoDAAttention(nn.Module):
    """MoDA attention layer (the reference's module API, moda/attention.py:16-116).

    Attends to the causal sequence KV of this layer and to the depth KV that
    preceding layers wrote for the same token, in one softmax.
    """

    def __init__(self, config: MoDAConfig):
        super().__init__()
        self.config = config
        self.num_heads = config.num_heads
        self.num_kv_heads = config.num_kv_heads
        self.head_dim = config.head_dim
        self.num_layers = config.num_layers
        self.scale = config.head_dim ** -0.5
        self.q_proj = nn.Linear(config.d_model, config.num_heads * config.head_dim, bias=False)
        self.k_proj = nn.Linear(config.d_model, config.num_kv_heads * config.head_dim, bias=False)
        self.v_proj = nn.Linear(config.d_model, config.num_kv_heads * config.head_dim, bias=False)
        self.o_proj = nn.Linear(config.num_heads * config.head_dim, config.d_model, bias=False)
        self.k_depth_proj = nn.Linear(config.d_model, config.num_kv_heads * config.head_dim,
                                      bias=False)
        self.v_depth_proj = nn.Linear(config.d_model, config.num_kv_heads * config.head_dim,
                                      bias=False)
        self.use_triton = False  # kept for API parity; there is one CUDA path
        self.dropout = nn.Dropout(config.dropout) if config.dropout > 0 else nn.Identity()
        # cat(W_q, W_k, W_v) for the fused projection (one extra copy of the three weights,
        # (H_q + 2*H_k)*d*D elements), the weights' (pointer, version) it was built from,
        # and whether the fused kernel takes this module's shapes (found on first use)
        self._w_qkv = None
        self._w_qkv_key = None
        self._qkv_fused_ok = None

    def _fused_qkv_weight(self) -> Tensor:
        ws = (self.q_proj.weight, self.k_proj.weight, self.v_proj.weight)
        key = tuple((w.data_ptr(), w._version, w.dtype, w.device) for w in ws)
        if self._w_qkv is None or self._w_qkv_key != key:
            self._w_qkv = torch.cat([w.detach() for w in ws], dim=0)
            self._w_qkv_key = key
        return self._w_qkv

    def _project_qkv(self, x: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        """Q, K, V as [B, H, T, d]. Without autograd: one fused GEMM (moda_qkv_proj)
        writing the head-major layout; otherwise (or where that kernel does not take the
        shape) the three nn.Linear of the reference, viewed as transposes (same values)."""
        B, T, _ = x.shape
        H_q, H_k, d = self.num_heads, self.num_kv_heads, self.head_dim
        if (not torch.is_grad_enabled() and x.is_cuda and self._qkv_fused_ok is not False
                and x.dtype in (torch.bfloat16, torch.float16)):
            try:
                out = qkv_proj(x.contiguous(), self._fused_qkv_weight(), H_q, H_k, d)
                self._qkv_fused_ok = True
                return out
            except MoDAUnsupported:
                # refused on the host before any launch (e.g. d not a multiple of 32): use
                # the library GEMMs for this module from now on
                self._qkv_fused_ok = False
                self._w_qkv = None
        # [B, H, T, d] views with strides (T*H*d, d, H*d, 1): the kernel reads them in place
        Q = self.q_proj(x).view(B, T, H_q, d).transpose(1, 2)
        K = self.k_proj(x).view(B, T, H_k, d).transpose(1, 2)
        V = self.v_proj(x).view(B, T, H_k, d).transpose(1, 2)
        return Q, K, V

    def forward(self, x: Tensor, K_depth: Optional[Tensor] = None,
                V_depth: Optional[Tensor] = None, *, zero_depth_rows: int = 0,
                write_tokens: Optional[int] = None) -> tuple[Tensor, Tensor, Tensor]:
        """Forward pass.

        Args:
            x: [B, T, D] input (CUDA).
            K_depth: [B, H_k, T*L', d] depth keys from preceding layers, or None.
            V_depth: [B, H_k, T*L', d] depth values, or None.
            zero_depth_rows: keyword-only, not in the reference. With no depth
                tensors, attend to this many all-zero depth rows per token (what a
                zero-filled cache holds) without reading them.
            write_tokens: keyword-only, not in the reference. Return k_write/v_write
                for the first ``write_tokens`` tokens only (None: all T; 0: skip the
                two depth projections).

        Returns:
            (output [B, T, D], k_write [B, H_k, T', d], v_write [B, H_k, T', d]),
            T' = T unless ``write_tokens`` is given.
        """
        B, T, D = x.shape
        H_q, H_k, d = self.num_heads, self.num_kv_heads, self.head_dim
        Q, K, V = self._project_qkv(x)
        n_w = T if write_tokens is None else max(0, min(int(write_tokens), T))
        if n_w > 0:
            # projected over all T tokens: a token slice of a batched x is strided and
            # would cost a copy larger than the GEMM work it saves
            k_write = self.k_depth_proj(x).view(B, T, H_k, d).transpose(1, 2)[:, :, :n_w]
            v_write = self.v_depth_proj(x).view(B, T, H_k, d).transpose(1, 2)[:, :, :n_w]
        else:
            k_write = v_write = x.new_empty(B, H_k, 0, d)

        # Without autograd the kernel writes O straight into the [B, T, H_q, d] layout
        # o_proj reads (its output strides are free), which replaces the reference's
        # transpose + contiguous copy (attention.py:98) with nothing.
        o_bt = None if torch.is_grad_enabled() else Q.new_empty(B, T, H_q, d)
        dst = None if o_bt is None else o_bt.transpose(1, 2)
        if K_depth is not None and V_depth is not None and K_depth.shape[2] > 0 and \
                torch.is_grad_enabled():
            # The depth views alias the cache, which later layers write in place; the
            # backward must see the rows as they are now (the reference's autograd
            # keeps its own copies), so the addressed rows are snapshot here.
            rows = T * self.num_layers
            K_depth = K_depth[:, :, :rows].clone()
            V_depth = V_depth[:, :, :rows].clone()
        if K_depth is not None and V_depth is not None and K_depth.shape[2] > 0:
            out = moda_attention_cuda(Q, K, V, K_depth, V_depth, num_layers=self.num_layers,
                                      scale=self.scale, chunk_size=self.config.chunk_size,
                                      out=dst)
        elif zero_depth_rows > 0:
            out = moda_attention_zero_depth(Q, K, V, zero_depth_rows, scale=self.scale, out=dst)
        else:
            empty = Q.new_empty(B, H_k, 0, d)
            out = moda_attention_cuda(Q, K, V, empty, empty, num_layers=0, scale=self.scale,
                                      out=dst)

        if o_bt is not None:
            out = o_bt.view(B, T, H_q * d)
        else:
            out = out.transpose(1, 2).contiguous().view(B, T, H_q * d)
        out = self.o_proj(out)
        out = self.dropout(out)
        return out, k_write, v_write
