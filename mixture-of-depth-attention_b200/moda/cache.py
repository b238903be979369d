"""Depth KV cache with the reference layout (moda/cache.py:8-95).

Token t's depth entries occupy rows [t*L, (t+1)*L) of
k_cache/v_cache [B, H_k, max_seq_len*L, d]; row t*L + l holds layer l. The
write is one fused CUDA launch for k and v (``moda_depth_append``) instead of
two strided slice copies (cache.py:73-74).
"""

from typing import Optional

import torch
from torch import Tensor

from .kernels.moda_cuda import depth_append, depth_append_autograd, depth_proj_append


class DepthKVCache:
    """Depth KV cache shared by all layers of one forward pass.

    Same constructor, ``write``, ``read`` and ``reset`` as the reference. The
    buffers are zero-initialised like the reference's (cache.py:38-47), so
    unwritten slots read as zeros.

    ``zero_prefix_rows`` (keyword-only, not in the reference): zero only rows
    [0, zero_prefix_rows) of each (batch, head) and leave the rest uninitialised,
    for a caller that never reads unwritten rows past that prefix.
    """

    def __init__(self, batch_size: int, max_seq_len: int, num_layers: int, num_kv_heads: int,
                 head_dim: int, device: Optional[torch.device] = None,
                 dtype: Optional[torch.dtype] = None, *,
                 zero_prefix_rows: Optional[int] = None):
        self.batch_size = batch_size
        self.max_seq_len = max_seq_len
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        total_depth = max_seq_len * num_layers
        shape = (batch_size, num_kv_heads, total_depth, head_dim)
        if zero_prefix_rows is None:
            self.k_cache = torch.zeros(shape, device=device, dtype=dtype)
            self.v_cache = torch.zeros(shape, device=device, dtype=dtype)
        else:
            self.k_cache = torch.empty(shape, device=device, dtype=dtype)
            self.v_cache = torch.empty(shape, device=device, dtype=dtype)
            n = max(0, min(int(zero_prefix_rows), total_depth))
            for buf in (self.k_cache, self.v_cache):
                if n == 0:
                    continue
                if batch_size * num_kv_heads <= 64:
                    # one contiguous run per (batch, head): the fill's fast path
                    for b in range(batch_size):
                        for h in range(num_kv_heads):
                            buf[b, h, :n].zero_()
                else:
                    buf[:, :, :n].zero_()
        self._layer_count = 0
        self._seq_len = 0
        self._written = False  # any write since construction / reset

    def write(self, layer_idx: int, k_depth: Tensor, v_depth: Tensor,
              seq_len: Optional[int] = None):
        """Write layer ``layer_idx``'s depth KV: row t*L + layer_idx <- token t.

        Args:
            layer_idx: the writing layer's slot, 0 <= layer_idx < num_layers.
            k_depth: [B, H_k, T, d] depth keys (any strides).
            v_depth: [B, H_k, T, d] depth values.
            seq_len: tokens to write; None writes all k_depth.shape[2] of them.
        """
        T = seq_len or k_depth.shape[2]
        self._seq_len = max(self._seq_len, T)
        self._written = True
        if torch.is_grad_enabled() and (k_depth.requires_grad or v_depth.requires_grad or
                                        self.k_cache.requires_grad or
                                        self.v_cache.requires_grad):
            # training: the write is part of the graph, as the reference's slice
            # assignment is (gradients reach k_depth / v_depth and their projections)
            self.k_cache, self.v_cache = depth_append_autograd(
                self.k_cache, self.v_cache, layer_idx, k_depth, v_depth, self.num_layers, T)
        else:
            depth_append(self.k_cache, self.v_cache, layer_idx, k_depth, v_depth,
                         self.num_layers, T)

    def write_projected(self, layer_idx: int, x: Tensor, w_kv: Tensor,
                        seq_len: Optional[int] = None):
        """``write(layer_idx, x @ W_k^T, x @ W_v^T)`` as one kernel: the projection GEMM
        stores its tiles straight into the cache rows (not in the reference).

        x: [B, T, D]; w_kv: [2*H_k*d, D] = cat(W_k, W_v) (nn.Linear weight layout).
        No autograd. Raises ``MoDAUnsupported`` before any work for layouts the fused
        kernel does not take (fp32, head_dim not a multiple of 32, ...).
        """
        T = seq_len or x.shape[1]
        depth_proj_append(x, w_kv, self.k_cache, self.v_cache, layer_idx, self.num_layers, T)
        self._seq_len = max(self._seq_len, T)
        self._written = True

    def read(self, seq_len: Optional[int] = None) -> tuple[Tensor, Tensor]:
        """Views [B, H_k, T*L, d] of the first T tokens' depth rows (cache.py:76-88)."""
        T = seq_len or self._seq_len
        total = T * self.num_layers
        return self.k_cache[:, :, :total], self.v_cache[:, :, :total]

    def reset(self):
        """Clear the cache."""
        self.k_cache.zero_()
        self.v_cache.zero_()
        self._layer_count = 0
        self._seq_len = 0
        self._written = False
