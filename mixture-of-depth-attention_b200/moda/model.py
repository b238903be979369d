"""MoDA transformer block and model (reference: moda/model.py:13-158).

Unchanged structure: LayerNorm/GELU/Linear stay PyTorch; attention and the
depth-cache writes run on the B200 kernels. The cache holds 2*num_layers slots
per token (attention writes slot 2i, the FFN slot 2i+1) while MoDAAttention
addresses it with L = num_layers (moda/model.py:143-151, moda/attention.py:90);
that addressing is reproduced as is, so outputs match the reference.

With ``config.lean_depth_cache`` (opt-in, off by default) the model skips the
cache work no layer reads, given that addressing: the attention reads rows
[0, T*num_layers) of a buffer of T*2*num_layers rows per (batch, head), so only
that prefix is zero-filled, writes land only in it (``live_write_tokens``), the
last layer writes nothing, and the first layer, which would read nothing but
zeros, attends to implicit zero rows instead of reading them.
"""

from typing import Optional

import torch
import torch.nn as nn
from torch import Tensor

from .config import MoDAConfig
from .attention import MoDAAttention
from .cache import DepthKVCache
from .kernels._lib import MoDAUnsupported


def live_write_tokens(seq_len: int, read_layers: int, cache_slots: int, slot: int) -> int:
    """Tokens t whose cache row t*cache_slots + slot lies in the rows
    [0, seq_len*read_layers) that MoDAAttention addresses. They are a prefix
    t < ceil((seq_len*read_layers - slot) / cache_slots), capped at seq_len."""
    rows = seq_len * read_layers - slot
    if rows <= 0:
        return 0
    return min(seq_len, -(-rows // cache_slots))


class MoDATransformerBlock(nn.Module):
    """MoDAAttention + FFN; both write depth KV (post-norm or pre-norm).

    Without autograd and for 16-bit weights, each depth write -- the attention's (slot
    2i) and the FFN's (slot 2i+1) -- is one fused kernel: the k/v depth projections with
    the cache append in the GEMM epilogue (``DepthKVCache.write_projected``). The
    attention's write still lands after its own attention, as in the reference: with
    the 2N-slot addressing, layer i's attention reads slot 2i for half of the tokens,
    and those rows must still be zero then.
    """

    def __init__(self, config: MoDAConfig, layer_idx: int):
        super().__init__()
        self.config = config
        self.layer_idx = layer_idx
        self.attn = MoDAAttention(config)
        self.ffn = nn.Sequential(
            nn.Linear(config.d_model, config.ffn_dim, bias=False),
            nn.GELU(),
            nn.Linear(config.ffn_dim, config.d_model, bias=False),
        )
        self.norm1 = nn.LayerNorm(config.d_model)
        self.norm2 = nn.LayerNorm(config.d_model)
        self.ffn_k_depth_proj = nn.Linear(config.d_model, config.num_kv_heads * config.head_dim,
                                          bias=False)
        self.ffn_v_depth_proj = nn.Linear(config.d_model, config.num_kv_heads * config.head_dim,
                                          bias=False)
        self._kv_weights = {}  # concatenated [W_k; W_v] per projection pair, by weight version

    def _kv_weight(self, k_lin: nn.Linear, v_lin: nn.Linear) -> Tensor:
        wk, wv = k_lin.weight, v_lin.weight
        key = (id(k_lin), wk.data_ptr(), wk._version, wv.data_ptr(), wv._version, wk.dtype)
        hit = self._kv_weights.get(id(k_lin))
        if hit is None or hit[0] != key:
            hit = (key, torch.cat([wk, wv]).detach())
            self._kv_weights[id(k_lin)] = hit
        return hit[1]

    def _write(self, cache: Optional[DepthKVCache], slot: int, h: Tensor,
               k_w: Optional[Tensor], v_w: Optional[Tensor], n: int, fuse: bool,
               k_lin: nn.Linear, v_lin: nn.Linear) -> None:
        """Cache slot ``slot`` <- depth projections of h for tokens t < n."""
        if cache is None or n <= 0:
            return
        if fuse:
            try:
                cache.write_projected(slot, h, self._kv_weight(k_lin, v_lin), seq_len=n)
                return
            except MoDAUnsupported:
                pass  # layout the fused kernel does not take: project, then append
        B, T, _ = h.shape
        H_k, d = self.config.num_kv_heads, self.config.head_dim
        if k_w is None or k_w.shape[2] < n:
            k_w = k_lin(h).view(B, T, H_k, d).transpose(1, 2)
            v_w = v_lin(h).view(B, T, H_k, d).transpose(1, 2)
        cache.write(slot, k_w, v_w, seq_len=n)

    def forward(self, x: Tensor, depth_cache: Optional[DepthKVCache] = None) -> Tensor:
        B, T, D = x.shape
        i = self.layer_idx
        K_depth, V_depth = None, None
        zero_rows = 0
        n_attn = n_ffn = T
        if depth_cache is not None:
            if self.config.lean_depth_cache:
                # the cache work no layer reads is skipped (see the module docstring)
                n_read, slots = self.attn.num_layers, depth_cache.num_layers
                last = i == self.config.num_layers - 1
                n_attn = 0 if last else live_write_tokens(T, n_read, slots, 2 * i)
                n_ffn = 0 if last else live_write_tokens(T, n_read, slots, 2 * i + 1)
            if self.config.lean_depth_cache and not depth_cache._written and \
                    T * depth_cache.num_layers > 0:
                zero_rows = self.attn.num_layers  # nothing written yet: all rows are zero
            else:
                K_depth, V_depth = depth_cache.read(seq_len=T)
        fuse = (depth_cache is not None and not torch.is_grad_enabled() and
                x.dtype in (torch.float16, torch.bfloat16))
        n_proj = 0 if fuse else (None if n_attn == T else n_attn)

        def attend(h):
            return self.attn(h, K_depth, V_depth, zero_depth_rows=zero_rows, write_tokens=n_proj)

        if self.config.post_norm:
            attn_out, k_w, v_w = attend(x)
            h_attn = x
            x = self.norm1(x + attn_out)
            self._write(depth_cache, 2 * i, h_attn, k_w, v_w, n_attn, fuse,
                        self.attn.k_depth_proj, self.attn.v_depth_proj)
            x = self.norm2(x + self.ffn(x))
            self._write(depth_cache, 2 * i + 1, x, None, None, n_ffn, fuse,
                        self.ffn_k_depth_proj, self.ffn_v_depth_proj)
        else:
            h_attn = self.norm1(x)
            attn_out, k_w, v_w = attend(h_attn)
            x = x + attn_out
            self._write(depth_cache, 2 * i, h_attn, k_w, v_w, n_attn, fuse,
                        self.attn.k_depth_proj, self.attn.v_depth_proj)
            x = x + self.ffn(self.norm2(x))
            self._write(depth_cache, 2 * i + 1, x, None, None, n_ffn, fuse,
                        self.ffn_k_depth_proj, self.ffn_v_depth_proj)
        return x


class MoDAModel(nn.Module):
    """Stack of MoDATransformerBlocks sharing one DepthKVCache per forward."""

    def __init__(self, config: MoDAConfig):
        super().__init__()
        self.config = config
        self.embed = nn.Embedding(config.max_seq_len, config.d_model)
        self.layers = nn.ModuleList(
            [MoDATransformerBlock(config, layer_idx=i) for i in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.d_model)
        self.head = nn.Linear(config.d_model, config.d_model, bias=False)

    def forward(self, x: Tensor, use_depth_cache: bool = True) -> Tensor:
        if x.dtype in (torch.long, torch.int):
            x = self.embed(x)
        B, T, D = x.shape
        depth_cache = None
        if use_depth_cache:
            # lean: only the rows the attention addresses need zeros
            zero_prefix = T * self.config.num_layers if self.config.lean_depth_cache else None
            depth_cache = DepthKVCache(batch_size=B, max_seq_len=T,
                                       num_layers=self.config.num_layers * 2,
                                       num_kv_heads=self.config.num_kv_heads,
                                       head_dim=self.config.head_dim, device=x.device,
                                       dtype=x.dtype, zero_prefix_rows=zero_prefix)
        for layer in self.layers:
            x = layer(x, depth_cache=depth_cache)
        x = self.final_norm(x)
        return self.head(x)
