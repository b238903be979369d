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


def live_write_tokens(seq_len: int, read_layers: int, cache_slots: int, slot: int) -> int:
    """Tokens t whose cache row t*cache_slots + slot lies in the rows
    [0, seq_len*read_layers) that MoDAAttention addresses. They are a prefix
    t < ceil((seq_len*read_layers - slot) / cache_slots), capped at seq_len."""
    rows = seq_len * read_layers - slot
    if rows <= 0:
        return 0
    return min(seq_len, -(-rows // cache_slots))


class MoDATransformerBlock(nn.Module):
    """MoDAAttention + FFN; both write depth KV (post-norm or pre-norm)."""

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

    def forward(self, x: Tensor, depth_cache: Optional[DepthKVCache] = None) -> Tensor:
        if self.config.lean_depth_cache and depth_cache is not None:
            return self._forward_lean(x, depth_cache)
        B, T, D = x.shape
        H_k = self.config.num_kv_heads
        d = self.config.head_dim
        K_depth, V_depth = None, None
        if depth_cache is not None:
            K_depth, V_depth = depth_cache.read(seq_len=T)

        if self.config.post_norm:
            attn_out, k_w, v_w = self.attn(x, K_depth, V_depth)
            x = self.norm1(x + attn_out)
            if depth_cache is not None:
                depth_cache.write(self.layer_idx * 2, k_w, v_w, seq_len=T)
            x = self.norm2(x + self.ffn(x))
            if depth_cache is not None:
                k_f = self.ffn_k_depth_proj(x).view(B, T, H_k, d).transpose(1, 2)
                v_f = self.ffn_v_depth_proj(x).view(B, T, H_k, d).transpose(1, 2)
                depth_cache.write(self.layer_idx * 2 + 1, k_f, v_f, seq_len=T)
        else:
            attn_out, k_w, v_w = self.attn(self.norm1(x), K_depth, V_depth)
            x = x + attn_out
            if depth_cache is not None:
                depth_cache.write(self.layer_idx * 2, k_w, v_w, seq_len=T)
            x = x + self.ffn(self.norm2(x))
            if depth_cache is not None:
                k_f = self.ffn_k_depth_proj(x).view(B, T, H_k, d).transpose(1, 2)
                v_f = self.ffn_v_depth_proj(x).view(B, T, H_k, d).transpose(1, 2)
                depth_cache.write(self.layer_idx * 2 + 1, k_f, v_f, seq_len=T)
        return x

    def _forward_lean(self, x: Tensor, depth_cache: DepthKVCache) -> Tensor:
        """The default forward minus cache work whose result no layer reads."""
        B, T, D = x.shape
        H_k = self.config.num_kv_heads
        d = self.config.head_dim
        n_read = self.attn.num_layers
        slots = depth_cache.num_layers
        last = self.layer_idx == self.config.num_layers - 1
        n_attn = 0 if last else live_write_tokens(T, n_read, slots, 2 * self.layer_idx)
        n_ffn = 0 if last else live_write_tokens(T, n_read, slots, 2 * self.layer_idx + 1)
        if depth_cache._written or T * slots == 0:
            K_depth, V_depth = depth_cache.read(seq_len=T)
            zero_rows = 0
        else:  # nothing written yet: every addressed row is zero
            K_depth = V_depth = None
            zero_rows = n_read

        def attend(h):
            return self.attn(h, K_depth, V_depth, zero_depth_rows=zero_rows, write_tokens=n_attn)

        def write_ffn(h):
            if n_ffn > 0:  # projected over all T tokens (a token slice would be copied)
                k_f = self.ffn_k_depth_proj(h).view(B, T, H_k, d).transpose(1, 2)
                v_f = self.ffn_v_depth_proj(h).view(B, T, H_k, d).transpose(1, 2)
                depth_cache.write(self.layer_idx * 2 + 1, k_f, v_f, seq_len=n_ffn)

        if self.config.post_norm:
            attn_out, k_w, v_w = attend(x)
            x = self.norm1(x + attn_out)
            if n_attn > 0:
                depth_cache.write(self.layer_idx * 2, k_w, v_w, seq_len=n_attn)
            x = self.norm2(x + self.ffn(x))
            write_ffn(x)
        else:
            attn_out, k_w, v_w = attend(self.norm1(x))
            x = x + attn_out
            if n_attn > 0:
                depth_cache.write(self.layer_idx * 2, k_w, v_w, seq_len=n_attn)
            x = x + self.ffn(self.norm2(x))
            write_ffn(x)
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
