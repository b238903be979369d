"""MoDA transformer block and model (reference: moda/model.py:13-158).

Unchanged structure: LayerNorm/GELU/Linear stay PyTorch; attention and the
depth-cache writes run on the B200 kernels. The cache holds 2*num_layers slots
per token (attention writes slot 2i, the FFN slot 2i+1) while MoDAAttention
addresses it with L = num_layers (moda/model.py:143-151, moda/attention.py:90);
that addressing is reproduced as is, so outputs match the reference.
"""

from typing import Optional

import torch
import torch.nn as nn
from torch import Tensor

from .config import MoDAConfig
from .attention import MoDAAttention
from .cache import DepthKVCache


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
            depth_cache = DepthKVCache(batch_size=B, max_seq_len=T,
                                       num_layers=self.config.num_layers * 2,
                                       num_kv_heads=self.config.num_kv_heads,
                                       head_dim=self.config.head_dim, device=x.device,
                                       dtype=x.dtype)
        for layer in self.layers:
            x = layer(x, depth_cache=depth_cache)
        x = self.final_norm(x)
        return self.head(x)
