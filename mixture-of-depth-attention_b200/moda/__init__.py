"""MoDA (Mixture-of-Depths Attention) on NVIDIA B200.

Drop-in for the public API of sahilmalik27/mixture-of-depth-attention
(moda/__init__.py:7-26): MoDAConfig, DepthKVCache, MoDAAttention,
MoDATransformerBlock, MoDAModel, plus the CUDA kernel entry point
``moda_attention_cuda`` (same signature as moda_attention_naive).
"""

from .config import MoDAConfig
from .cache import DepthKVCache
from .attention import MoDAAttention
from .model import MoDATransformerBlock, MoDAModel
from .kernels import moda_attention_cuda

__all__ = [
    "MoDAConfig",
    "DepthKVCache",
    "MoDAAttention",
    "MoDATransformerBlock",
    "MoDAModel",
    "moda_attention_cuda",
]
