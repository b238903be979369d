"""MoDA (Mixture-of-Depths Attention) on NVIDIA B200.

Drop-in for the public API of sahilmalik27/mixture-of-depth-attention
(moda/__init__.py:7-26): MoDAConfig, DepthKVCache, MoDAAttention,
MoDATransformerBlock, MoDAModel and ``moda_attention_naive`` (here the fused CUDA
kernel under the reference's name; see ``moda.kernels.moda_naive``), plus
``moda_attention_cuda`` (the same function under this package's own name). There is
no ``moda_attention_triton``: the reference exports it only when Triton imports.
"""

from .config import MoDAConfig
from .cache import DepthKVCache
from .attention import MoDAAttention
from .model import MoDATransformerBlock, MoDAModel
from .kernels import moda_attention_cuda, moda_attention_naive

__all__ = [
    "MoDAConfig",
    "DepthKVCache",
    "MoDAAttention",
    "MoDATransformerBlock",
    "MoDAModel",
    "moda_attention_naive",
    "moda_attention_cuda",
]
