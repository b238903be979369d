"""MoDA configuration (field-for-field the reference's moda/config.py:7-60)."""

from dataclasses import dataclass
from typing import Optional


@dataclass
class MoDAConfig:
    """Configuration for MoDA (Mixture-of-Depths Attention).

    Attributes:
        d_model: Model dimension (D).
        num_heads: Number of query attention heads (H_q).
        num_kv_heads: Number of KV attention heads (H_k). Defaults to num_heads.
        head_dim: Per-head dimension (d). Defaults to d_model // num_heads.
        num_layers: Number of transformer layers; also the L that MoDAAttention
            passes to the kernel (moda/attention.py:90).
        chunk_size: Query chunk size (C). Kept for API parity; the fused kernel
            is chunk-aware by construction (a tile of n tokens reads n*L depth
            rows) and its result does not depend on C.
        ffn_dim: FFN intermediate dimension. Defaults to 4 * d_model.
        dropout: Attention dropout probability.
        max_seq_len: Maximum sequence length.
        use_triton: Accepted for API parity and ignored: CUDA tensors always run
            the B200 kernel.
        post_norm: Use post-norm (True) vs pre-norm (False).
        lean_depth_cache: Opt-in (not in the reference; default False keeps its
            behaviour). MoDAModel then skips the depth-cache work whose result no
            layer reads: the zero-fill of cache rows the attention never addresses,
            writes into those rows and their projections, the last layer's writes,
            and the first layer's read of an all-zero cache (computed as implicit
            zero rows instead). Outputs equal the default up to floating-point
            rounding of the first layer's softmax sum.
    """

    d_model: int = 768
    num_heads: int = 12
    num_kv_heads: Optional[int] = None
    head_dim: Optional[int] = None
    num_layers: int = 12
    chunk_size: int = 64
    ffn_dim: Optional[int] = None
    dropout: float = 0.0
    max_seq_len: int = 2048
    use_triton: bool = False
    post_norm: bool = True
    lean_depth_cache: bool = False

    def __post_init__(self):
        if self.num_kv_heads is None:
            self.num_kv_heads = self.num_heads
        if self.head_dim is None:
            self.head_dim = self.d_model // self.num_heads
        if self.ffn_dim is None:
            self.ffn_dim = 4 * self.d_model
        assert self.num_heads % self.num_kv_heads == 0, (
            f"num_heads ({self.num_heads}) must be divisible by "
            f"num_kv_heads ({self.num_kv_heads})"
        )

    @property
    def gqa_groups(self) -> int:
        """Number of query heads per KV head (G)."""
        return self.num_heads // self.num_kv_heads

    @property
    def kv_dim(self) -> int:
        """Total KV dimension: num_kv_heads * head_dim."""
        return self.num_kv_heads * self.head_dim
