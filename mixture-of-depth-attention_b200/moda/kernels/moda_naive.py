"""The reference's ``moda.kernels.moda_naive`` module path, kept for import compatibility.

The reference defines ``moda_attention_naive`` (moda/kernels/moda_naive.py:13-162) as
its PyTorch definition of MoDA attention, and its callers import it by that name
(moda/attention.py:9, experiments/train_ab.py:32, benchmarks/bench_attention.py:18,
tests/test_kernel.py:5). In this package the name resolves to the fused CUDA kernel:
the same function (one softmax over the causal keys and the token's own L depth rows,
GQA by head groups, ``scale=None`` meaning ``d**-0.5``), computed by libmoda_b200.so
on the tensors' CUDA device, with autograd. Differences a caller can see:

* CPU tensors raise ``RuntimeError``: there is no CPU path in this package. For a CPU
  reference implementation use the original package.
* A depth buffer with more rows than ``T * num_layers`` is accepted with or without
  ``chunk_size`` (only rows ``[0, T*L)`` are read, as in the reference's chunked form);
  the reference's unchunked form raises for it.
* Fewer rows than ``T * num_layers`` raise ``MoDAShapeError`` (a ``ValueError`` and a
  ``RuntimeError``) before any launch.
* Results match the reference within fp32 1e-4 relative / bf16 2e-2 absolute, not
  bit for bit.
"""

from __future__ import annotations

from typing import Optional

from torch import Tensor

from .moda_cuda import moda_attention_cuda


def moda_attention_naive(Q: Tensor, K: Tensor, V: Tensor, K_depth: Tensor, V_depth: Tensor,
                         num_layers: int, scale: Optional[float] = None,
                         chunk_size: Optional[int] = None) -> Tensor:
    """MoDA attention under the reference's name; runs the fused CUDA kernel
    (``moda_attention_cuda``). Arguments and result as moda/kernels/moda_naive.py:13-43."""
    return moda_attention_cuda(Q, K, V, K_depth, V_depth, num_layers, scale, chunk_size)


__all__ = ["moda_attention_naive"]
