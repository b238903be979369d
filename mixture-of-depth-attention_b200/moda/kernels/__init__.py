"""MoDA kernels for B200 (reference registry: moda/kernels/__init__.py:1-12).

``moda_attention_cuda`` has the signature of the reference's
``moda_attention_naive`` / ``moda_attention_triton``. The reference's naive
PyTorch function is its test oracle and is not part of this package.
"""

from .moda_cuda import (moda_attention_cuda, moda_attention_zero_depth, moda_backward,
                        moda_forward_lse, depth_append, device_status, moda_plan)

HAS_CUDA_KERNEL = True

__all__ = ["moda_attention_cuda", "moda_attention_zero_depth", "moda_forward_lse", "moda_backward", "depth_append",
           "device_status", "moda_plan", "HAS_CUDA_KERNEL"]
