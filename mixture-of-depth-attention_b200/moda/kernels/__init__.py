"""MoDA kernels for B200 (reference registry: moda/kernels/__init__.py:1-12).

``moda_attention_cuda`` has the signature of the reference's
``moda_attention_naive`` / ``moda_attention_triton``. The reference's names are
kept so its import lines work unchanged:

* ``moda_attention_naive`` (also at ``moda.kernels.moda_naive``) is the fused CUDA
  kernel under the reference's name (see ``moda_naive.py`` for what differs from the
  reference's PyTorch definition: no CPU path).
* ``HAS_TRITON`` is ``False`` and ``moda_attention_triton`` is not exported: this
  package has no Triton path, which is how the reference's registry looks when Triton
  is missing (its ``try``/``except ImportError`` branch).
"""

from .moda_cuda import (moda_attention_cuda, moda_attention_zero_depth, moda_backward,
                        moda_forward_lse, depth_append, device_status, moda_plan)
from .moda_naive import moda_attention_naive

HAS_CUDA_KERNEL = True
HAS_TRITON = False

__all__ = ["moda_attention_cuda", "moda_attention_naive", "moda_attention_zero_depth",
           "moda_forward_lse", "moda_backward", "depth_append", "device_status", "moda_plan",
           "HAS_CUDA_KERNEL", "HAS_TRITON"]
