"""The reference's import lines run unchanged against this package (CPU, no GPU needed).

Each statement below is copied from a reference caller (file:line given), so a user of
the reference who puts this package first on sys.path keeps their imports.
"""

import importlib
import sys

import pytest
import torch


def test_kernel_registry_names():
    # moda/attention.py:9-13
    from moda.kernels import moda_attention_naive  # noqa: F401
    from moda.kernels import HAS_TRITON
    assert HAS_TRITON is False
    # moda/kernels/__init__.py:5: __all__ starts with the naive name
    import moda.kernels as k
    assert "moda_attention_naive" in k.__all__ and "HAS_TRITON" in k.__all__
    assert "moda_attention_triton" not in k.__all__


def test_submodule_paths():
    # tests/test_kernel.py:5, tests/test_gqa.py:5, benchmarks/bench_attention.py:18
    from moda.kernels.moda_naive import moda_attention_naive
    from moda.kernels import moda_attention_naive as via_registry
    assert moda_attention_naive is via_registry
    # tests/test_kernel.py:154 and experiments/train_ab.py:34 guard this import with
    # try/except ImportError: without Triton it fails, as in the reference.
    with pytest.raises(ImportError):
        importlib.import_module("moda.kernels.moda_triton")


def test_top_level_names():
    # moda/__init__.py:7-19 and experiments/train_ab.py:28-32
    import moda
    from moda import (DepthKVCache, MoDAAttention, MoDAConfig, MoDAModel,  # noqa: F401
                      MoDATransformerBlock, moda_attention_naive)
    for name in ("MoDAConfig", "DepthKVCache", "MoDAAttention", "MoDATransformerBlock",
                 "MoDAModel", "moda_attention_naive"):
        assert name in moda.__all__, name
    assert "moda_attention_triton" not in moda.__all__
    with pytest.raises(ImportError):
        exec("from moda import moda_attention_triton", {})


def test_naive_name_has_the_reference_signature_and_no_cpu_path():
    import inspect
    from moda.kernels import moda_attention_naive
    params = list(inspect.signature(moda_attention_naive).parameters)
    assert params == ["Q", "K", "V", "K_depth", "V_depth", "num_layers", "scale", "chunk_size"]
    q = torch.zeros(1, 2, 4, 8)
    kv = torch.zeros(1, 1, 4, 8)
    kd = torch.zeros(1, 1, 8, 8)
    with pytest.raises(RuntimeError, match="no CPU path"):
        moda_attention_naive(q, kv, kv, kd, kd, 2)


def test_no_oracle_behind_the_names():
    """The names resolve to the CUDA path: nothing under oracle/ is imported by them."""
    before = set(sys.modules)
    import moda  # noqa: F401
    from moda.kernels.moda_naive import moda_attention_naive  # noqa: F401
    assert not any(m == "oracle" or m.startswith("oracle.") for m in set(sys.modules) - before)
    src = open(sys.modules["moda.kernels.moda_naive"].__file__).read()
    assert "oracle" not in src.replace("# ", "")
