"""ctypes binding of libmoda_b200.so (the C ABI declared in include/moda_b200.h).

The library is built in-tree by ``csrc/build.py`` into ``moda/_lib/``. There is
no fallback: if the library is missing or cannot be loaded, every CUDA entry
point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "_lib", "libmoda_b200.so")

# include/moda_b200.h enums
MODA_F32, MODA_BF16, MODA_F16 = 0, 1, 2
MODA_OK = 0
MODA_ERR_ARG, MODA_ERR_SHAPE, MODA_ERR_DEPTH_ROWS = -1, -2, -3
MODA_ERR_DTYPE, MODA_ERR_LAUNCH, MODA_ERR_UNSUPPORTED = -4, -5, -6
KERNEL_AUTO, KERNEL_TC, KERNEL_SIMT = 0, 1, 2

EXPORTED_SYMBOLS = ("moda_fwd", "moda_fwd_ex", "moda_fwd_lse", "moda_fwd_zero_depth",
                    "moda_fwd_plan", "moda_bwd", "moda_depth_proj_append", "moda_qkv_proj",
                    "moda_bwd_noalloc", "moda_bwd_workspace_size", "moda_depth_append",
                    "moda_last_error", "moda_device_status", "moda_version")
NOALLOC_ROWS = 1 << 20   # MODA_NOALLOC_ROWS


class ModaTensor(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p),
                ("sizes", ctypes.c_int64 * 4),
                ("strides", ctypes.c_int64 * 4)]


class MoDAUnsupported(RuntimeError):
    """The requested kernel cannot run this dtype / shape / layout (checked on the
    host before any launch)."""


class MoDADtypeError(TypeError, RuntimeError):
    """Unsupported or mixed dtypes. A TypeError, and also a RuntimeError like the one
    torch raises inside moda_attention_naive for mixed dtypes ("expected scalar type ...");
    float64, which the reference computes in, has no kernel here."""


class MoDAShapeError(ValueError, RuntimeError):
    """Inconsistent shapes. A ValueError, and also a RuntimeError like the shape
    errors moda_attention_naive raises for the same inputs (moda_naive.py:137-149)."""


_lock = threading.Lock()
_lib = None


def load():
    """Load (once) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"libmoda_b200.so not found at {LIB_PATH}; build it with "
                "`python mixture-of-depth-attention_b200/csrc/build.py`")
        lib = ctypes.CDLL(LIB_PATH)
        T = ctypes.POINTER(ModaTensor)
        i, f, vp = ctypes.c_int, ctypes.c_float, ctypes.c_void_p
        lib.moda_fwd.argtypes = [T, T, T, T, T, T, i, f, i, i, vp]
        lib.moda_fwd.restype = i
        lib.moda_fwd_ex.argtypes = [T, T, T, T, T, T, i, f, i, i, i, vp]
        lib.moda_fwd_ex.restype = i
        lib.moda_fwd_lse.argtypes = [T, T, T, T, T, T, vp, i, f, i, i, i, vp]
        lib.moda_fwd_lse.restype = i
        lib.moda_fwd_zero_depth.argtypes = [T, T, T, T, vp, i, f, i, i, vp]
        lib.moda_fwd_zero_depth.restype = i
        i64 = ctypes.c_int64
        lib.moda_bwd_workspace_size.argtypes = [i64, i64, i64]
        lib.moda_bwd_workspace_size.restype = i64
        lib.moda_bwd.argtypes = [T] * 7 + [vp] + [T] * 5 + [vp, i64, i, f, i, vp]
        lib.moda_bwd.restype = i
        lib.moda_bwd_noalloc.argtypes = [T] * 7 + [vp] + [T] * 5 + [i, f, i, vp]
        lib.moda_bwd_noalloc.restype = i
        lib.moda_fwd_plan.argtypes = [T, T, T, T, T, T, i, i, i]
        lib.moda_fwd_plan.restype = i
        lib.moda_depth_append.argtypes = [T, T, T, T, i, i, i, i, vp]
        lib.moda_depth_append.restype = i
        lib.moda_depth_proj_append.argtypes = [T, T, T, T, i, i, i, i, vp]
        lib.moda_depth_proj_append.restype = i
        lib.moda_qkv_proj.argtypes = [T, T, T, T, T, i, vp]
        lib.moda_qkv_proj.restype = i
        lib.moda_last_error.argtypes = []
        lib.moda_last_error.restype = ctypes.c_char_p
        lib.moda_device_status.argtypes = [vp]
        lib.moda_device_status.restype = i
        lib.moda_version.argtypes = []
        lib.moda_version.restype = i
        _lib = lib
        return lib


def describe(ptr: int, sizes, strides) -> ModaTensor:
    t = ModaTensor()
    t.ptr = ctypes.c_void_p(ptr)
    for j in range(4):
        t.sizes[j] = int(sizes[j])
        t.strides[j] = int(strides[j])
    return t


def check(code: int, what: str) -> None:
    """Map a ModaStatus to the Python exception the reference would raise."""
    if code >= 0:
        return
    msg = f"{what}: {load().moda_last_error().decode(errors='replace')}"
    if code in (MODA_ERR_SHAPE, MODA_ERR_DEPTH_ROWS):
        raise MoDAShapeError(msg)
    if code == MODA_ERR_ARG:
        raise ValueError(msg)
    if code == MODA_ERR_DTYPE:
        raise MoDADtypeError(msg)
    if code == MODA_ERR_UNSUPPORTED:
        raise MoDAUnsupported(msg)
    raise RuntimeError(msg)
