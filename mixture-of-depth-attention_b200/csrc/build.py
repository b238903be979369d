"""Build the MoDA B200 shared library in-tree with nvcc (sm_100a).

    python mixture-of-depth-attention_b200/csrc/build.py [--force] [--verbose]

Output: mixture-of-depth-attention_b200/moda/_lib/libmoda_b200.so
The library links the CUDA runtime dynamically, so inside a PyTorch process it
shares the runtime instance PyTorch already loaded.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
OUT_DIR = os.path.join(PKG, "moda", "_lib")
OUT = os.path.join(OUT_DIR, "libmoda_b200.so")
SOURCES = ["moda_abi.cu", "moda_fwd_simt.cu", "moda_fwd_tc.cu", "moda_bwd.cu", "moda_bwd_f32.cu",
           "moda_bwd_tc.cu", "moda_proj_tc.cu"]
HEADERS = ["moda_common.cuh", "moda_internal.h", os.path.join("..", "..", "include", "moda_b200.h")]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def stale() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    deps = [os.path.join(HERE, s) for s in SOURCES + HEADERS] + [os.path.abspath(__file__)]
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not stale():
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-cudart", "shared", "--expt-relaxed-constexpr", "-rdc=false",
           f"-I{os.path.join(REPO, 'include')}",
           f"-Xlinker", f"-rpath,{os.path.join(cuda_home, 'lib64')}",
           *([] if not verbose else ["-Xptxas", "-v"]),
           "-o", OUT + ".tmp", *[os.path.join(HERE, s) for s in SOURCES]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("nvcc failed building libmoda_b200.so")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
