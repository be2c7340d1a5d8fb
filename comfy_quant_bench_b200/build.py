"""Build libcq_b200.so in-tree with nvcc for sm_100a (one translation unit: csrc/libcq.cu).

    python -m comfy_quant_bench_b200.build [--verbose]

The CUDA runtime is linked statically, so the library depends only on the NVIDIA driver; it shares the
process's primary context (and therefore torch's device memory and streams) through the driver.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
SRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libcq_b200.so")
SOURCES = ["libcq.cu", "rotquant.cu", "gemm_sm100.cu", "gemm_pair.cu", "gemv.cu", "dit.cu", "selftest.cu", "capi.cu", "noalloc.cu", "kernels.cuh",
           "cq_common.cuh"]
HEADER = os.path.join(ROOT, "include", "cq_b200.h")


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(SRC, s) for s in SOURCES] + [HEADER]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB
    cmd = [nvcc_path(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "--expt-relaxed-constexpr", "-shared", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
           "-Xptxas", "-v" if verbose else "-O3", "-o", LIB + ".tmp", os.path.join(SRC, "libcq.cu")]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode})")
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
