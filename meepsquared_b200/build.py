"""Builds libmeep2b.so in the package directory with nvcc for sm_100a (B200) only.

    python -m meepsquared_b200.build [--verbose]

The library is one translation unit (csrc/libmeep2b.cu) with the CUDA runtime linked statically, so it loads
without the driver library present; it resolves cuTensorMapEncodeTiled through the runtime at first use.
"""

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libmeep2b.so")
SOURCES = ["libmeep2b.cu", "capi.cu", "route.cu", "grouped_gemm.cu", "grouped_gemm_q.cuh", "grouped_gemm_qpair.cuh",
           "reduce.cu", "quant.cu", "merge.cu", "fp8_products.cu", "swiglu.cu",
           "common.cuh", "host.hpp"]


def nvcc() -> str:
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libmeep2b")


def stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(HERE, "csrc", s) for s in SOURCES] + [os.path.join(HERE, "..", "include", "meep2b.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and not stale():
        return LIB
    cmd = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
           "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
           "-o", LIB + ".tmp", os.path.join(HERE, "csrc", "libmeep2b.cu")]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose:
        sys.stderr.write(r.stdout + r.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
