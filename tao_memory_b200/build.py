"""Build libtao_b200.so in-tree with nvcc for sm_100a.

``python -m tao_memory_b200.build`` (or ``build()``) compiles every ``csrc/*.cu``
into ``tao_memory_b200/libtao_b200.so``.  The library is a plain CUDA shared
object with a C ABI (``include/tao_b200.h``); it links only the CUDA runtime.
No fast-math: the kernels reproduce the reference's IEEE rounding points.
"""

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libtao_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def sources():
    csrc = os.path.join(HERE, "csrc")
    return sorted(os.path.join(csrc, f) for f in os.listdir(csrc) if f.endswith(".cu"))


def build(verbose=False, extra=()):
    nvcc = os.environ.get("NVCC", "nvcc")
    cmd = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", os.path.join(ROOT, "include"), "-o", LIB, *sources(), "-lcudart", *extra]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:])
