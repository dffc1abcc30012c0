"""Build ``libcdlb200.so`` in-tree with nvcc for sm_100a.

The library is plain CUDA C++ behind a C ABI (``include/cdlb200.h``); it does
not link against torch.  Run ``python -m cdl_b200.build`` (or
``__graft_entry__.build()``).  Sources are compiled in parallel and the link
is skipped when nothing changed.
"""

from __future__ import annotations

import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libcdlb200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No --use_fast_math: the kernels rely on IEEE divide and on subnormals.
FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-ftz=false", "-prec-div=true",
    "-prec-sqrt=true", "-fmad=true", "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include"),
]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))]
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        subprocess.run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcuda"], check=True)
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print(LIB)
