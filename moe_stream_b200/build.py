"""Build libmoestream.so (sm_100a) in-tree with nvcc.

    python -m moe_stream_b200.build          # or build_library() from Python

The library is written next to this file so that it travels with the
package; it is a plain C-ABI shared object (include/moestream.h), loaded by
``moe_stream_b200._lib`` through ctypes.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libmoestream.so")
SOURCES = ["api.cu", "route.cu", "expert.cu", "expert_mx.cu", "gemm.cu", "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found")


def _deps():
    files = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    files.append(os.path.join(ROOT, "include", "moestream.h"))
    return files


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _deps() + [__file__])


def build_library(force=False, verbose=False, extra=()):
    if not force and up_to_date():
        return LIB
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", os.path.join(ROOT, "include"), "-o", LIB + ".tmp",
           *[os.path.join(CSRC, s) for s in SOURCES], *extra]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout, r.stderr, file=sys.stderr)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    force = "--force" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else []
    print(build_library(force=force, verbose=True, extra=extra))
