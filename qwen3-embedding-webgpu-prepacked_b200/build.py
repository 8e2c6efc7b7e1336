"""Build libqwa.so (the C-ABI library) in-tree with nvcc for sm_100a.

The library links the CUDA runtime statically and resolves the driver's
tensor-map encoder at run time, so it loads on a machine without a GPU
(the C-ABI symbol test runs there) and travels as a single file.
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libqwa.so")
SOURCES = ["api.cu", "attention.cu", "prologue.cu", "noalloc.cu", "pool.cu", "rmsnorm.cu", "gemm.cu", "q40.cu", "ffn.cu", "q40_small.cu"]
HEADERS = ["ptx.cuh", "internal.h", "attn_common.cuh", os.path.join("..", "..", "include", "qwa.h")]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-cudart", "static",
]


def nvcc() -> str:
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


STAMP = LIB + ".stamp"  # content hash of what built LIB (kept out of git like the .so)


def _fingerprint() -> str:
    """sha256 over every source, header, this file and the flags: a copy of the
    tree (with file times reset) rebuilds exactly when its contents differ."""
    h = hashlib.sha256()
    for d in SOURCES + HEADERS:
        with open(os.path.join(CSRC, d), "rb") as f:
            h.update(d.encode() + b"\0" + f.read())
    with open(os.path.abspath(__file__), "rb") as f:
        h.update(f.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def _stale() -> bool:
    if not os.path.exists(LIB) or not os.path.exists(STAMP):
        return True
    with open(STAMP) as f:
        return f.read().strip() != _fingerprint()


TRACE_LIB = os.path.join(HERE, "libqwa_trace.so")


def build(force: bool = False, verbose: bool = False, trace: bool = False) -> str:
    """Build libqwa.so; trace=True builds the clock64-timeline variant
    libqwa_trace.so (-DQWA_TRACE), used for kernel analysis only."""
    lib = TRACE_LIB if trace else LIB
    if not force and not trace and not _stale():
        return LIB
    objs = []
    for src in SOURCES:
        obj = os.path.join(CSRC, src.replace(".cu", ".trace.o" if trace else ".o"))
        cmd = [nvcc(), *NVCC_FLAGS, *(["-DQWA_TRACE"] if trace else []), "-c",
               os.path.join(CSRC, src), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = lib + ".tmp"
    subprocess.run([nvcc(), "-shared", *NVCC_FLAGS, *objs, "-o", tmp], check=True)
    os.replace(tmp, lib)
    for o in objs:
        os.remove(o)
    if not trace:
        with open(STAMP, "w") as f:
            f.write(_fingerprint() + "\n")
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv,
                trace="--trace" in sys.argv))
