"""Builds the ECF8 CUDA library in-tree: ecf8_b200/libecf8_b200.so (sm_100a).

    python -m ecf8_b200.build          # or __graft_entry__.build()

The library is plain nvcc output with a C ABI (include/ecf8.h); it is loaded
with ctypes and linked against the shared CUDA runtime, so it shares the
runtime (current device, streams) with PyTorch in the same process.
"""

import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_NAME = "libecf8_b200.so"
SOURCES = ["csrc/ecf8_decode.cu", "csrc/ecf8_encode.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    cand = shutil.which("nvcc")
    if cand:
        return cand
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda, "bin", "nvcc")
    if os.path.exists(cand):
        return cand
    raise RuntimeError("nvcc not found (set CUDA_HOME)")


def cuda_lib_dir():
    nvcc = nvcc_path()
    return os.path.join(os.path.dirname(os.path.dirname(nvcc)), "lib64")


def build(verbose=False, extra_flags=()):
    """Compiles the library if any source is newer than it; returns its path."""
    out = os.path.join(PKG, LIB_NAME)
    srcs = [os.path.join(PKG, s) for s in SOURCES]
    header = os.path.join(ROOT, "include", "ecf8.h")
    newest = max(os.path.getmtime(p) for p in srcs + [header, __file__])
    if os.path.exists(out) and os.path.getmtime(out) >= newest and not extra_flags:
        return out
    cmd = [
        nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC,-O3", "-shared", "-cudart", "shared",
        "-I", os.path.join(ROOT, "include"),
        "-Xlinker", "-rpath," + cuda_lib_dir(),
        *extra_flags, *srcs, "-o", out + f".tmp{os.getpid()}",
    ]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(out + f".tmp{os.getpid()}", out)  # per-process temp: ranks may build at once
    return out


if __name__ == "__main__":
    print(build(verbose=True))
