"""Builds libcudanet_b200.so in this folder with nvcc for sm_100a (B200). No GPU is needed to build.

    python -m mayfly_chess_b200.build [--force]

The library is one translation unit (csrc/net.cu includes the kernels) linked against the static CUDA
runtime, so it needs nothing at run time beyond the NVIDIA driver; the driver's cuTensorMapEncodeTiled is
fetched through cudaGetDriverEntryPoint.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libcudanet_b200.so")
SOURCES = ["net.cu"]
HEADERS = ["ptx.cuh", "gemm.cuh", "gemm_ln.cuh", "trunk.cuh", "attention_tc.cuh", "encode.cuh", "json_min.h"]
NVCC_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
              "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared", "-cudart", "static"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise FileNotFoundError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def _inputs():
    files = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    files.append(os.path.join(REPO, "include", "cudanet_b200.h"))
    files.append(os.path.abspath(__file__))
    return files


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs())


def build(force=False, verbose=False):
    """Compile the library unless it is newer than every source. Returns its path."""
    if not force and up_to_date():
        return LIB
    cmd = [nvcc()] + NVCC_FLAGS + [os.path.join(CSRC, s) for s in SOURCES] + ["-o", LIB + ".tmp"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
