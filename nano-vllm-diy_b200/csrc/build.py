"""Build libb200ops.so for sm_100a with nvcc (no GPU needed).

Usage: python build.py [--verbose]   (writes ../lib/libb200ops.so)

The library is built in-tree so that it travels with the source tree to the
machine that runs it; a JIT cache would not.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
REPO = os.path.dirname(PKG)
LIB_DIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIB_DIR, "libb200ops.so")
SOURCES = ["b200ops.cu"]
HEADERS = ["common.cuh", "gemm.cuh", "gemm_pair.cuh", "attention.cuh", "decode_attention.cuh",
           "elementwise.cuh", "exchange.cuh", "metadata.cuh", "prefill_tc.cuh"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")


def _inputs():
    files = [os.path.join(HERE, f) for f in SOURCES + HEADERS]
    files += [os.path.join(REPO, "include", "b200ops.h"), os.path.abspath(__file__)]
    return files


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(f) <= t for f in _inputs() if os.path.exists(f))


def build(verbose: bool = False, force: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    cmd = [
        NVCC,
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-shared", "-Xcompiler", "-fPIC",
        "-I", os.path.join(REPO, "include"),
        "-o", LIB + ".tmp",
    ] + [os.path.join(HERE, s) for s in SOURCES] + ["-lcudart"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force=True))
