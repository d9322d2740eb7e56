"""Build liblssab8_b200.so in place (nvcc, sm_100a only).

The library is one translation unit (csrc/capi.cu includes the kernel headers).  Floating-point
flags are part of the contract, not tuning: no fast math, no FMA contraction, IEEE division and
denormals, so every binary32 operation in the fold is the single RN operation the contract names.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "liblssab8_b200.so")
SOURCES = ["capi.cu", "common.cuh", "tcgen05.cuh", "prep.cuh", "prefill.cuh", "decode.cuh", "decode_tc.cuh", "t2_table.inc"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "-ftz=false", "-prec-div=true", "-prec-sqrt=true", "-fmad=false",
]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.sep not in cand or os.path.exists(cand)):
            return cand
    return "nvcc"


def stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    srcs = [os.path.join(CSRC, s) for s in SOURCES] + [os.path.join(HERE, "..", "include", "lssab8.h")]
    return any(os.path.getmtime(s) > t for s in srcs if os.path.exists(s))


def build(force=False, verbose=False):
    if not force and not stale():
        return LIB
    cmd = [nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if verbose else []) + ["-o", LIB, os.path.join(CSRC, "capi.cu")]
    r = subprocess.run(cmd, cwd=CSRC, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building liblssab8_b200.so")
    if verbose:
        sys.stderr.write(r.stderr)
    return LIB


if __name__ == "__main__":
    build(force=True, verbose="-v" in sys.argv)
    print(LIB)
