"""Build step for libtkm_b200.so (sm_100a).  Cross-compiles without a GPU.

    python -m tokamak_b200.build            # build if sources are newer
    python -m tokamak_b200.build --force
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtkm_b200.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=default",
]


def _newer(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build_kernels(force=False, verbose=False):
    sources = glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(CSRC, "*.h")) + [os.path.join(ROOT, "include", "tkm_b200.h")]
    if not force and not _newer(LIB, sources):
        return LIB
    cmd = ["nvcc"] + NVCC_FLAGS + ["-o", LIB, os.path.join(CSRC, "tkb_all.cu")]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed for libtkm_b200.so")
    return LIB


def build_all(force=False, verbose=False):
    out = [build_kernels(force, verbose)]
    return out


if __name__ == "__main__":
    print(build_all(force="--force" in sys.argv, verbose=True))
