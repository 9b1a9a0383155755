"""Build step for the two shared libraries (cross-compiles without a GPU).

  libtkm_b200.so   sm_100a kernels behind the C ABI of include/tkm_b200.h
  libtkm.so        the Tokamak engine of include/tkm.h (registry, DSL front
                   end, NVRTC code generator, runtime) in C, linked to
                   libtkm_b200.so; the device prelude is embedded as a string

    python -m tokamak_b200.build            # build what is out of date
    python -m tokamak_b200.build --force
"""
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
HOST = os.path.join(HERE, "host")
GEN = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtkm_b200.so")
ENGINE = os.path.join(HERE, "libtkm.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")

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


def _run(cmd, what, verbose):
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build failed: " + what)


def build_kernels(force=False, verbose=False):
    sources = glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(CSRC, "*.h")) + [os.path.join(ROOT, "include", "tkm_b200.h")]
    if not force and not _newer(LIB, sources):
        return LIB
    _run(["nvcc"] + NVCC_FLAGS + ["-o", LIB, os.path.join(CSRC, "tkb_all.cu")], "libtkm_b200.so", verbose)
    return LIB


def _embed_prelude():
    """tkm_prelude.cuh -> a C array (NVRTC compiles it in front of the generated code)."""
    os.makedirs(GEN, exist_ok=True)
    src = os.path.join(HOST, "tkm_prelude.cuh")
    out = os.path.join(GEN, "tkm_prelude_embed.c")
    if os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(src):
        return out
    data = open(src, "rb").read() + b"\0"
    rows = [", ".join(str(b) for b in data[i:i + 24]) for i in range(0, len(data), 24)]
    with open(out, "w") as f:
        f.write("/* generated from tkm_prelude.cuh by tokamak_b200/build.py */\n")
        f.write("const char tkm_prelude_src[] = {\n" + ",\n".join(rows) + "\n};\n")
    return out


def build_engine(force=False, verbose=False):
    build_kernels(force, verbose)
    csrcs = sorted(glob.glob(os.path.join(HOST, "*.c")))
    deps = csrcs + glob.glob(os.path.join(HOST, "*.h")) + [os.path.join(HOST, "tkm_prelude.cuh"),
                                                          os.path.join(ROOT, "include", "tkm.h"),
                                                          os.path.join(ROOT, "include", "tkm_b200.h"), LIB]
    if not force and not _newer(ENGINE, deps):
        return ENGINE
    embed = _embed_prelude()
    cmd = ["gcc", "-O2", "-g", "-std=gnu11", "-fPIC", "-shared", "-Wall", "-Wno-unused-function",
           "-D_GNU_SOURCE", "-I" + os.path.join(ROOT, "include"), "-I" + HOST, "-I" + os.path.join(CUDA, "include"),
           "-o", ENGINE] + csrcs + [embed] + [
        "-L" + HERE, "-ltkm_b200", "-L" + os.path.join(CUDA, "lib64"), "-lcudart", "-lcublas", "-lnvrtc",
        "-ldl", "-lpthread", "-lm", "-Wl,-rpath,$ORIGIN", "-Wl,-rpath," + os.path.join(CUDA, "lib64")]
    _run(cmd, "libtkm.so", verbose)
    return ENGINE


def build_all(force=False, verbose=False):
    return [build_kernels(force, verbose), build_engine(force, verbose)]


if __name__ == "__main__":
    print(build_all(force="--force" in sys.argv, verbose=True))
