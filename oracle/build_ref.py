"""Build recipe for oracle/_ref/ -- TEST INFRASTRUCTURE ONLY.

Compiles the reference (BSODsystem32/Tokamak, a read-only source tree) from
its own source files where they lie, with this recipe (the reference's
Makefile is not used).  The tree is found through the TKM_REFERENCE
environment variable, else as the directory `reference` beside this
repository.  Outputs go to oracle/_ref/ only:

  libtkm_ref.so       the full reference library (registry, DSL core, codegen,
                      GPU runtime) built for sm_100a plus oracle/ref_gpu_harness.cu
                      launchers of its static kernels.  Needs a driver to load.
  libtkm_ref_host.so  the host-only compiler pieces (registry, DSL core,
                      codegen) built with gcc; loads without a GPU.

Machines without the reference tree use the built files, which travel with
a copy of the repository (oracle/_ref is ignored by git only).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("TKM_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
OUT = os.path.join(HERE, "_ref")


def run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout[-4000:] + r.stderr[-4000:])
        raise RuntimeError("reference build failed")


def build():
    if not os.path.isdir(os.path.join(REF, "src")):
        print("reference tree not present; skipping oracle/_ref build")
        return []
    os.makedirs(OUT, exist_ok=True)
    inc = os.path.join(REF, "include")
    src = os.path.join(REF, "src")
    host_srcs = [os.path.join(src, f) for f in ("tkm_registry.c", "tkm_core.c", "tkm_codegen.c")]
    outs = []
    host = os.path.join(OUT, "libtkm_ref_host.so")
    run(["gcc", "-O2", "-fPIC", "-shared", "-I" + inc, "-o", host] + host_srcs + ["-lm"])
    outs.append(host)
    gpu = os.path.join(OUT, "libtkm_ref.so")
    cuda_lib = "/usr/local/cuda/lib64"
    run(["nvcc", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC", "-shared",
         "-I" + inc, "-I" + src, "-o", gpu, os.path.join(HERE, "ref_gpu_harness.cu")] + host_srcs +
        ["-L" + cuda_lib, "-L" + cuda_lib + "/stubs", "-lnvrtc", "-lcuda", "-lcublas",
         "-Xlinker", "-rpath=" + cuda_lib])
    outs.append(gpu)
    return outs


if __name__ == "__main__":
    print(build())
