"""Compile generated plasma code with NVRTC for sm_100a on the host (no GPU
needed): the same prelude + options the runtime uses."""
import ctypes
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PRELUDE = os.path.join(ROOT, "tokamak_b200", "host", "tkm_prelude.cuh")


def _nvrtc():
    for name in ("libnvrtc.so.12", "libnvrtc.so", "/usr/local/cuda/lib64/libnvrtc.so"):
        try:
            return ctypes.CDLL(name)
        except OSError:
            continue
    raise OSError("libnvrtc not found")


def compile_source(src, act_bytes):
    """Returns (ok, log, cubin_size)."""
    L = _nvrtc()
    full = f"#define TKM_ACT_BYTES {act_bytes}\n" + open(PRELUDE).read() + "\n" + src
    prog = ctypes.c_void_p()
    assert L.nvrtcCreateProgram(ctypes.byref(prog), full.encode(), b"tkm_plasma.cu", 0, None, None) == 0
    opts = [b"--gpu-architecture=sm_100a", b"-std=c++17", b"--fmad=true", b"-lineinfo"]
    arr = (ctypes.c_char_p * len(opts))(*opts)
    rc = L.nvrtcCompileProgram(prog, len(opts), arr)
    n = ctypes.c_size_t()
    L.nvrtcGetProgramLogSize(prog, ctypes.byref(n))
    log = ctypes.create_string_buffer(n.value + 1)
    L.nvrtcGetProgramLog(prog, log)
    size = ctypes.c_size_t()
    if rc == 0:
        L.nvrtcGetCUBINSize(prog, ctypes.byref(size))
    L.nvrtcDestroyProgram(ctypes.byref(prog))
    return rc == 0, log.value.decode(errors="replace"), size.value
