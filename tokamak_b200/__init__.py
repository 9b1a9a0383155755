"""tokamak_b200 -- B200-native (sm_100a) implementation of Tokamak's GPU hot path.

The product is the C ABI in ``include/tkm_b200.h`` implemented by
``libtkm_b200.so`` (CUDA kernels written for sm_100a).  This package only
loads that library and offers thin torch-tensor wrappers so tests and the
benchmark can call it; it contains no compute of its own and no fallback:
if the library is missing or a call fails, an exception is raised.
"""
import ctypes
import os

__all__ = ["lib", "lib_path", "engine", "engine_path", "TkbError", "DTYPE_F32", "DTYPE_BF16", "DTYPE_F16"]

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


class TkbError(RuntimeError):
    pass


def lib_path():
    return os.path.join(_HERE, "libtkm_b200.so")


_vp, _i, _f, _sz, _ll = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_longlong
_SIGS = {
    "tkb_version": ([], ctypes.c_char_p),
    "tkb_last_error": ([], ctypes.c_char_p),
    "tkb_device_error": ([ctypes.POINTER(ctypes.c_uint), _vp], _i),
    "tkb_selftest_wait_timeout": ([ctypes.c_ulonglong, _vp], _i),
    "tkb_launch_count": ([], ctypes.c_ulonglong),
    "tkb_gqa_attn_fwd": ([_vp, _vp, _vp, _i, _i, _i, _i, _i, _f, _i, _i, _vp], _i),
    "tkb_gqa_attn_bwd_workspace": ([_i, _i, _i, _i, _i], _sz),
    "tkb_gqa_attn_bwd_workspace_ex": ([_i, _i, _i, _i, _i, _i], _sz),
    "tkb_gqa_attn_bwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _i, _i, _f, _i, _i, _vp], _i),
    "tkb_add_rmsnorm_fwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _f, _i, _vp], _i),
    "tkb_add_rmsnorm_bwd_workspace": ([_i, _i], _sz),
    "tkb_add_rmsnorm_bwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _vp], _i),
    "tkb_swiglu_fwd": ([_vp, _vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "tkb_swiglu_bwd_workspace": ([_i, _i], _sz),
    "tkb_swiglu_bwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _vp], _i),
    "tkb_qkv_prep_fwd": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _f, _f, _f, _f, _f, _i, _vp], _i),
    "tkb_qkv_prep_bwd_workspace": ([_i, _i, _i, _i], _sz),
    "tkb_qkv_prep_bwd": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _i, _i, _i, _i,
                          _f, _f, _f, _f, _f, _i, _vp], _i),
    "tkb_softmax_fwd": ([_vp, _vp, _i, _i, _i, _vp], _i),
    "tkb_softmax_bwd": ([_vp, _vp, _vp, _i, _i, _i, _vp], _i),
    "tkb_softmax_loss_workspace": ([_i], _sz),
    "tkb_softmax_loss": ([_vp, _vp, _vp, _vp, _vp, _vp, _sz, _i, _i, _i, _f, _i, _vp], _i),
    "tkb_softmax_loss_noalloc": ([_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _f, _i, _vp], _i),
    "tkb_sgd_step": ([_vp, _i, _vp, _f, _f, _vp, _vp], _i),
    "tkb_gemm_workspace": ([_i, _i, _i, _i], _sz),
    "tkb_lmhead_ce_workspace": ([_i, _i], _sz),
    "tkb_lmhead_ce": ([_vp, _ll, _vp, _ll, _vp, _vp, _vp, _ll, _vp, _vp, _vp, _sz, _i, _i, _i, _vp], _i),
    "tkb_gemm": ([_vp, _ll, _i, _vp, _ll, _i, _vp, _ll, _i, _i, _vp, _i, _i, _i, _vp, _sz, _vp], _i),
    "tkb_gemm_swiglu": ([_vp, _ll, _vp, _ll, _i, _vp, _vp, _vp, _ll, _vp, _ll, _i, _i, _vp], _i),
}


def lib():
    """Load libtkm_b200.so (raises if it has not been built)."""
    global _LIB
    if _LIB is None:
        path = lib_path()
        if not os.path.exists(path):
            raise TkbError(f"{path} is missing: build it with __graft_entry__.build()")
        L = ctypes.CDLL(path)
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _LIB = L
    return _LIB


_ENGINE = None


def engine_path():
    return os.path.join(_HERE, "libtkm.so")


def engine():
    """Load libtkm.so, the Tokamak engine of include/tkm.h (raises if missing).
    Signatures are declared by the callers (tests/tkm_abi.py, tokamak_b200.runtime)."""
    global _ENGINE
    if _ENGINE is None:
        lib()  # libtkm.so links libtkm_b200.so
        path = engine_path()
        if not os.path.exists(path):
            raise TkbError(f"{path} is missing: build it with __graft_entry__.build()")
        _ENGINE = ctypes.CDLL(path)
    return _ENGINE


def check(rc, what=""):
    if rc != 0:
        msg = lib().tkb_last_error().decode(errors="replace")
        raise TkbError(f"{what or 'tkb call'} failed ({rc}): {msg}")
