"""ctypes bindings of the CPU oracle (oracle/tkm_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, never by the product path.  All arrays are
float32 numpy arrays (int32 for labels); the C code accumulates in fp64.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None


def lib_path():
    return os.path.join(_HERE, "libtkm_oracle.so")


def build():
    """Compile the oracle with gcc (OpenMP)."""
    src = os.path.join(_HERE, "tkm_oracle.c")
    out = lib_path()
    cmd = f"gcc -O2 -fopenmp -fPIC -shared -o {out} {src} -lm"
    if os.system(cmd) != 0:
        raise RuntimeError("oracle build failed: " + cmd)
    return out


def lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(lib_path()):
            build()
        _LIB = ctypes.CDLL(lib_path())
        _LIB.tko_softmax_loss.restype = ctypes.c_float
    return _LIB


def _f(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(ctypes.c_void_p)


def _i32(a):
    if a is None:
        return None
    assert a.dtype == np.int32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def attn_fwd(qkv, B, S, Hq, Hkv, D, scale, causal):
    out = np.zeros((B, S, Hq * D), np.float32)
    lse = np.zeros((B * Hq, S), np.float32)
    lib().tko_attn_fwd(_f(qkv), _f(out), _f(lse), B, S, Hq, Hkv, D, ctypes.c_float(scale), int(causal))
    return out, lse


def attn_bwd(qkv, out, dout, lse, B, S, Hq, Hkv, D, scale, causal):
    dqkv = np.zeros_like(qkv)
    lib().tko_attn_bwd(_f(qkv), _f(out), _f(dout), _f(lse), _f(dqkv), B, S, Hq, Hkv, D, ctypes.c_float(scale),
                       int(causal))
    return dqkv


def add_rmsnorm_fwd(x, r, gamma, eps=1e-5):
    rows, C = x.shape
    s = np.zeros_like(x)
    y = np.zeros_like(x)
    istd = np.zeros(rows, np.float32)
    lib().tko_add_rmsnorm_fwd(_f(x), _f(r), _f(s), _f(y), _f(gamma), _f(istd), rows, C, ctypes.c_float(eps))
    return s, y, istd


def add_rmsnorm_bwd(dy, s, gamma, istd, ds_skip=None):
    rows, C = s.shape
    dx = np.zeros_like(s)
    dg = np.zeros(C, np.float32)
    lib().tko_add_rmsnorm_bwd(_f(dy), _f(s), _f(gamma), _f(istd), _f(ds_skip), _f(dx), _f(dg), rows, C)
    return dx, dg


def swiglu_fwd(gu, bg=None, bu=None):
    rows, F2 = gu.shape
    h = np.zeros((rows, F2 // 2), np.float32)
    lib().tko_swiglu_fwd(_f(gu), _f(bg), _f(bu), _f(h), rows, F2 // 2)
    return h


def swiglu_bwd(dh, gu, bg=None, bu=None):
    rows, F2 = gu.shape
    F = F2 // 2
    dgu = np.zeros_like(gu)
    dbg = np.zeros(F, np.float32)
    dbu = np.zeros(F, np.float32)
    lib().tko_swiglu_bwd(_f(dh), _f(gu), _f(bg), _f(bu), _f(dgu), _f(dbg), _f(dbu), rows, F)
    return dgu, dbg, dbu


def qkv_prep_fwd(x, bias, gain, S, Hq, Hkv, D, qknorm, rope, theta=10000.0, scale=1.0, low=1.0, high=4.0,
                 octx=8192.0):
    rows = x.shape[0]
    out = np.zeros_like(x)
    istd = np.zeros((rows, Hq + Hkv), np.float32)
    c = ctypes.c_float
    lib().tko_qkv_prep_fwd(_f(x), _f(bias), _f(gain), _f(out), _f(istd), rows, S, Hq, Hkv, D, int(qknorm), int(rope),
                           c(theta), c(scale), c(low), c(high), c(octx))
    return out, istd


def qkv_prep_bwd(dout, x, bias, gain, istd, S, Hq, Hkv, D, qknorm, rope, theta=10000.0, scale=1.0, low=1.0,
                 high=4.0, octx=8192.0):
    rows = x.shape[0]
    din = np.zeros_like(x)
    db = np.zeros(x.shape[1], np.float32)
    dg = np.zeros((Hq + Hkv) * D, np.float32)
    c = ctypes.c_float
    lib().tko_qkv_prep_bwd(_f(dout), _f(x), _f(bias), _f(gain), _f(istd), _f(din), _f(db), _f(dg), rows, S, Hq, Hkv,
                           D, int(qknorm), int(rope), c(theta), c(scale), c(low), c(high), c(octx))
    return din, db, dg


def softmax_fwd(x):
    p = np.zeros_like(x)
    lib().tko_softmax_fwd(_f(x), _f(p), x.shape[0], x.shape[1])
    return p


def softmax_bwd(p, dp, dx):
    dx = dx.copy()
    lib().tko_softmax_bwd(_f(p), _f(dp), _f(dx), p.shape[0], p.shape[1])
    return dx


def softmax_loss(logits, labels, kind=0, gamma=2.0):
    rows, C = logits.shape
    dl = np.zeros_like(logits)
    corr = ctypes.c_int(0)
    loss = lib().tko_softmax_loss(_f(logits), _i32(labels), _f(dl), ctypes.byref(corr), rows, C, kind,
                                  ctypes.c_float(gamma))
    return float(loss), dl, corr.value


def sgd(p, v, g, lr, momentum=0.9, wd=1e-4, apply_wd=True):
    p = p.copy()
    v = v.copy()
    lib().tko_sgd(_f(p), _f(v), _f(g), ctypes.c_long(p.size), ctypes.c_float(lr), ctypes.c_float(momentum),
                  ctypes.c_float(wd), int(apply_wd))
    return p, v


def num_threads():
    return lib().tko_num_threads()


def set_num_threads(n):
    lib().tko_set_num_threads(int(n))
