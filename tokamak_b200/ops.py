"""Torch-tensor wrappers over the C ABI (include/tkm_b200.h).

Each function allocates its outputs with torch on the tensors' device, calls
the corresponding ``tkb_*`` entry point on the current CUDA stream and raises
``TkbError`` on any failure.  No computation happens in Python.
"""
import ctypes

import torch

from . import DTYPE_BF16, DTYPE_F16, DTYPE_F32, TkbError, check, lib

_DT = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}


def dtype_code(t):
    try:
        return _DT[t.dtype]
    except KeyError:
        raise TkbError(f"unsupported dtype {t.dtype}")


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ws(nbytes, device):
    if nbytes == 0:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


def gqa_attn_fwd(qkv, B, S, Hq, Hkv, D, scale=None, causal=True):
    """qkv: [B, S, (Hq+2Hkv)*D] -> (out [B, S, Hq*D], lse [B*Hq, S] fp32)."""
    scale = D ** -0.5 if scale is None else scale
    out = torch.empty(B, S, Hq * D, dtype=qkv.dtype, device=qkv.device)
    lse = torch.empty(B * Hq, S, dtype=torch.float32, device=qkv.device)
    check(lib().tkb_gqa_attn_fwd(_p(qkv), _p(out), _p(lse), B, S, Hq, Hkv, D, scale, int(causal),
                                 dtype_code(qkv), _stream()), "tkb_gqa_attn_fwd")
    return out, lse


def gqa_attn_bwd(qkv, out, dout, lse, B, S, Hq, Hkv, D, scale=None, causal=True, workspace=None, dqkv=None,
                 keep_ds=True):
    """keep_ds: offer the workspace that stores dS (dQ as a GEMM over it);
    False gives the minimum workspace, on which dQ recomputes S, P and dP."""
    scale = D ** -0.5 if scale is None else scale
    L = lib()
    dt = dtype_code(qkv)
    if keep_ds:
        need = L.tkb_gqa_attn_bwd_workspace_ex(B, S, Hq, D, int(causal), dt)
    else:
        need = L.tkb_gqa_attn_bwd_workspace(B, S, Hq, D, dt)
    if workspace is None:
        workspace, _ = _ws(need, qkv.device)
    else:
        need = workspace.numel() * workspace.element_size()
    if dqkv is None:
        dqkv = torch.empty_like(qkv)
    check(L.tkb_gqa_attn_bwd(_p(qkv), _p(out), _p(dout), _p(lse), _p(dqkv), _p(workspace), need, B, S, Hq, Hkv,
                             D, scale, int(causal), dt, _stream()), "tkb_gqa_attn_bwd")
    return dqkv


def add_rmsnorm_fwd(x, r, gamma, eps=1e-5):
    rows, C = x.shape[0], x.shape[-1]
    s = torch.empty_like(x) if r is not None else None
    y = torch.empty_like(x)
    istd = torch.empty(rows, dtype=torch.float32, device=x.device)
    check(lib().tkb_add_rmsnorm_fwd(_p(x), _p(r), _p(s), _p(y), _p(gamma), _p(istd), rows, C, eps,
                                    dtype_code(x), _stream()), "tkb_add_rmsnorm_fwd")
    return (s if s is not None else x), y, istd


def add_rmsnorm_bwd(dy, s, gamma, istd, ds_skip=None, dgamma=None):
    rows, C = s.shape[0], s.shape[-1]
    L = lib()
    dx = torch.empty_like(s)
    need = L.tkb_add_rmsnorm_bwd_workspace(rows, C)
    ws, _ = _ws(need, s.device)
    check(L.tkb_add_rmsnorm_bwd(_p(dy), _p(s), _p(gamma), _p(istd), _p(ds_skip), _p(dx), _p(dgamma), _p(ws),
                                need, rows, C, dtype_code(s), _stream()), "tkb_add_rmsnorm_bwd")
    return dx


def swiglu_fwd(gu, bg=None, bu=None):
    rows, F = gu.shape[0], gu.shape[-1] // 2
    h = torch.empty(rows, F, dtype=gu.dtype, device=gu.device)
    check(lib().tkb_swiglu_fwd(_p(gu), _p(bg), _p(bu), _p(h), rows, F, dtype_code(gu), _stream()),
          "tkb_swiglu_fwd")
    return h


def swiglu_bwd(dh, gu, bg=None, bu=None, dbg=None, dbu=None):
    rows, F = gu.shape[0], gu.shape[-1] // 2
    L = lib()
    dgu = torch.empty_like(gu)
    need = L.tkb_swiglu_bwd_workspace(rows, F)
    ws, _ = _ws(need, gu.device)
    check(L.tkb_swiglu_bwd(_p(dh), _p(gu), _p(bg), _p(bu), _p(dgu), _p(dbg), _p(dbu), _p(ws), need, rows, F,
                           dtype_code(gu), _stream()), "tkb_swiglu_bwd")
    return dgu


def qkv_prep_fwd(x, bias, gain, S, Hq, Hkv, D, qknorm=False, rope=True, theta=10000.0, rope_scale=1.0,
                 low=1.0, high=4.0, octx=8192.0):
    rows = x.shape[0]
    out = torch.empty_like(x)
    istd = torch.empty(rows, Hq + Hkv, dtype=torch.float32, device=x.device) if qknorm else None
    check(lib().tkb_qkv_prep_fwd(_p(x), _p(bias), _p(gain), _p(out), _p(istd), rows, S, Hq, Hkv, D, int(qknorm),
                                 int(rope), theta, rope_scale, low, high, octx, dtype_code(x), _stream()),
          "tkb_qkv_prep_fwd")
    return out, istd


def qkv_prep_bwd(dout, x, bias, gain, istd, din, S, Hq, Hkv, D, qknorm=False, rope=True, theta=10000.0,
                 rope_scale=1.0, low=1.0, high=4.0, octx=8192.0, dbias=None, dgain=None):
    rows = x.shape[0]
    L = lib()
    need = L.tkb_qkv_prep_bwd_workspace(rows, Hq, Hkv, D)
    ws, _ = _ws(need, x.device)
    check(L.tkb_qkv_prep_bwd(_p(dout), _p(x), _p(bias), _p(gain), _p(istd), _p(din), _p(dbias), _p(dgain), _p(ws),
                             need, rows, S, Hq, Hkv, D, int(qknorm), int(rope), theta, rope_scale, low, high, octx,
                             dtype_code(x), _stream()), "tkb_qkv_prep_bwd")
    return din


def softmax_fwd(x):
    rows, C = x.shape
    p = torch.empty_like(x)
    check(lib().tkb_softmax_fwd(_p(x), _p(p), rows, C, dtype_code(x), _stream()), "tkb_softmax_fwd")
    return p


def softmax_bwd(p, dp, dx):
    rows, C = p.shape
    check(lib().tkb_softmax_bwd(_p(p), _p(dp), _p(dx), rows, C, dtype_code(p), _stream()), "tkb_softmax_bwd")
    return dx


def softmax_loss(logits, labels, kind=0, gamma=2.0, want_grad=True):
    rows, C = logits.shape
    L = lib()
    dl = torch.empty_like(logits) if want_grad else None
    loss = torch.zeros(1, dtype=torch.float32, device=logits.device)
    corr = torch.zeros(1, dtype=torch.int32, device=logits.device)
    need = L.tkb_softmax_loss_workspace(rows)
    ws, _ = _ws(need, logits.device)
    check(L.tkb_softmax_loss(_p(logits), _p(labels), _p(dl), _p(loss), _p(corr), _p(ws), need, rows, C, kind,
                             gamma, dtype_code(logits), _stream()), "tkb_softmax_loss")
    return loss, dl, corr


class SgdTensor(ctypes.Structure):
    _fields_ = [("master", ctypes.c_void_p), ("vel", ctypes.c_void_p), ("grad", ctypes.c_void_p),
                ("lowp", ctypes.c_void_p), ("n", ctypes.c_longlong), ("apply_wd", ctypes.c_int),
                ("lowp_dtype", ctypes.c_int)]


def sgd_table(entries, device):
    """entries: list of (master, vel, grad, lowp_or_None, apply_wd) -> device table tensor."""
    arr = (SgdTensor * len(entries))()
    for i, (m, v, g, lp, wd) in enumerate(entries):
        arr[i] = SgdTensor(m.data_ptr(), v.data_ptr(), g.data_ptr(), lp.data_ptr() if lp is not None else None,
                           m.numel(), int(wd), dtype_code(lp) if lp is not None else 0)
    host = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
    return host.to(device)


def sgd_step(table, n, lr_dev, momentum=0.9, wd=1e-4, seed_dev=None):
    check(lib().tkb_sgd_step(_p(table), n, _p(lr_dev), momentum, wd, _p(seed_dev), _stream()), "tkb_sgd_step")


def gemm(A, B, a_trans=False, b_trans=False, out=None, out_dtype=None, accumulate=False, bias=None):
    """C (+)= op(A) op(B) on the tcgen05 GEMM (tkb_gemm).  A is [M][K] (a_trans:
    [K][M]); B is [K][N] (b_trans: [N][K]); bf16 operands, C bf16 or fp32."""
    M = A.shape[1] if a_trans else A.shape[0]
    K = A.shape[0] if a_trans else A.shape[1]
    N = B.shape[0] if b_trans else B.shape[1]
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype or torch.bfloat16, device=A.device)
    ws, nws = _ws(lib().tkb_gemm_workspace(M, N, K, dtype_code(out)), A.device)
    check(lib().tkb_gemm(_p(A), A.stride(0), int(a_trans), _p(B), B.stride(0), int(b_trans), _p(out), out.stride(0),
                         dtype_code(out), int(accumulate), _p(bias), M, N, K, _p(ws), nws, _stream()), "tkb_gemm")
    return out


def gemm_swiglu(A, B, F, bias_gate=None, bias_up=None):
    """([G|U] bf16 [M][2F], h bf16 [M][F]) with [G|U] = A B and h = SiLU(G + b_g) * (U + b_u)."""
    M, K = A.shape
    gu = torch.empty(M, 2 * F, dtype=torch.bfloat16, device=A.device)
    h = torch.empty(M, F, dtype=torch.bfloat16, device=A.device)
    check(lib().tkb_gemm_swiglu(_p(A), A.stride(0), _p(B), B.stride(0), F, _p(bias_gate), _p(bias_up), _p(gu),
                                gu.stride(0), _p(h), h.stride(0), M, K, _stream()), "tkb_gemm_swiglu")
    return gu, h


def lmhead_ce(X, W, labels, bias=None, want_grad=True):
    """(loss, d logits or None, correct) of softmax cross-entropy over
    logits = X W + bias, without storing the logits (tkb_lmhead_ce)."""
    rows, d = X.shape
    V = W.shape[1]
    loss = torch.zeros(1, dtype=torch.float32, device=X.device)
    corr = torch.zeros(1, dtype=torch.int32, device=X.device)
    dl = torch.empty(rows, V, dtype=torch.bfloat16, device=X.device) if want_grad else None
    ws, nws = _ws(lib().tkb_lmhead_ce_workspace(rows, V), X.device)
    check(lib().tkb_lmhead_ce(_p(X), X.stride(0), _p(W), W.stride(0), _p(bias), _p(labels), _p(dl),
                              dl.stride(0) if dl is not None else 0, _p(loss), _p(corr), _p(ws), nws, rows, d, V,
                              _stream()), "tkb_lmhead_ce")
    return loss, dl, corr
