"""The C ABI library loads without a GPU, exports every declared entry point,
and rejects bad arguments before touching the device."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"\b(tkb_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol():
    import tokamak_b200
    L = tokamak_b200.lib()
    names = declared("tkm_b200.h")
    assert len(names) >= 20, names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing
    assert b"sm_100a" in L.tkb_version()


def test_python_signatures_cover_header():
    import tokamak_b200
    assert set(declared("tkm_b200.h")) <= set(tokamak_b200._SIGS)


def test_argument_errors_without_device():
    import tokamak_b200
    L = tokamak_b200.lib()
    vp = ctypes.c_void_p
    # head dim 96 is not supported: rejected before any CUDA call
    rc = L.tkb_gqa_attn_fwd(vp(16), vp(16), vp(16), 1, 128, 2, 1, 96, 0.1, 1, 1, None)
    assert rc == -3
    assert b"head dim" in L.tkb_last_error()
    # Hq not a multiple of Hkv
    rc = L.tkb_gqa_attn_fwd(vp(16), vp(16), vp(16), 1, 128, 3, 2, 64, 0.1, 1, 1, None)
    assert rc == -1
    # odd channel count (the reference requires even C, src/tkm_core.c:341-345)
    rc = L.tkb_add_rmsnorm_fwd(vp(16), None, None, vp(16), vp(16), None, 4, 7, 1e-5, 1, None)
    assert rc == -1
    # bad dtype
    rc = L.tkb_softmax_fwd(vp(16), vp(16), 4, 8, 9, None)
    assert rc == -1
    # missing workspace
    rc = L.tkb_softmax_loss(vp(16), None, None, vp(16), None, None, 0, 4, 8, 0, 2.0, 1, None)
    assert rc == -4
    # rows of a multiple of 8 move in 16-byte vectors (bulk copies at 8192-32768):
    # an 8-byte-aligned pointer is refused, as is a 2-byte one for odd pairs
    rc = L.tkb_softmax_loss(vp(24), None, None, None, None, None, 0, 4, 32000, 0, 2.0, 1, None)
    assert rc == -1 and b"16-byte aligned" in L.tkb_last_error()
    rc = L.tkb_softmax_loss(vp(16), None, vp(40), None, None, None, 0, 4, 32000, 0, 2.0, 1, None)
    assert rc == -1
    rc = L.tkb_softmax_loss(vp(18), None, None, None, None, None, 0, 4, 10, 0, 2.0, 1, None)
    assert rc == -1
    rc = L.tkb_softmax_loss_noalloc(vp(24), None, None, None, None, 4, 32000, 0, 2.0, 1, None)
    assert rc == -1 and b"16-byte aligned" in L.tkb_last_error()


def test_workspace_sizes():
    import tokamak_b200
    L = tokamak_b200.lib()
    # LSE*log2(e) and Delta for B*Hq*S_pad rows (no dQ accumulator: the dQ kernel owns its rows)
    n = L.tkb_gqa_attn_bwd_workspace(8, 4096, 16, 128, 1)
    rows = 8 * 16 * 4096
    assert rows * 2 * 4 <= n < rows * 2 * 4 + 1024
    assert L.tkb_gqa_attn_bwd_workspace(8, 4096, 16, 128, 0) == 0
    # with dS kept: 32 KB per 128x128 tile, lower triangle of tiles when causal
    nq = 4096 // 128
    assert L.tkb_gqa_attn_bwd_workspace_ex(8, 4096, 16, 128, 1, 1) == n + 8 * 16 * nq * (nq + 1) // 2 * 32768
    assert L.tkb_gqa_attn_bwd_workspace_ex(8, 4096, 16, 128, 0, 1) == n + 8 * 16 * nq * nq * 32768
    # beyond 32 GiB of dS the minimum workspace is offered (dQ recomputes):
    # S=32768 with 64 heads needs 69 GB of dS, S=16384 17.3 GB (kept)
    assert L.tkb_gqa_attn_bwd_workspace_ex(1, 32768, 64, 128, 1, 1) == L.tkb_gqa_attn_bwd_workspace(1, 32768, 64, 128, 1)
    nq16 = 16384 // 128
    assert L.tkb_gqa_attn_bwd_workspace_ex(1, 16384, 64, 128, 1, 1) == \
        L.tkb_gqa_attn_bwd_workspace(1, 16384, 64, 128, 1) + 64 * nq16 * (nq16 + 1) // 2 * 32768
    assert L.tkb_gqa_attn_bwd_workspace_ex(8, 4096, 16, 128, 1, 0) == 0
    assert L.tkb_add_rmsnorm_bwd_workspace(16384, 4096) > 0
    assert L.tkb_softmax_loss_workspace(8192) >= 8192 * 4


def declared_tkm():
    text = open(os.path.join(ROOT, "include", "tkm.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tkm_[a-z0-9_]+)\s*\(", text)))


def test_engine_exports_every_tkm_h_function():
    import tokamak_b200
    L = tokamak_b200.engine()
    names = declared_tkm()
    assert len(names) >= 45, names
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_engine_runtime_calls_fail_cleanly_without_gpu():
    """Runtime entry points return NULL / 0 with a message instead of exiting
    (the reference exits the process on CUDA errors)."""
    import ctypes
    import torch
    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    from tokamak_b200 import runtime
    L = runtime.lib()
    assert not L.tkm_load_string_ex(b"input: 1x1x32\nt: SiLU -> SoftmaxCE", 2, 1)
    assert runtime.last_error()
    assert L.tkm_runtime_weight_bytes(None) == 0
    assert L.tkm_runtime_input_elements(None) == 0
    assert not L.tkm_load_string(None, 2)
