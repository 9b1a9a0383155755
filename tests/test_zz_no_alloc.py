"""tkb_softmax_loss_noalloc: the softmax-loss entry point for callers that
cannot allocate device memory (for example code running during a global-mode
CUDA graph capture, when cudaMalloc fails, or foreign-language callers that
only hold raw device pointers).  It must give the same results as
tkb_softmax_loss with a caller-provided workspace, call after call, even
though every call reuses the one scratch array built into the library.

Collected last on purpose (file name), so a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL16 = 2e-2  # the 16-bit tolerance the other parity tests use
MAX_ROWS = 1 << 18


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _run(L, noalloc, logits, labels, kind, gamma):
    rows, C = logits.shape
    dl = torch.empty_like(logits)
    loss = torch.zeros(1, dtype=torch.float32, device="cuda")
    corr = torch.zeros(1, dtype=torch.int32, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = L.tkb_softmax_loss_noalloc(_p(logits), _p(labels), _p(dl), _p(loss), _p(corr), rows, C, kind, gamma, 1, st)
    else:
        n = L.tkb_softmax_loss_workspace(rows)
        ws = torch.empty(n, dtype=torch.uint8, device="cuda")
        rc = L.tkb_softmax_loss(_p(logits), _p(labels), _p(dl), _p(loss), _p(corr), _p(ws), n, rows, C, kind, gamma,
                                1, st)
    assert rc == 0, L.tkb_last_error()
    torch.cuda.synchronize()
    return loss.item(), dl.float().cpu().numpy(), corr.item()


def test_noalloc_matches_workspace_entry_point_twice():
    from tokamak_b200 import lib
    L = lib()
    g = torch.Generator(device="cuda").manual_seed(99)
    # two calls in a row with different shapes: the second reuses (and must
    # fully overwrite what it reads of) the scratch left by the first
    for rows, C, kind in ((512, 1000, 0), (300, 32000, 1)):
        logits = (2 * torch.randn(rows, C, device="cuda", generator=g)).bfloat16()
        labels = torch.randint(0, C, (rows,), device="cuda", generator=g, dtype=torch.int32)
        a = _run(L, True, logits, labels, kind, 2.0)
        b = _run(L, False, logits, labels, kind, 2.0)
        assert abs(a[0] - b[0]) <= TOL16 * abs(b[0])
        err = np.linalg.norm(a[1] - b[1]) / np.linalg.norm(b[1])
        assert err < TOL16, err
        assert a[2] == b[2]


def test_noalloc_rejects_rows_beyond_its_scratch():
    from tokamak_b200 import lib
    L = lib()
    x = torch.zeros(8, 8, dtype=torch.bfloat16, device="cuda")
    rc = L.tkb_softmax_loss_noalloc(_p(x), None, None, None, None, MAX_ROWS + 1, 8, 0, 2.0, 1, None)
    assert rc == -1
    assert b"exceeds the built-in scratch limit" in L.tkb_last_error()
