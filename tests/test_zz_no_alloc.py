"""tkb_softmax_loss_noalloc: the softmax-loss entry point for callers that
cannot allocate device memory (for example code running during a global-mode
CUDA graph capture, when cudaMalloc fails, or foreign-language callers that
only hold raw device pointers).  It must give the same results as
tkb_softmax_loss with a caller-provided workspace, call after call, even
though every call reuses the one scratch array built into the library.

Both entry points launch the same kernels and sum the per-row losses in the
same fixed order, so their results must agree bit for bit; any row of the
scratch that a call reads without having written it first would show up as a
different loss.

Collected last on purpose (file name), so a stop-at-first-failure run has
already run every other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

MAX_ROWS = 1 << 18


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _call(L, noalloc, logits, labels, dl, loss, corr, kind, gamma, ws=None):
    rows, C = logits.shape
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        return L.tkb_softmax_loss_noalloc(_p(logits), _p(labels), _p(dl), _p(loss), _p(corr), rows, C, kind, gamma, 1,
                                          st)
    return L.tkb_softmax_loss(_p(logits), _p(labels), _p(dl), _p(loss), _p(corr), _p(ws), ws.numel(), rows, C, kind,
                              gamma, 1, st)


def _run(L, noalloc, logits, labels, kind, gamma):
    rows, C = logits.shape
    dl = torch.empty_like(logits)
    loss = torch.zeros(1, dtype=torch.float32, device="cuda")
    corr = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = None if noalloc else torch.empty(L.tkb_softmax_loss_workspace(rows), dtype=torch.uint8, device="cuda")
    rc = _call(L, noalloc, logits, labels, dl, loss, corr, kind, gamma, ws)
    assert rc == 0, L.tkb_last_error()
    torch.cuda.synchronize()
    return loss.item(), dl.float().cpu().numpy(), corr.item()


def _same(a, b):
    assert a[0] == b[0], (a[0], b[0])
    assert np.array_equal(a[1], b[1])
    assert a[2] == b[2]


def test_noalloc_matches_workspace_entry_point_call_after_call():
    from tokamak_b200 import lib
    L = lib()
    g = torch.Generator(device="cuda").manual_seed(99)
    # First call: the scratch limit itself, with extreme logits, so every
    # entry of the scratch holds a large per-row loss afterwards.  The later,
    # smaller calls reuse the array and must overwrite every entry they read.
    cases = ((MAX_ROWS, 64, 0, 40.0), (300, 32000, 1, 2.0), (512, 1000, 0, 2.0), (4097, 4096, 2, 2.0))
    for rows, C, kind, sd in cases:
        logits = (sd * torch.randn(rows, C, device="cuda", generator=g)).bfloat16()
        labels = torch.randint(0, C, (rows,), device="cuda", generator=g, dtype=torch.int32)
        a = _run(L, True, logits, labels, kind, 2.0)
        b = _run(L, False, logits, labels, kind, 2.0)
        _same(a, b)


def test_noalloc_inside_a_global_mode_graph_capture():
    """The reason the entry point exists: a call recorded while a CUDA graph
    is captured in global mode (where cudaMalloc would fail), replayed twice."""
    from tokamak_b200 import lib
    L = lib()
    g = torch.Generator(device="cuda").manual_seed(7)
    rows, C = 1024, 32000
    logits = (2 * torch.randn(rows, C, device="cuda", generator=g)).bfloat16()
    labels = torch.randint(0, C, (rows,), device="cuda", generator=g, dtype=torch.int32)
    ref = _run(L, False, logits, labels, 0, 2.0)
    _same(_run(L, True, logits, labels, 0, 2.0), ref)  # first call on the device: before the capture
    dl = torch.empty_like(logits)
    loss = torch.zeros(1, dtype=torch.float32, device="cuda")
    corr = torch.zeros(1, dtype=torch.int32, device="cuda")
    graph = torch.cuda.CUDAGraph()
    rcs = []
    with torch.cuda.graph(graph, capture_error_mode="global"):
        loss.zero_()
        corr.zero_()
        rcs.append(_call(L, True, logits, labels, dl, loss, corr, 0, 2.0))
    assert rcs == [0], L.tkb_last_error()
    for _ in range(2):
        dl.zero_()
        graph.replay()
        torch.cuda.synchronize()
        _same((loss.item(), dl.float().cpu().numpy(), corr.item()), ref)
    del graph


def test_noalloc_rejects_rows_beyond_its_scratch():
    from tokamak_b200 import lib
    L = lib()
    x = torch.zeros(8, 8, dtype=torch.bfloat16, device="cuda")
    rc = L.tkb_softmax_loss_noalloc(_p(x), None, None, None, None, MAX_ROWS + 1, 8, 0, 2.0, 1, None)
    assert rc == -1
    assert b"exceeds the built-in scratch limit" in L.tkb_last_error()
