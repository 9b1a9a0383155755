"""The tcgen05 GEMM (tkb_gemm, tkb_gemm_swiglu) against an fp32 torch
matmul of the same bf16 operands on the GPU (tf32 off).

Tolerances: the kernel accumulates in fp32, like the reference; a bf16 C is
one bf16 rounding away (relative L2 below 5e-3), an fp32 C agrees to
summation-order differences (1e-5).  Shapes cover every operand layout
(forward X W, input gradient dY W^T, weight gradient X^T dY), ragged tails in
M, N and K, accumulation into C, the bias and SwiGLU epilogues, and the
~1B model's (configuration 4) GEMM shapes.
"""
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL_BF16 = 5e-3
TOL_F32 = 1e-5


def _rel(a, b):
    a, b = a.double(), b.double()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)).item()


def _ref(A, B, a_trans, b_trans):
    torch.backends.cuda.matmul.allow_tf32 = False
    a = A.float().T if a_trans else A.float()
    b = B.float().T if b_trans else B.float()
    return a @ b


def _operands(M, N, K, a_trans, b_trans, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(*((K, M) if a_trans else (M, K)), device="cuda", generator=g).bfloat16()
    B = torch.randn(*((N, K) if b_trans else (K, N)), device="cuda", generator=g).bfloat16()
    return A, B


@pytest.mark.parametrize("a_trans,b_trans", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (200, 312, 136), (1000, 520, 2056), (64, 40, 8)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_layouts_and_tails(a_trans, b_trans, M, N, K, out_dtype):
    from tokamak_b200 import ops
    A, B = _operands(M, N, K, a_trans, b_trans, seed=M + N + K)
    C = ops.gemm(A, B, a_trans, b_trans, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ref = _ref(A, B, a_trans, b_trans)
    assert _rel(C.float(), ref) < (TOL_BF16 if out_dtype == torch.bfloat16 else TOL_F32)


@pytest.mark.parametrize("accumulate", [False, True])
@pytest.mark.parametrize("M,N,K", [(512, 512, 8192), (2000, 768, 6000)])
def test_gemm_split_k_weight_gradient(M, N, K, accumulate):
    """Few output tiles with a long K (a weight gradient): fp32 C from K
    split into partial sums in the workspace, added in a fixed order --
    identical results on repeated calls."""
    from tokamak_b200 import lib, ops
    assert lib().tkb_gemm_workspace(M, N, K, 0) > 0  # this shape splits
    A, B = _operands(M, N, K, True, False, seed=9)
    C0 = torch.randn(M, N, device="cuda")
    C1 = ops.gemm(A, B, True, False, out=C0.clone(), accumulate=accumulate)
    C2 = ops.gemm(A, B, True, False, out=C0.clone(), accumulate=accumulate)
    torch.cuda.synchronize()
    assert torch.equal(C1, C2)
    ref = _ref(A, B, True, False) + (C0 if accumulate else 0)
    assert _rel(C1, ref) < TOL_F32


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_gemm_accumulates_into_c(out_dtype):
    from tokamak_b200 import ops
    M, N, K = 384, 512, 320
    A, B = _operands(M, N, K, False, True, seed=5)
    C0 = torch.randn(M, N, device="cuda").to(out_dtype)
    C = C0.clone()
    ops.gemm(A, B, False, True, out=C, accumulate=True)
    torch.cuda.synchronize()
    assert _rel(C.float(), C0.float() + _ref(A, B, False, True)) < (TOL_BF16 if out_dtype == torch.bfloat16 else TOL_F32)


def test_gemm_bias_epilogue():
    from tokamak_b200 import ops
    M, N, K = 300, 712, 192
    A, B = _operands(M, N, K, False, False, seed=6)
    bias = torch.randn(N, device="cuda")
    C = ops.gemm(A, B, bias=bias)
    torch.cuda.synchronize()
    assert _rel(C.float(), _ref(A, B, False, False) + bias) < TOL_BF16


@pytest.mark.parametrize("M,K,F", [(256, 128, 256), (300, 200, 688), (1024, 256, 5632)])
def test_gemm_swiglu_epilogue(M, K, F):
    from tokamak_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(F)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = (0.1 * torch.randn(K, 2 * F, device="cuda", generator=g)).bfloat16()
    bg = torch.randn(F, device="cuda", generator=g)
    bu = torch.randn(F, device="cuda", generator=g)
    gu, h = ops.gemm_swiglu(A, B, F, bg, bu)
    torch.cuda.synchronize()
    ref_gu = _ref(A, B, False, False)
    assert _rel(gu.float(), ref_gu) < TOL_BF16
    gub = ref_gu.bfloat16().float()  # the epilogue works from the stored bf16 gate and up values
    ref_h = torch.nn.functional.silu(gub[:, :F] + bg) * (gub[:, F:] + bu)
    assert _rel(h.float(), ref_h) < TOL_BF16


# (name, M, N, K, a_trans, b_trans) of one layer of the ~1B decoder (16384 tokens per GPU)
C4_SHAPES = [
    ("qkv fwd", 16384, 3072, 2048, False, False),
    ("o-proj dX", 16384, 2048, 2048, False, True),
    ("down dW", 5632, 2048, 16384, True, False),
    ("lm-head fwd", 16384, 32000, 2048, False, False),
]


@pytest.mark.slow
@pytest.mark.parametrize("name,M,N,K,a_trans,b_trans", C4_SHAPES, ids=[s[0] for s in C4_SHAPES])
def test_gemm_configuration4_shapes(name, M, N, K, a_trans, b_trans):
    from tokamak_b200 import ops
    A, B = _operands(M, N, K, a_trans, b_trans, seed=K)
    A = A * 0.05
    B = B * 0.05
    out_dtype = torch.float32 if "dW" in name else torch.bfloat16
    C = ops.gemm(A, B, a_trans, b_trans, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ref = _ref(A, B, a_trans, b_trans)
    assert _rel(C.float(), ref) < (TOL_BF16 if out_dtype == torch.bfloat16 else 1e-4)


@pytest.mark.slow
def test_gemm_swiglu_configuration4_shape():
    from tokamak_b200 import ops
    M, K, F = 16384, 2048, 5632
    g = torch.Generator(device="cuda").manual_seed(44)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    B = (0.02 * torch.randn(K, 2 * F, device="cuda", generator=g)).bfloat16()
    gu, h = ops.gemm_swiglu(A, B, F)
    torch.cuda.synchronize()
    ref_gu = _ref(A, B, False, False)
    assert _rel(gu.float(), ref_gu) < TOL_BF16
    gub = ref_gu.bfloat16().float()
    assert _rel(h.float(), torch.nn.functional.silu(gub[:, :F]) * gub[:, F:]) < TOL_BF16


def test_gemm_rejects_bad_arguments():
    from tokamak_b200 import lib
    L = lib()
    x = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
    import ctypes
    p = ctypes.c_void_p(x.data_ptr())
    assert L.tkb_gemm(p, 60, 0, p, 64, 0, p, 64, 1, 0, None, 64, 64, 60, None, 0, None) == -1  # lda % 8
    assert L.tkb_gemm(p, 64, 0, p, 64, 0, p, 64, 2, 0, None, 64, 64, 64, None, 0, None) == -1  # fp16 C
    assert L.tkb_gemm(p, 64, 0, p, 64, 0, p, 64, 1, 0, None, 0, 64, 64, None, 0, None) == -1   # empty M
    assert L.tkb_gemm_swiglu(p, 64, p, 64, 12, None, None, p, 64, p, 64, 64, 64, None) == -1  # F % 8
