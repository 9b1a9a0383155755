"""Parity of the sm_100a attention kernels (C ABI) with the CPU oracle.

Tolerances (north_star): bf16/f16 mode within 2e-2 relative L2 on O, dQ,
dK, dV; fp32 mode within 1e-4.  LSE is compared with a 1e-2 absolute bound
in 16-bit mode (it is computed from the same fp32 scores).
"""
import numpy as np
import pytest

import oracle
from tests.conftest import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL16 = 2e-2
TOL32 = 1e-4


def _ops():
    from tokamak_b200 import ops
    return ops


def _case(rng, B, S, Hq, Hkv, D, dtype):
    qkv = rng.standard_normal((B, S, (Hq + 2 * Hkv) * D)).astype(np.float32)
    dout = rng.standard_normal((B, S, Hq * D)).astype(np.float32)
    tq = torch.from_numpy(qkv).to("cuda", dtype)
    td = torch.from_numpy(dout).to("cuda", dtype)
    # the oracle sees exactly the values the GPU sees
    return tq.float().cpu().numpy(), td.float().cpu().numpy(), tq, td


CASES = [
    # B, S, Hq, Hkv, D, causal
    (1, 128, 1, 1, 128, True),
    (1, 256, 2, 2, 128, False),
    (2, 256, 4, 2, 128, True),
    (1, 384, 2, 1, 64, True),
    (1, 200, 2, 2, 128, True),      # ragged: S not a multiple of the tile
    (1, 77, 2, 1, 64, False),       # ragged and shorter than one tile
    (1, 640, 8, 2, 128, True),      # GQA group of 4, odd number of query tiles
    (2, 1024, 2, 1, 64, True),
]


@pytest.mark.parametrize("B,S,Hq,Hkv,D,causal", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("keep_ds", [True, False], ids=["dS-GEMM", "recompute"])
def test_attn_fwd_bwd_16bit(rng, B, S, Hq, Hkv, D, causal, dtype, keep_ds):
    ops = _ops()
    qkv, dout, tq, td = _case(rng, B, S, Hq, Hkv, D, dtype)
    scale = D ** -0.5
    ref_o, ref_lse = oracle.attn_fwd(qkv, B, S, Hq, Hkv, D, scale, causal)
    o, lse = ops.gqa_attn_fwd(tq, B, S, Hq, Hkv, D, scale, causal)
    torch.cuda.synchronize()
    o_np = o.float().cpu().numpy()
    assert np.isfinite(o_np).all()
    assert rel_l2(o_np, ref_o) < TOL16, rel_l2(o_np, ref_o)
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < 1e-2
    # backward from the oracle's own O/LSE so that the check isolates the bwd kernel
    ref_d = oracle.attn_bwd(qkv, ref_o, dout, ref_lse, B, S, Hq, Hkv, D, scale, causal)
    to = torch.from_numpy(ref_o).to("cuda", dtype)
    tl = torch.from_numpy(ref_lse).cuda()
    dq = ops.gqa_attn_bwd(tq, to, td, tl, B, S, Hq, Hkv, D, scale, causal, keep_ds=keep_ds)
    torch.cuda.synchronize()
    d = dq.float().cpu().numpy().reshape(B, S, Hq + 2 * Hkv, D)
    r = ref_d.reshape(B, S, Hq + 2 * Hkv, D)
    for name, sl in (("dQ", slice(0, Hq)), ("dK", slice(Hq, Hq + Hkv)), ("dV", slice(Hq + Hkv, Hq + 2 * Hkv))):
        err = rel_l2(d[:, :, sl], r[:, :, sl])
        assert err < TOL16, (name, err)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_attn_fwd_running_max_jumps(rng, D, causal):
    """The forward's lazy rescale: odd query rows scaled by 150, so their
    scores spread over hundreds of log2 units and their running maximum
    jumps past the rescale threshold at different key blocks, while the
    even rows of the same warp rarely do (12 to 16 of the 16 warps mixed);
    30-70 rows jump by more than 126, where the rescale factor is 0 and the
    partial O of the earlier blocks must be cleared, not kept."""
    ops = _ops()
    B, S, Hq, Hkv = 1, 512, 2, 1
    qkv = rng.standard_normal((B, S, (Hq + 2 * Hkv) * D)).astype(np.float32)
    qkv[0, 1::2, :Hq * D] *= 150.0
    tq = torch.from_numpy(qkv).to("cuda", torch.bfloat16)
    qkv = tq.float().cpu().numpy()
    scale = D ** -0.5
    ref_o, ref_lse = oracle.attn_fwd(qkv, B, S, Hq, Hkv, D, scale, causal)
    o, lse = ops.gqa_attn_fwd(tq, B, S, Hq, Hkv, D, scale, causal)
    torch.cuda.synchronize()
    o_np = o.float().cpu().numpy()
    assert np.isfinite(o_np).all()
    assert rel_l2(o_np, ref_o) < TOL16, rel_l2(o_np, ref_o)
    assert np.abs(lse.cpu().numpy() - ref_lse).max() < 2e-2 * max(1.0, np.abs(ref_lse).max() / 100)


@pytest.mark.parametrize("B,S,Hq,Hkv,D,causal", [(1, 128, 2, 1, 64, True), (2, 96, 4, 2, 128, False),
                                                   (1, 130, 2, 2, 64, True)])
def test_attn_fp32_mode(rng, B, S, Hq, Hkv, D, causal):
    ops = _ops()
    qkv, dout, tq, td = _case(rng, B, S, Hq, Hkv, D, torch.float32)
    scale = D ** -0.5
    ref_o, ref_lse = oracle.attn_fwd(qkv, B, S, Hq, Hkv, D, scale, causal)
    o, lse = ops.gqa_attn_fwd(tq, B, S, Hq, Hkv, D, scale, causal)
    assert rel_l2(o.cpu().numpy(), ref_o) < TOL32
    ref_d = oracle.attn_bwd(qkv, ref_o, dout, ref_lse, B, S, Hq, Hkv, D, scale, causal)
    dq = ops.gqa_attn_bwd(tq, o, td, lse, B, S, Hq, Hkv, D, scale, causal)
    assert rel_l2(dq.cpu().numpy(), ref_d) < TOL32


def _torch_reference(q, k, v, do, causal, scale):
    """fp32 attention with autograd on the GPU (no tf32)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    q = q.float().requires_grad_()
    k = k.float().requires_grad_()
    v = v.float().requires_grad_()
    s = torch.einsum("bhqd,bhkd->bhqk", q, k) * scale
    if causal:
        n = s.shape[-1]
        mask = torch.ones(n, n, dtype=torch.bool, device=s.device).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhqk,bhkd->bhqd", p, v)
    o.backward(do.float())
    return o.detach(), q.grad, k.grad, v.grad


@pytest.mark.slow
def test_attn_headline_shape_vs_torch_fp32(rng):
    """B=8, H=16, S=4096, D=128 causal bf16 (the benchmark shape): two heads
    of batch 0 checked against an fp32 torch reference; every head checked
    for finiteness and the LSE bound."""
    ops = _ops()
    B, S, H, D = 8, 4096, 16, 128
    g = torch.Generator(device="cuda").manual_seed(7)
    qkv = torch.randn(B, S, 3 * H * D, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.randn(B, S, H * D, device="cuda", generator=g).to(torch.bfloat16)
    scale = D ** -0.5
    o, lse = ops.gqa_attn_fwd(qkv, B, S, H, H, D, scale, True)
    dqkv = ops.gqa_attn_bwd(qkv, o, dout, lse, B, S, H, H, D, scale, True)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(dqkv).all()
    v4 = qkv.view(B, S, 3, H, D)
    for h in (0, 11):
        q = v4[0, :, 0, h][None, None]
        k = v4[0, :, 1, h][None, None]
        v = v4[0, :, 2, h][None, None]
        do = dout.view(B, S, H, D)[0, :, h][None, None]
        ro, rdq, rdk, rdv = _torch_reference(q, k, v, do, True, scale)
        got_o = o.view(B, S, H, D)[0, :, h].float()
        got = dqkv.view(B, S, 3, H, D)[0, :, :, h].float()
        for name, a, b in (("O", got_o, ro[0, 0]), ("dQ", got[:, 0], rdq[0, 0]), ("dK", got[:, 1], rdk[0, 0]),
                           ("dV", got[:, 2], rdv[0, 0])):
            err = (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)).item()
            assert err < TOL16, (h, name, err)


@pytest.mark.slow
def test_attn_long_sequence_ds_path_vs_recompute():
    """S=16384, 8 query heads over 1 kv head (GQA group of 8), D=128, causal,
    bf16: the backward that keeps every dS tile (8256 tiles per head) and
    computes dQ as a GEMM over them matches the backward that recomputes S, P
    and dP, and one head matches an fp32 torch reference."""
    ops = _ops()
    B, S, Hq, Hkv, D = 1, 16384, 8, 1, 128
    g = torch.Generator(device="cuda").manual_seed(21)
    qkv = torch.randn(B, S, (Hq + 2 * Hkv) * D, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.randn(B, S, Hq * D, device="cuda", generator=g).to(torch.bfloat16)
    scale = D ** -0.5
    o, lse = ops.gqa_attn_fwd(qkv, B, S, Hq, Hkv, D, scale, True)
    d_ds = ops.gqa_attn_bwd(qkv, o, dout, lse, B, S, Hq, Hkv, D, scale, True, keep_ds=True)
    d_rc = ops.gqa_attn_bwd(qkv, o, dout, lse, B, S, Hq, Hkv, D, scale, True, keep_ds=False)
    torch.cuda.synchronize()
    assert torch.isfinite(d_ds).all()
    a, b = d_ds.float(), d_rc.float()
    assert (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)).item() < 1e-2
    # head 5 (kv head 0) against fp32 torch; its dK/dV are the group's sums,
    # so only O and dQ are compared per head here
    v4 = qkv.view(B, S, Hq + 2 * Hkv, D)
    h = 5
    ro, rdq, _, _ = _torch_reference(v4[0, :, h][None, None], v4[0, :, Hq][None, None], v4[0, :, Hq + 1][None, None],
                                     dout.view(B, S, Hq, D)[0, :, h][None, None], True, scale)
    for name, got, ref in (("O", o.view(B, S, Hq, D)[0, :, h].float(), ro[0, 0]),
                           ("dQ", d_ds.view(B, S, Hq + 2 * Hkv, D)[0, :, h].float(), rdq[0, 0])):
        err = (torch.linalg.vector_norm(got - ref) / torch.linalg.vector_norm(ref)).item()
        assert err < TOL16, (name, err)
