"""Parity of the sm_100a row kernels (C ABI) with the CPU oracle.

Tolerances: 16-bit storage within 2e-2 relative L2 (the north_star bf16
bound), fp32 storage within 1e-4 relative L2 (1e-5 for pure elementwise).
Parameter gradients (fp32 sums) are compared at the same bounds.
"""
import numpy as np
import pytest

import oracle
from tests.conftest import rel_l2

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.bfloat16, torch.float16]


def tol(dtype):
    return 1e-4 if dtype == torch.float32 else 2e-2


def dev(a, dtype):
    t = torch.from_numpy(np.ascontiguousarray(a)).to("cuda", dtype)
    return t, t.float().cpu().numpy()


def ops():
    from tokamak_b200 import ops as o
    return o


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,C", [(64, 256), (33, 4096), (17, 688), (8, 1030), (5, 11008)])
def test_add_rmsnorm(rng, dtype, rows, C):
    o = ops()
    x, xn = dev(rng.standard_normal((rows, C)), dtype)
    r, rn = dev(rng.standard_normal((rows, C)), dtype)
    g = torch.from_numpy((1 + 0.02 * rng.standard_normal(C)).astype(np.float32)).cuda()
    gn = g.cpu().numpy()
    s, y, istd = o.add_rmsnorm_fwd(x, r, g)
    rs, ry, ristd = oracle.add_rmsnorm_fwd(xn, rn, gn)
    assert rel_l2(s.float().cpu().numpy(), rs) < tol(dtype)
    assert rel_l2(y.float().cpu().numpy(), ry) < tol(dtype)
    assert rel_l2(istd.cpu().numpy(), ristd) < tol(dtype)
    dy, dyn = dev(rng.standard_normal((rows, C)), dtype)
    dsk, dskn = dev(rng.standard_normal((rows, C)), dtype)
    dg = torch.zeros(C, device="cuda")
    sn = s.float().cpu().numpy()
    dx = o.add_rmsnorm_bwd(dy, s, g, istd, dsk, dg)
    rdx, rdg = oracle.add_rmsnorm_bwd(dyn, sn, gn, istd.cpu().numpy(), dskn)
    assert rel_l2(dx.float().cpu().numpy(), rdx) < tol(dtype)
    assert rel_l2(dg.cpu().numpy(), rdg) < tol(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,F", [(64, 688), (9, 11008), (16, 130)])
@pytest.mark.parametrize("bias", [False, True])
def test_swiglu(rng, dtype, rows, F, bias):
    o = ops()
    gu, gun = dev(rng.standard_normal((rows, 2 * F)), dtype)
    if bias:
        bg = torch.from_numpy((0.1 * rng.standard_normal(F)).astype(np.float32)).cuda()
        bu = torch.from_numpy((0.1 * rng.standard_normal(F)).astype(np.float32)).cuda()
        bgn, bun = bg.cpu().numpy(), bu.cpu().numpy()
    else:
        bg = bu = bgn = bun = None
    h = o.swiglu_fwd(gu, bg, bu)
    rh = oracle.swiglu_fwd(gun, bgn, bun)
    assert rel_l2(h.float().cpu().numpy(), rh) < tol(dtype)
    dh, dhn = dev(rng.standard_normal((rows, F)), dtype)
    dbg = torch.zeros(F, device="cuda") if bias else None
    dbu = torch.zeros(F, device="cuda") if bias else None
    dgu = o.swiglu_bwd(dh, gu, bg, bu, dbg, dbu)
    rdgu, rdbg, rdbu = oracle.swiglu_bwd(dhn, gun, bgn, bun)
    assert rel_l2(dgu.float().cpu().numpy(), rdgu) < tol(dtype)
    if bias:
        assert rel_l2(dbg.cpu().numpy(), rdbg) < tol(dtype)
        assert rel_l2(dbu.cpu().numpy(), rdbu) < tol(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("qknorm,rope,scale", [(False, True, 1.0), (True, True, 1.0), (False, True, 8.0),
                                               (True, False, 1.0)])
@pytest.mark.parametrize("Hq,Hkv,D", [(4, 2, 64), (2, 1, 128)])
def test_qkv_prep(rng, dtype, qknorm, rope, scale, Hq, Hkv, D):
    if qknorm and D != 64:
        pytest.skip("QKNorm is defined for 64-wide heads (src/tkm_registry.c:728-731)")
    o = ops()
    S, B = 48, 2
    rows, C = B * S, (Hq + 2 * Hkv) * D
    x, xn = dev(rng.standard_normal((rows, C)), dtype)
    b = torch.from_numpy((0.1 * rng.standard_normal(C)).astype(np.float32)).cuda()
    gq = torch.from_numpy((1 + 0.1 * rng.standard_normal((Hq + Hkv) * D)).astype(np.float32)).cuda()
    kw = dict(theta=500000.0 if scale > 1 else 10000.0, rope_scale=scale, low=1.0, high=4.0, octx=32.0)
    out, istd = o.qkv_prep_fwd(x, b, gq if qknorm else None, S, Hq, Hkv, D, qknorm, rope, **kw)
    okw = dict(theta=kw["theta"], scale=scale, low=1.0, high=4.0, octx=32.0)
    rout, ristd = oracle.qkv_prep_fwd(xn, b.cpu().numpy(), gq.cpu().numpy() if qknorm else None, S, Hq, Hkv, D,
                                      qknorm, rope, **okw)
    assert rel_l2(out.float().cpu().numpy(), rout) < tol(dtype)
    dout, doutn = dev(rng.standard_normal((rows, C)), dtype)
    din0, din0n = dev(rng.standard_normal((rows, C)), dtype)
    din = din0.clone()
    db = torch.zeros(C, device="cuda")
    dgn = torch.zeros((Hq + Hkv) * D, device="cuda")
    o.qkv_prep_bwd(dout, x, b, gq if qknorm else None, istd, din, S, Hq, Hkv, D, qknorm, rope, **kw,
                   dbias=db, dgain=dgn if qknorm else None)
    rdin, rdb, rdg = oracle.qkv_prep_bwd(doutn, xn, b.cpu().numpy(), gq.cpu().numpy() if qknorm else None,
                                         ristd, S, Hq, Hkv, D, qknorm, rope, **okw)
    # din is accumulated in place: compare the stored result with din0 + J^T dout
    assert rel_l2(din.float().cpu().numpy(), din0n + rdin) < tol(dtype)
    assert rel_l2(db.cpu().numpy(), rdb) < tol(dtype)
    if qknorm:
        assert rel_l2(dgn.cpu().numpy(), rdg) < tol(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("rows,C", [(32, 10), (64, 1024), (7, 32000), (3, 1002)])
def test_softmax(rng, dtype, rows, C):
    o = ops()
    x, xn = dev(2 * rng.standard_normal((rows, C)), dtype)
    p = o.softmax_fwd(x)
    rp = oracle.softmax_fwd(xn)
    assert rel_l2(p.float().cpu().numpy(), rp) < tol(dtype)
    dp, dpn = dev(rng.standard_normal((rows, C)), dtype)
    dx0, dx0n = dev(rng.standard_normal((rows, C)), dtype)
    dx = dx0.clone()
    o.softmax_bwd(p, dp, dx)
    rdx = oracle.softmax_bwd(p.float().cpu().numpy(), dpn, dx0n)
    # dx is accumulated in place (dx += p*(dp - <p,dp>)): compare the stored result
    assert rel_l2(dx.float().cpu().numpy(), rdx) < tol(dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("kind", [0, 1, 2])
@pytest.mark.parametrize("rows,C", [(64, 1024), (5, 32000), (13, 10), (1500, 8192)])
def test_softmax_loss(rng, dtype, kind, rows, C):
    o = ops()
    x, xn = dev(2 * rng.standard_normal((rows, C)), dtype)
    lab = rng.integers(0, C, rows).astype(np.int32)
    lab[0] = int(np.argmax(xn[0]))  # at least one correct prediction
    tl = torch.from_numpy(lab).cuda()
    loss, dl, corr = o.softmax_loss(x, tl, kind, 2.0)
    rloss, rdl, rcorr = oracle.softmax_loss(xn, lab, kind, 2.0)
    assert abs(loss.item() - rloss) <= 1e-5 + (1e-5 if dtype == torch.float32 else 1e-2) * abs(rloss)
    got = dl.float().cpu().numpy()
    if dtype == torch.float16 and kind == 2:
        # Brier gradients are O(1/(C*rows)) and fall into fp16's subnormal range:
        # compare at fp16 resolution instead of relatively
        assert np.abs(got - rdl).max() <= 1e-7 + 1e-2 * np.abs(rdl).max()
    else:
        assert rel_l2(got, rdl) < tol(dtype)
    assert corr.item() == rcorr


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("kind", [0, 1, 2])
@pytest.mark.parametrize("rows,C", [(300, 8200), (7, 32768), (160, 16392)])
def test_softmax_loss_wide_rows_ties(rng, dtype, kind, rows, C):
    """16-bit vocabulary rows (8192 to 32768 wide, ragged against the
    kernel's 4096-element strides, more rows than resident blocks): rows
    whose maximum occurs twice count as correct only for the first index,
    a label on the second occurrence does not."""
    o = ops()
    x, xn = dev(2 * rng.standard_normal((rows, C)), dtype)
    lab = rng.integers(0, C, rows).astype(np.int32)
    host = x.float().cpu().numpy()
    for r in range(0, rows, 3):
        i, j = sorted(rng.choice(C, 2, replace=False))
        host[r, i] = host[r, j] = 20.0
        lab[r] = i if r % 2 == 0 else j
    x = torch.from_numpy(host).to(dtype).cuda()
    xn = x.float().cpu().numpy()
    tl = torch.from_numpy(lab).cuda()
    loss, dl, corr = o.softmax_loss(x, tl, kind, 2.0)
    rloss, rdl, rcorr = oracle.softmax_loss(xn, lab, kind, 2.0)
    assert abs(loss.item() - rloss) <= 1e-5 + 1e-2 * abs(rloss)
    got = dl.float().cpu().numpy()
    if dtype == torch.float16 and kind == 2:
        assert np.abs(got - rdl).max() <= 1e-7 + 1e-2 * np.abs(rdl).max()
    else:
        assert rel_l2(got, rdl) < tol(dtype)
    assert corr.item() == rcorr


def test_sgd(rng):
    o = ops()
    n1, n2 = 1000, 37
    p1 = torch.from_numpy(rng.standard_normal(n1).astype(np.float32)).cuda()
    p2 = torch.from_numpy(rng.standard_normal(n2).astype(np.float32)).cuda()
    v1 = torch.from_numpy(rng.standard_normal(n1).astype(np.float32)).cuda()
    v2 = torch.zeros(n2, device="cuda")
    g1 = torch.from_numpy(rng.standard_normal(n1).astype(np.float32)).cuda()
    g2 = torch.from_numpy(rng.standard_normal(n2).astype(np.float32)).cuda()
    lp1 = torch.empty(n1, dtype=torch.bfloat16, device="cuda")
    r1 = oracle.sgd(p1.cpu().numpy(), v1.cpu().numpy(), g1.cpu().numpy(), 0.05, 0.9, 1e-4, True)
    r2 = oracle.sgd(p2.cpu().numpy(), v2.cpu().numpy(), g2.cpu().numpy(), 0.05, 0.9, 1e-4, False)
    table = o.sgd_table([(p1, v1, g1, lp1, True), (p2, v2, g2, None, False)], "cuda")
    lr = torch.tensor([0.05], device="cuda")
    seed = torch.tensor([0x13579BDF], dtype=torch.int32, device="cuda")
    o.sgd_step(table, 2, lr, 0.9, 1e-4, seed)
    torch.cuda.synchronize()
    assert np.allclose(p1.cpu().numpy(), r1[0], rtol=1e-6, atol=1e-6)
    assert np.allclose(v1.cpu().numpy(), r1[1], rtol=1e-6, atol=1e-6)
    assert np.allclose(p2.cpu().numpy(), r2[0], rtol=1e-6, atol=1e-6)
    assert np.allclose(lp1.float().cpu().numpy(), r1[0], rtol=1e-2, atol=1e-2)
    assert (seed.cpu().numpy().view(np.uint32)[0] == (0x13579BDF + 0x9E3779B9) & 0xFFFFFFFF)
