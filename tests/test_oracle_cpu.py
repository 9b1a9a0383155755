"""The CPU oracle checked against independent numpy restatements and
finite differences (the reference's own verification method: central
differences, src/main.c:202-304).  Runs without a GPU."""
import numpy as np
import pytest

import oracle
from tests.conftest import rel_l2


# ------------------------------------------------------------------ numpy references
def np_attn_fwd(qkv, B, S, Hq, Hkv, D, scale, causal):
    qkv = qkv.astype(np.float64).reshape(B, S, Hq + 2 * Hkv, D)
    G = Hq // Hkv
    out = np.zeros((B, S, Hq, D))
    lse = np.zeros((B, Hq, S))
    for b in range(B):
        for h in range(Hq):
            q, k, v = qkv[b, :, h], qkv[b, :, Hq + h // G], qkv[b, :, Hq + Hkv + h // G]
            s = q @ k.T * scale
            if causal:
                s = np.where(np.triu(np.ones((S, S), bool), 1), -np.inf, s)
            m = s.max(1, keepdims=True)
            p = np.exp(s - m)
            l = p.sum(1, keepdims=True)
            out[b, :, h] = (p @ v) / (l + 1e-8)
            lse[b, h] = (m + np.log(l + 1e-8))[:, 0]
    return out.reshape(B, S, Hq * D), lse.reshape(B * Hq, S)


def attn_case(rng, B, S, Hq, Hkv, D):
    return rng.standard_normal((B, S, (Hq + 2 * Hkv) * D)).astype(np.float32)


@pytest.mark.parametrize("B,S,Hq,Hkv,D,causal", [(1, 17, 2, 1, 8, True), (2, 33, 4, 2, 16, False),
                                                   (1, 40, 3, 3, 8, True)])
def test_attn_fwd_vs_numpy(rng, B, S, Hq, Hkv, D, causal):
    qkv = attn_case(rng, B, S, Hq, Hkv, D)
    o, l = oracle.attn_fwd(qkv, B, S, Hq, Hkv, D, D ** -0.5, causal)
    ro, rl = np_attn_fwd(qkv, B, S, Hq, Hkv, D, D ** -0.5, causal)
    assert rel_l2(o, ro) < 1e-6
    assert np.abs(l - rl).max() < 1e-5


@pytest.mark.parametrize("causal", [True, False])
def test_attn_bwd_finite_differences(rng, causal):
    B, S, Hq, Hkv, D = 1, 12, 4, 2, 8
    qkv = attn_case(rng, B, S, Hq, Hkv, D)
    W = rng.standard_normal((B, S, Hq * D)).astype(np.float32)   # L = sum(O * W) -> dO = W
    sc = D ** -0.5
    o, l = oracle.attn_fwd(qkv, B, S, Hq, Hkv, D, sc, causal)
    d = oracle.attn_bwd(qkv, o, W, l, B, S, Hq, Hkv, D, sc, causal)

    def loss(x):
        ox, _ = np_attn_fwd(x, B, S, Hq, Hkv, D, sc, causal)
        return float((ox * W).sum())

    eps = 1e-3
    idx = rng.choice(qkv.size, 40, replace=False)
    for i in idx:
        xp = qkv.astype(np.float64).copy().ravel()
        xm = xp.copy()
        xp[i] += eps
        xm[i] -= eps
        num = (loss(xp.reshape(qkv.shape)) - loss(xm.reshape(qkv.shape))) / (2 * eps)
        ana = d.ravel()[i]
        assert abs(num - ana) <= 5e-3 * max(1.0, abs(num)), (i, num, ana)


def test_attn_bwd_gqa_sums_group(rng):
    """dK/dV of a shared kv head = sum of the per-query-head contributions."""
    B, S, D = 1, 16, 8
    qkv = attn_case(rng, B, S, 2, 1, D)
    W = rng.standard_normal((B, S, 2 * D)).astype(np.float32)
    o, l = oracle.attn_fwd(qkv, B, S, 2, 1, D, 0.3, True)
    d = oracle.attn_bwd(qkv, o, W, l, B, S, 2, 1, D, 0.3, True)
    parts = []
    for h in range(2):
        sub = np.concatenate([qkv[..., h * D:(h + 1) * D], qkv[..., 2 * D:4 * D]], -1)
        so, sl = oracle.attn_fwd(np.ascontiguousarray(sub), B, S, 1, 1, D, 0.3, True)
        parts.append(oracle.attn_bwd(np.ascontiguousarray(sub), so, np.ascontiguousarray(W[..., h * D:(h + 1) * D]),
                                     sl, B, S, 1, 1, D, 0.3, True))
    assert np.allclose(d[..., 2 * D:], parts[0][..., D:] + parts[1][..., D:], atol=1e-5)


# ------------------------------------------------------------------ rows
def num_grad(f, x, idx, eps=1e-3):
    xp = x.astype(np.float64).copy()
    xm = xp.copy()
    xp.flat[idx] += eps
    xm.flat[idx] -= eps
    return (f(xp) - f(xm)) / (2 * eps)


def test_add_rmsnorm(rng):
    rows, C = 5, 48
    x = rng.standard_normal((rows, C)).astype(np.float32)
    r = rng.standard_normal((rows, C)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(C)).astype(np.float32)
    s, y, istd = oracle.add_rmsnorm_fwd(x, r, g)
    sn = x.astype(np.float64) + r
    ref = sn / np.sqrt((sn ** 2).mean(1, keepdims=True) + 1e-5) * g
    assert rel_l2(y, ref) < 1e-6
    W = rng.standard_normal((rows, C)).astype(np.float32)
    skip = rng.standard_normal((rows, C)).astype(np.float32)
    dx, dg = oracle.add_rmsnorm_bwd(W, s, g, istd, skip)

    def L(sv):
        return float((sv / np.sqrt((sv ** 2).mean(1, keepdims=True) + 1e-5) * g * W).sum() + (sv * skip).sum())
    for i in rng.choice(s.size, 20, replace=False):
        assert abs(num_grad(L, s, i) - dx.flat[i]) < 5e-3 * max(1, abs(dx.flat[i]))
    xh = s / np.sqrt((s.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-5)
    assert rel_l2(dg, (W * xh).sum(0)) < 1e-5


def test_swiglu_matches_numcheck_points():
    """SiLU derivative at the reference's numcheck points (src/main.c:214-225):
    x in {-1.6, -0.4, 0.5, 1.4}, dy = 1.3, eps = 1e-3, tolerance 5e-3."""
    pts = np.array([-1.6, -0.4, 0.5, 1.4], np.float32)
    gu = np.stack([pts, np.ones(4, np.float32)], 0).T.reshape(4, 2).astype(np.float32)  # F = 1, up = 1
    dh = np.full((4, 1), 1.3, np.float32)
    dgu, _, _ = oracle.swiglu_bwd(dh, np.ascontiguousarray(gu))
    eps = 1e-3
    for i, x in enumerate(pts.astype(np.float64)):
        silu = lambda a: a / (1 + np.exp(-a))  # noqa: E731
        num = 1.3 * (silu(x + eps) - silu(x - eps)) / (2 * eps)
        assert abs(dgu[i, 0] - num) / max(1.0, abs(num)) < 5e-3


def test_swiglu_finite_differences(rng):
    rows, F = 4, 6
    gu = rng.standard_normal((rows, 2 * F)).astype(np.float32)
    bg = (0.1 * rng.standard_normal(F)).astype(np.float32)
    bu = (0.1 * rng.standard_normal(F)).astype(np.float32)
    W = rng.standard_normal((rows, F)).astype(np.float32)
    h = oracle.swiglu_fwd(gu, bg, bu)
    a, b = gu[:, :F].astype(np.float64) + bg, gu[:, F:].astype(np.float64) + bu
    assert rel_l2(h, a / (1 + np.exp(-a)) * b) < 1e-6
    dgu, dbg, dbu = oracle.swiglu_bwd(W, gu, bg, bu)

    def L(x):
        aa, bb = x[:, :F] + bg, x[:, F:] + bu
        return float((aa / (1 + np.exp(-aa)) * bb * W).sum())
    for i in range(gu.size):
        assert abs(num_grad(L, gu, i) - dgu.flat[i]) < 1e-4
    assert rel_l2(dbg, dgu[:, :F].sum(0)) < 1e-5 and rel_l2(dbu, dgu[:, F:].sum(0)) < 1e-5


@pytest.mark.parametrize("qknorm", [False, True])
@pytest.mark.parametrize("scale", [1.0, 8.0])
def test_qkv_prep(rng, qknorm, scale):
    S, B, Hq, Hkv, D = 6, 2, 2, 1, 8
    rows, C = S * B, (Hq + 2 * Hkv) * D
    x = rng.standard_normal((rows, C)).astype(np.float32)
    bias = (0.1 * rng.standard_normal(C)).astype(np.float32)
    gain = (1 + 0.1 * rng.standard_normal((Hq + Hkv) * D)).astype(np.float32)
    kw = dict(theta=10000.0, scale=scale, low=1.0, high=4.0, octx=4.0)
    out, istd = oracle.qkv_prep_fwd(x, bias, gain, S, Hq, Hkv, D, qknorm, True, **kw)
    # V columns pass through with the bias only
    assert np.allclose(out[:, (Hq + Hkv) * D:], x[:, (Hq + Hkv) * D:] + bias[(Hq + Hkv) * D:], atol=1e-6)
    # row 0 is position 0: no rotation
    if not qknorm:
        assert np.allclose(out[0], x[0] + bias, atol=1e-6)
    W = rng.standard_normal((rows, C)).astype(np.float32)
    din, db, dgn = oracle.qkv_prep_bwd(W, x, bias, gain, istd, S, Hq, Hkv, D, qknorm, True, **kw)

    def L(xv):
        o, _ = oracle.qkv_prep_fwd(xv.astype(np.float32), bias, gain, S, Hq, Hkv, D, qknorm, True, **kw)
        return float((o.astype(np.float64) * W).sum())
    for i in rng.choice(x.size, 24, replace=False):
        assert abs(num_grad(L, x, i, 1e-2) - din.flat[i]) < 2e-2 * max(1, abs(din.flat[i]))
    assert rel_l2(db, din.sum(0)) < 1e-5


def test_rope_convention_pair_frequencies():
    """Pair i of a head rotates by pos * theta^(-i/D) (src/tkm_codegen.c:45)."""
    S, D = 5, 8
    x = np.zeros((S, 3 * D), np.float32)
    x[:, 0:D:2] = 1.0   # every pair of the Q head = (1, 0)
    out, _ = oracle.qkv_prep_fwd(x, None, None, S, 1, 1, D, False, True, theta=10000.0)
    for pos in range(S):
        for i in range(D // 2):
            ang = pos * 10000.0 ** (-i / D)
            assert abs(out[pos, 2 * i] - np.cos(ang)) < 1e-6
            assert abs(out[pos, 2 * i + 1] - np.sin(ang)) < 1e-6


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_softmax_loss_finite_differences(rng, kind):
    rows, C = 3, 7
    x = (2 * rng.standard_normal((rows, C))).astype(np.float32)
    lab = rng.integers(0, C, rows).astype(np.int32)
    loss, dl, corr = oracle.softmax_loss(x, lab, kind, 2.0)
    assert corr == int((x.argmax(1) == lab).sum())

    def L(xv):
        return oracle.softmax_loss(xv.astype(np.float32), lab, kind, 2.0)[0]
    if kind == 1:
        # focal loss value: mean of -(1-pt)^gamma ln(pt) (src/tkm_gpu.cu:651-667); the
        # reference's gradient scale (src/tkm_gpu.cu:652-654) is its exact derivative
        pt = np.exp(x - x.max(1, keepdims=True))
        pt /= pt.sum(1, keepdims=True)
        ptl = np.maximum(pt[np.arange(rows), lab], 1e-7)
        ref = float((-(1 - ptl) ** 2 * np.log(ptl)).mean())
        assert abs(loss - ref) < 1e-5
    for i in range(x.size):
        assert abs(num_grad(L, x, i, 1e-2) - dl.flat[i]) < 2e-3


def test_softmax_vjp(rng):
    x = rng.standard_normal((4, 9)).astype(np.float32)
    p = oracle.softmax_fwd(x)
    e = np.exp(x - x.max(1, keepdims=True))
    assert rel_l2(p, e / e.sum(1, keepdims=True)) < 1e-6
    dp = rng.standard_normal((4, 9)).astype(np.float32)
    dx = oracle.softmax_bwd(p, dp, np.zeros_like(p))
    J = p.astype(np.float64)[..., None] * (np.eye(9) - p[:, None, :])
    assert rel_l2(dx, np.einsum("rij,rj->ri", J.transpose(0, 2, 1), dp)) < 1e-5


def test_sgd_reference_update(rng):
    p = rng.standard_normal(10).astype(np.float32)
    v = rng.standard_normal(10).astype(np.float32)
    g = rng.standard_normal(10).astype(np.float32)
    p1, v1 = oracle.sgd(p, v, g, 0.1, 0.9, 1e-4, True)
    gg = g + 1e-4 * p
    vv = 0.9 * v + gg
    assert np.allclose(v1, vv, atol=1e-6)
    assert np.allclose(p1, p - 0.1 * (0.9 * vv + gg), atol=1e-6)
