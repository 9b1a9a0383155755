"""Parity at the benchmark configurations' own shapes (3
and 5), where the full CPU oracle would take minutes: every point runs the
CUDA path at full size and checks sampled heads or rows against the oracle,
or the whole result against an fp32 torch reference on the GPU (tf32 off).

Tolerances (north_star): bf16 within 2e-2 relative L2 on O, dQ, dK, dV and
on the fused row kernels' outputs and gradients, loss within 1 %.
"""
import numpy as np
import pytest

import oracle
from tests.conftest import rel_l2

torch = pytest.importorskip("torch")
pytestmark = [pytest.mark.gpu, pytest.mark.slow]

TOL16 = 2e-2


def _rel(a, b):
    a, b = a.double(), b.double()
    return (torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b)).item()


def attn_reference_group(q, k, v, do, causal, scale, chunk=1024):
    """fp32 attention of one GQA group on the GPU, chunked over queries so
    that S = 16384 fits: q, do [G, S, D] (the group's query heads), k, v
    [S, D].  Returns O [G, S, D], LSE [G, S], dQ [G, S, D] and dK, dV [S, D]
    summed over the group (the GQA gradient)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    q, k, v, do = q.float(), k.float(), v.float(), do.float()
    G, S, D = q.shape
    o = torch.empty_like(q)
    lse = torch.empty(G, S, device=q.device)
    dq = torch.empty_like(q)
    dk = torch.zeros_like(k)
    dv = torch.zeros_like(v)
    cols = torch.arange(S, device=q.device)
    for c0 in range(0, S, chunk):
        c1 = min(S, c0 + chunk)
        kend = c1 if causal else S  # keys past the chunk's last query are all masked
        s = torch.matmul(q[:, c0:c1], k[:kend].T) * scale
        if causal:
            s = s.masked_fill(cols[None, :kend] > torch.arange(c0, c1, device=q.device)[:, None], float("-inf"))
        m = torch.logsumexp(s, dim=-1)
        lse[:, c0:c1] = m
        p = torch.exp(s - m[..., None])
        o[:, c0:c1] = torch.matmul(p, v[:kend])
        delta = (o[:, c0:c1] * do[:, c0:c1]).sum(-1)
        dp = torch.matmul(do[:, c0:c1], v[:kend].T)
        ds = p * (dp - delta[..., None])
        dq[:, c0:c1] = torch.matmul(ds, k[:kend]) * scale
        dk[:kend] += torch.einsum("gqk,gqd->kd", ds, q[:, c0:c1]) * scale
        dv[:kend] += torch.einsum("gqk,gqd->kd", p, do[:, c0:c1])
    return o, lse, dq, dk, dv


def _check_group(o, lse, dqkv, qkv, dout, b, kvh, Hq, Hkv, D, causal, scale):
    """Compare KV group `kvh` of batch `b` (its Hq/Hkv query heads)."""
    S = qkv.shape[1]
    G = Hq // Hkv
    v4 = qkv.view(-1, S, Hq + 2 * Hkv, D)[b]
    d4 = dqkv.view(-1, S, Hq + 2 * Hkv, D)[b]
    hs = slice(kvh * G, (kvh + 1) * G)
    q = v4[:, hs].permute(1, 0, 2)
    do = dout.view(-1, S, Hq, D)[b][:, hs].permute(1, 0, 2)
    ro, rl, rdq, rdk, rdv = attn_reference_group(q, v4[:, Hq + kvh], v4[:, Hq + Hkv + kvh], do, causal, scale)
    got_o = o.view(-1, S, Hq, D)[b][:, hs].permute(1, 0, 2)
    errs = {"O": _rel(got_o.float(), ro), "dQ": _rel(d4[:, hs].permute(1, 0, 2).float(), rdq),
            "dK": _rel(d4[:, Hq + kvh].float(), rdk), "dV": _rel(d4[:, Hq + Hkv + kvh].float(), rdv)}
    for name, e in errs.items():
        assert e < TOL16, (b, kvh, name, e)
    got_lse = lse.view(-1, Hq, S)[b][hs]
    assert (got_lse - rl).abs().max().item() < 1e-2
    return errs


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("S", [512, 1024, 2048, 4096])
@pytest.mark.parametrize("causal", [True, False], ids=["causal", "full"])
def test_config2_attention_sweep_point(S, D, causal):
    """Every point of configuration 2 (B=8, H=16, bf16, fwd+bwd with the dS
    workspace) at its full shape; three (batch, head) pairs against fp32."""
    from tokamak_b200 import ops
    B, H = 8, 16
    g = torch.Generator(device="cuda").manual_seed(1000 + S + D + int(causal))
    qkv = torch.randn(B, S, 3 * H * D, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.randn(B, S, H * D, device="cuda", generator=g).to(torch.bfloat16)
    scale = D ** -0.5
    o, lse = ops.gqa_attn_fwd(qkv, B, S, H, H, D, scale, causal)
    dqkv = ops.gqa_attn_bwd(qkv, o, dout, lse, B, S, H, H, D, scale, causal)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(dqkv).all()
    for b, h in ((0, 0), (3, 9), (7, 15)):
        _check_group(o, lse, dqkv, qkv, dout, b, h, H, H, D, causal, scale)


def test_config5_long_context_group():
    """Configuration 5 at S=16384: B=1, 64 query / 8 KV heads, D=128, causal,
    bf16, full shape (the dS path: 17.3 GB of dS tiles).  KV group 3 -- its 8
    query heads' O and dQ and the group's summed dK, dV -- against fp32."""
    from tokamak_b200 import ops
    B, S, Hq, Hkv, D = 1, 16384, 64, 8, 128
    g = torch.Generator(device="cuda").manual_seed(55)
    qkv = torch.randn(B, S, (Hq + 2 * Hkv) * D, device="cuda", generator=g).to(torch.bfloat16)
    dout = torch.randn(B, S, Hq * D, device="cuda", generator=g).to(torch.bfloat16)
    scale = D ** -0.5
    o, lse = ops.gqa_attn_fwd(qkv, B, S, Hq, Hkv, D, scale, True)
    dqkv = ops.gqa_attn_bwd(qkv, o, dout, lse, B, S, Hq, Hkv, D, scale, True)
    torch.cuda.synchronize()
    assert torch.isfinite(o).all() and torch.isfinite(dqkv).all()
    _check_group(o, lse, dqkv, qkv, dout, 0, 3, Hq, Hkv, D, True, scale)


def test_config3_softmax_ce_8192x32000():
    """The fused softmax cross-entropy (forward + gradient) on configuration
    3's [8192 x 32000] bf16 logits ~ N(0, 2), uniform labels, against the C
    oracle on the same bf16 values."""
    from tokamak_b200 import ops
    rows, C = 8192, 32000
    g = torch.Generator(device="cuda").manual_seed(3)
    logits = (2.0 * torch.randn(rows, C, device="cuda", generator=g)).bfloat16()
    labels = torch.randint(0, C, (rows,), device="cuda", generator=g, dtype=torch.int32)
    loss, dl, corr = ops.softmax_loss(logits, labels, 0, 2.0)
    torch.cuda.synchronize()
    loss, corr = loss.item(), corr.item()
    ref_loss, ref_dl, ref_corr = oracle.softmax_loss(logits.float().cpu().numpy(), labels.cpu().numpy(), 0, 2.0)
    assert abs(loss - ref_loss) <= 1e-2 * abs(ref_loss)
    assert rel_l2(dl.float().cpu().numpy(), ref_dl) < TOL16
    assert corr == ref_corr


def _engine(dsl, params):
    from tokamak_b200 import runtime
    rt = runtime.Runtime.from_dsl(dsl, 1, runtime.DTYPE_BF16)
    rt.load_weights(runtime.tkm1_pack(params))
    return rt


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).bfloat16().float().numpy()


def test_config3_residual_add_rmsnorm_group_16384x4096():
    """The generated plasma group {SiLU branch + residual Add} -> RMSNorm at
    configuration 3's [16384 x 4096] (one fused kernel forward, one backward
    plus the gain-gradient finalize), inside an engine step ending in a
    softmax CE over the 4096 normalised channels, against the float64 graph
    oracle on the whole tensor: normalised output, d(input), d(gain), loss."""
    from oracle.graph_oracle import oracle_for
    from oracle.tkm_abi import bind
    from tokamak_b200 import engine
    dsl = "input: 1x16384x4096\nflow:\n  r: {\n    branch: SiLU\n    skip: Identity\n  } -> Add\n" \
          "  n: RMSNorm -> SoftmaxCE\n"
    rng = np.random.default_rng(9)
    orc = oracle_for(dsl, 1, bind(engine()))
    params = [(1.0 + rng.normal(0, 0.02, n)).astype(np.float32) for _, _, n in orc.tensors]
    orc.set_params([p.astype(np.float64) for p in params])
    x = _bf16(rng.normal(0, 1, orc.rows(0) * orc.C[0]))
    y = rng.integers(0, 4096, orc.rows(0)).astype(np.int32)
    ref = orc.run(x.astype(np.float64), y)
    rt = _engine(dsl, params)
    loss = rt.step(x, y, 0.0)
    n_out = orc.rows(0) * 4096
    assert abs(loss - ref["loss"]) <= 1e-2 * abs(ref["loss"])
    from oracle.graph_oracle import LOSS_OPS
    loss_node = [i for i in range(orc.n) if not orc.nodes[i].dead and orc.nodes[i].op in LOSS_OPS][-1]
    assert rel_l2(rt.logits(n_out), ref["acts"][orc.nodes[loss_node].in0].ravel()) < TOL16
    assert rel_l2(rt.input_grad(), ref["dinput"].ravel()) < TOL16
    (t, (_, _, n)), = list(enumerate(orc.tensors))
    assert rel_l2(rt.param_grad(t, n), ref["grads"][t]) < TOL16
    rt.close()


def test_config3_swiglu_twin_group_16384x11008():
    """The generated SwiGLU twin epilogue (gate and up biases, SiLU(gate) *
    up) on the [16384 x 2*11008] output of the fused twin GEMM, configuration
    3's shape, inside an engine step ending in a softmax CE over the 11008
    channels.  Reference: the same graph in fp32 torch on the GPU from the
    same bf16 input and bf16 GEMM weights (tf32 off): loss, h, d(input) and
    the two bias gradients."""
    from oracle.graph_oracle import oracle_for
    from oracle.tkm_abi import bind
    from tokamak_b200 import engine
    torch.backends.cuda.matmul.allow_tf32 = False
    R, K, F = 16384, 256, 11008
    dsl = f"input: 1x{R}x{K}\nflow:\n  f: {{\n    gate: FC({F}) -> SiLU\n    up: FC({F})\n  }} -> Mul -> SoftmaxCE\n"
    orc = oracle_for(dsl, 1, bind(engine()))
    rng = np.random.default_rng(10)
    params = [(rng.normal(0, 0.05, n) if k == 0 else rng.normal(0, 0.5, n)).astype(np.float32)
              for _, k, n in orc.tensors]
    x = _bf16(rng.normal(0, 1, R * K))
    y = rng.integers(0, F, R).astype(np.int32)
    rt = _engine(dsl, params)
    loss = rt.step(x, y, 0.0)
    h_got = torch.from_numpy(rt.logits(R * F)).cuda().view(R, F)
    dx_got = torch.from_numpy(rt.input_grad()).cuda().view(R, K)
    ti = {(node, kind): t for t, (node, kind, _) in enumerate(orc.tensors)}
    twin = [i for i in range(orc.n) if not orc.nodes[i].dead and orc.nodes[i].left_len > 0][0]
    fc = orc.nodes[twin].in0
    bg_t = ti[(orc.nodes[twin].left_nodes[0], 3)]
    bu_t = ti[(orc.nodes[twin].right_nodes[0], 3)]
    dbg_got = torch.from_numpy(rt.param_grad(bg_t, F)).cuda()
    dbu_got = torch.from_numpy(rt.param_grad(bu_t, F)).cuda()
    rt.close()
    # fp32 reference from the bf16 values the engine used
    W = torch.from_numpy(params[ti[(fc, 0)]]).cuda().view(K, 2 * F).bfloat16().float()
    xt = torch.from_numpy(x).cuda().view(R, K).requires_grad_()
    bg = torch.from_numpy(params[bg_t]).cuda().requires_grad_()
    bu = torch.from_numpy(params[bu_t]).cuda().requires_grad_()
    gu = (xt @ W).bfloat16().float()  # the GEMM writes bf16
    h = torch.nn.functional.silu(gu[:, :F] + bg) * (gu[:, F:] + bu)
    ref_loss = torch.nn.functional.cross_entropy(h, torch.from_numpy(y).long().cuda())
    ref_loss.backward()
    assert abs(loss - ref_loss.item()) <= 1e-2 * abs(ref_loss.item())
    assert _rel(h_got, h.detach()) < TOL16
    assert _rel(dx_got, xt.grad) < TOL16
    assert _rel(dbg_got, bg.grad) < TOL16
    assert _rel(dbu_got, bu.grad) < TOL16
