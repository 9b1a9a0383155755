"""Pin the CPU oracle against golden vectors produced by the REFERENCE itself.

tests/golden/*.npz were written by tests/golden/make_golden.py running the
reference's own kernels and runtime (oracle/_ref/libtkm_ref.so, built from
the reference's src/ for sm_100a by oracle/build_ref.py) on a B200.  Inputs are fp16-exact, the
reference computes in fp16 storage with fp32 accumulation (P rounded to fp16
inside its attention), so the oracle must agree to fp16 precision:
1e-2 relative L2 on tensors, 1e-3 relative on scalar losses.
"""
import glob
import os

import numpy as np
import pytest

import oracle
from tests.conftest import rel_l2

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def files(prefix):
    out = sorted(glob.glob(os.path.join(GOLD, prefix + "*.npz")))
    assert out, f"no golden vectors {prefix}* (generate with tests/golden/make_golden.py on a GPU box)"
    return out


@pytest.mark.parametrize("path", files("attn_"))
def test_attention_forward_matches_reference(path):
    z = np.load(path)
    B, S, Hq, Hkv, D, causal = (int(v) for v in z["shape"])
    o, lse = oracle.attn_fwd(z["qkv"], B, S, Hq, Hkv, D, float(z["scale"]), causal)
    assert rel_l2(o, z["out"]) < 1e-2
    assert np.abs(lse - z["lse"]).max() < 5e-3


@pytest.mark.parametrize("path", files("attn_"))
def test_attention_dq_matches_reference(path):
    """The reference's dQ math (src/tkm_gpu.cu:503-564) is right, but its
    read-back of each 16x16 dQ fragment is not: the fragment is stored with
    leading dimension 16 (src/tkm_gpu.cu:569) and read as s_s[warp][lane][c],
    whose rows are SMEM_PAD_16 = 24 floats apart (src/tkm_gpu.cu:573).  Row
    `lane` of every 16-row warp tile therefore receives flat element
    lane*24 + c of the stored fragment; lanes >= 11 read past it.  The oracle's
    true dQ, pushed through that same mapping, must reproduce the reference's
    output for lanes 0..10 (row 0 of each tile is the only unshifted one)."""
    z = np.load(path)
    B, S, Hq, Hkv, D, causal = (int(v) for v in z["shape"])
    d = oracle.attn_bwd(z["qkv"], z["out"], z["dout"], z["lse"], B, S, Hq, Hkv, D, float(z["scale"]), causal)
    true_dq = d.reshape(B, S, Hq + 2 * Hkv, D)[:, :, :Hq]
    ref = z["dqkv"].reshape(B, S, Hq + 2 * Hkv, D)[:, :, :Hq]
    mapped, got = [], []
    for q_base in range(0, S, 16):
        for lane in range(11):
            r = q_base + lane
            if r >= S:
                continue
            for blk in range(D // 16):
                for c in range(16):
                    off = lane * 24 + c
                    src = q_base + off // 16
                    if src >= S:
                        continue
                    mapped.append(true_dq[:, src, :, blk * 16 + off % 16])
                    got.append(ref[:, r, :, blk * 16 + c])
    mapped, got = np.array(mapped), np.array(got)
    assert rel_l2(got, mapped) < 1e-2
    # row 0 of every warp tile is the true dQ row
    rows0 = np.arange(0, S, 16)
    assert rel_l2(ref[:, rows0], true_dq[:, rows0]) < 1e-2


@pytest.mark.parametrize("path", files("attn_"))
def test_attention_dkdv_reference_defect_is_documented(path):
    """The reference writes dK := dQ and dV := dO for the first query head of
    each group (src/tkm_gpu.cu:588-596).  The oracle deliberately differs:
    this test pins that the golden data show the defect, and that the
    oracle's dK/dV are the true gradients (checked by finite differences in
    test_oracle_cpu.py)."""
    z = np.load(path)
    B, S, Hq, Hkv, D, causal = (int(v) for v in z["shape"])
    G = Hq // Hkv
    ref = z["dqkv"].reshape(B, S, Hq + 2 * Hkv, D)
    dout = z["dout"].reshape(B, S, Hq, D)
    for g in range(Hkv):
        assert np.allclose(ref[:, :, Hq + g], ref[:, :, g * G], atol=1e-3)      # dK == dQ of head g*G
        assert np.allclose(ref[:, :, Hq + Hkv + g], dout[:, :, g * G], atol=1e-3)  # dV == dO


@pytest.mark.parametrize("path", files("loss_"))
def test_softmax_losses_match_reference(path):
    z = np.load(path)
    kind, gamma = int(z["kind"]), float(z["gamma"])
    loss, dl, corr = oracle.softmax_loss(z["logits"], z["labels"].astype(np.int32), kind, gamma)
    ref_loss = float(z["loss"][0])
    assert abs(loss - ref_loss) <= 1e-3 * abs(ref_loss) + 1e-6
    # the reference stores dlogits in fp16: compare in absolute terms at fp16 resolution
    assert np.abs(dl - z["dlogits"]).max() < 2e-5 + 2e-3 * np.abs(z["dlogits"]).max()
    assert corr == int(z["correct"][0])


def test_softmax_matches_reference():
    z = np.load(os.path.join(GOLD, "softmax.npz"))
    p = oracle.softmax_fwd(z["x"])
    assert rel_l2(p, z["p"]) < 2e-3
    dx = oracle.softmax_bwd(z["p"], z["dp"], z["dx0"])
    assert rel_l2(dx, z["dx"]) < 1e-2


def test_rmsnorm_matches_reference_runtime():
    """The reference runtime's NVRTC RMSNorm group at C = 64 (gain 1, eps 1e-5)."""
    z = np.load(os.path.join(GOLD, "rmsnorm_c64.npz"))
    x = z["x"].reshape(-1, 64)
    _, y, _ = oracle.add_rmsnorm_fwd(x, None, np.ones(64, np.float32))
    assert rel_l2(y, z["y"].reshape(-1, 64)) < 2e-3


def test_silu_residual_matches_reference_runtime():
    """{ branch: SiLU, skip: Identity } -> Add through the reference runtime."""
    z = np.load(os.path.join(GOLD, "silu_add.npz"))
    x = z["x"].reshape(-1, 64).astype(np.float64)
    # SiLU via the oracle's SwiGLU with up = 1, plus the residual
    gu = np.concatenate([x, np.ones_like(x)], 1).astype(np.float32)
    h = oracle.swiglu_fwd(np.ascontiguousarray(gu))
    assert rel_l2(h + x, z["y"].reshape(-1, 64)) < 2e-3


@pytest.mark.parametrize("path", files("qkvprep_"))
def test_qkv_prep_matches_reference_runtime(path):
    """The reference runtime's fused QKV-prep group (bias, optional per-head
    QKNorm, RoPE on the Q and K channels; src/tkm_codegen.c:43-70, 211-295)
    inside a GQA graph, fed with the fused GEMM output it saw.  The bias and
    the QKNorm gain come from the TKM1 weights the reference ran with, found
    through the graph's tensor registration order.  The reference stores fp16
    and uses fast-math exponentials and sincos, so the bound is fp16-level;
    a different pair convention or frequency rule is off by O(1)."""
    from oracle.graph_oracle import oracle_for, reference_front_end
    from tokamak_b200.runtime import tkm1_unpack
    z = np.load(path)
    S, Hq, Hkv, D, qkn = (int(v) for v in z["shape"])
    front = reference_front_end()
    if front is None:
        pytest.skip("reference host library not built (oracle/build_ref.py)")
    orc = oracle_for(str(z["dsl"]), int(z["batch"]), front)
    tensors = tkm1_unpack(z["weights"].tobytes())
    assert [t.size for t in tensors] == [n for _, _, n in orc.tensors]
    pid = int(z["prep_node"])
    bias = tensors[orc.tidx[(pid, 3)]]
    gain = tensors[orc.tidx[(pid, 1)]]
    rope = dict(zip(("theta", "scale", "low", "high", "octx"), (float(v) for v in z["rope"])))
    out, _ = oracle.qkv_prep_fwd(z["prep_in"], bias, gain, S, Hq, Hkv, D, bool(qkn), True, **rope)
    ref = z["prep_out"]
    assert rel_l2(out, ref) < 2e-3
    assert np.abs(out - ref).max() < 1e-2 * np.abs(ref).max()
    # V channels pass through with the bias only
    qk = (Hq + Hkv) * D
    assert np.abs(out[:, qk:] - ref[:, qk:]).max() <= 2e-3 * np.abs(ref[:, qk:]).max()


def test_sgd_matches_reference_kernel():
    """k_tkm_multi_tensor_sgd (src/tkm_gpu.cu:695-720) on three tensors: the
    oracle repeats its fmaf chain, so masters and velocities agree bit for
    bit; the fp16 GEMM copy is the master rounded to nearest; the seed
    advances by 0x9E3779B9."""
    z = np.load(os.path.join(GOLD, "sgd.npz"))
    lr, mom, wd = float(z["lr"]), float(z["momentum"]), float(z["wd"])
    for i, has16 in enumerate(z["fp16_copy"]):
        p, v = oracle.sgd(z[f"p0_{i}"], z[f"v0_{i}"], z[f"g_{i}"], lr, mom, wd, apply_wd=bool(has16))
        assert np.array_equal(p, z[f"p1_{i}"]), i
        assert np.array_equal(v, z[f"v1_{i}"]), i
        if has16:
            assert np.array_equal(p.astype(np.float16).astype(np.float32), z[f"h1_{i}"])
    assert int(z["seed_out"]) == (int(z["seed_in"]) + 0x9E3779B9) & 0xFFFFFFFF
