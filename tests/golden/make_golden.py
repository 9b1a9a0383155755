"""Generate golden vectors from the REFERENCE implementation itself.

Runs on a GPU box: loads oracle/_ref/libtkm_ref.so (the reference's own
src/tkm_gpu.cu, registry, DSL core and codegen, built by oracle/build_ref.py
for sm_100a) and records seeded inputs and the reference's outputs:

  attn_*.npz      k_gqa_flash_attn_tc_fwd / _bwd (fp16 WMMA) via ref_attn_*
  loss_*.npz      k_softmax_loss_fwd_bwd_h (CE, focal, Brier)
  softmax.npz     k_softmax_fwd_h / k_softmax_bwd_h
  rmsnorm_c64.npz the reference runtime (tkm_load_string + NVRTC plasma
                  group) on "RMSNorm", C = 64 (the width the reference's
                  warp reduction handles correctly)
  silu_add.npz    the runtime on "{ branch: SiLU, skip: Identity } -> Add"

Inputs are rounded to fp16 before use and stored as float32, so the CPU
oracle sees exactly the values the reference saw.  Usage:

    python tests/golden/make_golden.py OUTDIR
"""
import ctypes
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main(outdir):
    import torch
    os.makedirs(outdir, exist_ok=True)
    L = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libtkm_ref.so"))
    vp = ctypes.c_void_p
    P = lambda t: vp(t.data_ptr())  # noqa: E731
    rng = np.random.default_rng(20261201)

    def h16(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().half()

    # ---------------------------------------------------------------- attention
    for (B, S, Hq, Hkv, D, causal) in [(1, 128, 2, 1, 64, 1), (2, 96, 4, 2, 128, 0), (1, 77, 2, 2, 64, 1)]:
        scale = D ** -0.5
        qkv = h16(rng.standard_normal((B, S, (Hq + 2 * Hkv) * D)))
        dout = h16(rng.standard_normal((B, S, Hq * D)))
        out = torch.zeros(B, S, Hq * D, dtype=torch.half, device="cuda")
        lse = torch.zeros(B * Hq, S, dtype=torch.float32, device="cuda")
        assert L.ref_attn_fwd(P(qkv), P(out), P(lse), B, S, Hq, Hkv, D, ctypes.c_float(scale), causal, None) == 0
        dqkv = torch.zeros_like(qkv)
        assert L.ref_attn_bwd(P(qkv), P(out), P(dout), P(lse), P(dqkv), B, S, Hq, Hkv, D, ctypes.c_float(scale),
                              causal, None) == 0
        torch.cuda.synchronize()
        np.savez_compressed(os.path.join(outdir, f"attn_b{B}_s{S}_h{Hq}x{Hkv}_d{D}_c{causal}.npz"),
                            qkv=qkv.float().cpu().numpy(), dout=dout.float().cpu().numpy(),
                            out=out.float().cpu().numpy(), lse=lse.cpu().numpy(), dqkv=dqkv.float().cpu().numpy(),
                            shape=np.array([B, S, Hq, Hkv, D, causal]), scale=np.float32(scale))

    # ---------------------------------------------------------------- losses
    rows, C = 64, 200
    logits = h16(2.0 * rng.standard_normal((rows, C)))
    labels = rng.integers(0, C, rows).astype(np.uint8)
    labels[0] = np.argmax(logits[0].float().cpu().numpy())
    tl = torch.from_numpy(labels).cuda()
    for kind, gamma in ((0, 0.0), (1, 2.0), (2, 0.0)):
        dl = torch.zeros_like(logits)
        loss = torch.zeros(1, dtype=torch.float32, device="cuda")
        corr = torch.zeros(1, dtype=torch.int32, device="cuda")
        assert L.ref_softmax_loss(P(logits), P(tl), P(dl), P(loss), P(corr), rows, C, kind, ctypes.c_float(gamma),
                                  None) == 0
        torch.cuda.synchronize()
        np.savez_compressed(os.path.join(outdir, f"loss_kind{kind}.npz"), logits=logits.float().cpu().numpy(),
                            labels=labels.astype(np.int32), loss=loss.cpu().numpy(), dlogits=dl.float().cpu().numpy(),
                            correct=corr.cpu().numpy(), kind=np.int32(kind), gamma=np.float32(gamma))

    # ---------------------------------------------------------------- softmax
    x = h16(rng.standard_normal((32, 48)))
    p = torch.zeros_like(x)
    assert L.ref_softmax_fwd(P(x), P(p), 32, 48, None) == 0
    dp = h16(rng.standard_normal((32, 48)))
    dx0 = h16(0.1 * rng.standard_normal((32, 48)))
    dx = dx0.clone()
    assert L.ref_softmax_bwd(P(p), P(dp), P(dx), 32, 48, None) == 0
    torch.cuda.synchronize()
    np.savez_compressed(os.path.join(outdir, "softmax.npz"), x=x.float().cpu().numpy(), p=p.float().cpu().numpy(),
                        dp=dp.float().cpu().numpy(), dx0=dx0.float().cpu().numpy(), dx=dx.float().cpu().numpy())

    # ---------------------------------------------------------------- runtime (NVRTC plasma groups)
    L.tkm_load_string.restype = vp
    L.tkm_load_string.argtypes = [ctypes.c_char_p, ctypes.c_int]
    L.tkm_runtime_forward.restype = ctypes.c_size_t
    L.tkm_runtime_forward.argtypes = [vp, vp, vp, ctypes.c_size_t]
    L.tkm_runtime_free.argtypes = [vp]
    for name, dsl in (("rmsnorm_c64", b"input: 1x4x64\nflow:\n  n: RMSNorm\n"),
                      ("silu_add", b"input: 1x4x64\nflow:\n  r: {\n    branch: SiLU\n    skip: Identity\n  } -> Add\n")):
        batch = 3
        rt = L.tkm_load_string(dsl, batch)
        assert rt
        xin = np.round(rng.standard_normal((batch, 4, 64)).astype(np.float16)).astype(np.float32) \
            if False else rng.standard_normal((batch, 4, 64)).astype(np.float16).astype(np.float32)
        yout = np.zeros_like(xin)
        n = L.tkm_runtime_forward(rt, xin.ctypes.data_as(vp), yout.ctypes.data_as(vp), yout.size)
        assert n == yout.size, n
        L.tkm_runtime_free(rt)
        np.savez_compressed(os.path.join(outdir, f"{name}.npz"), x=xin, y=yout)
    print("golden vectors written to", outdir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden"))
