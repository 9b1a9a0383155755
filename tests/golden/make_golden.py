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
  qkvprep_*.npz   the runtime's fused QKV-prep group (NVRTC, emitted by
                  emit_qkv_prep_plasma_group / emit_rope_rotation) inside a
                  GQA graph: its input (the fused [Q|K|V] GEMM output), its
                  output, and the TKM1 weights it ran with (random bias and
                  QKNorm gain loaded with tkm_load_weights_buffer)
  sgd.npz         k_tkm_multi_tensor_sgd on three tensors, one with an fp16
                  GEMM copy (weight decay applies to it only)

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

    # ---------------------------------------------------------------- runtime: fused QKV prep + RoPE
    L.tkm_runtime_weight_bytes.restype = ctypes.c_size_t
    L.tkm_runtime_weight_bytes.argtypes = [vp]
    L.tkm_save_weights_buffer.argtypes = [vp, vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]
    L.tkm_load_weights_buffer.argtypes = [vp, vp, ctypes.c_size_t]
    L.ref_qkv_prep_acts.argtypes = [vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), vp, vp,
                                    ctypes.c_size_t]
    for name, S, dm, Hq, Hkv, D, qkn, rope in qkv_prep_cases():
        dsl = qkv_prep_dsl(S, dm, Hq, Hkv, D, qkn, rope).encode()
        batch = 2
        rt = L.tkm_load_string(dsl, batch)
        assert rt, name
        nb = L.tkm_runtime_weight_bytes(rt)
        buf = np.zeros(nb, np.uint8)
        size = ctypes.c_size_t(0)
        assert L.tkm_save_weights_buffer(rt, buf.ctypes.data_as(vp), nb, ctypes.byref(size)) == 1
        tensors = tkm1_unpack(buf[:size.value].tobytes())
        # every vector tensor (biases, QKNorm gains) random, GEMM weights as the reference drew them
        tensors = [t if t.size > 4 * dm else (rng.normal(0.0, 0.5, t.size) + (1.0 if i % 2 else 0.0)).astype(np.float32)
                   for i, t in enumerate(tensors)]
        blob = tkm1_pack(tensors)
        arr = np.frombuffer(blob, np.uint8).copy()
        assert L.tkm_load_weights_buffer(rt, arr.ctypes.data_as(vp), arr.size) == 1
        xin = (2.0 * rng.standard_normal((batch, S, dm))).astype(np.float16).astype(np.float32)
        yout = np.zeros(batch * S * Hq * D, np.float32)
        assert L.tkm_runtime_forward(rt, xin.ctypes.data_as(vp), yout.ctypes.data_as(vp), yout.size) == yout.size
        C = (Hq + 2 * Hkv) * D
        h_in = np.zeros(batch * S * C, np.float16)
        h_out = np.zeros(batch * S * C, np.float16)
        gid, pid = ctypes.c_int(-1), ctypes.c_int(-1)
        assert L.ref_qkv_prep_acts(rt, ctypes.byref(gid), ctypes.byref(pid), h_in.ctypes.data_as(vp),
                                   h_out.ctypes.data_as(vp), h_in.size) == 0
        L.tkm_runtime_free(rt)
        np.savez_compressed(os.path.join(outdir, f"{name}.npz"), dsl=np.array(dsl.decode()), batch=np.int32(batch),
                            weights=arr, prep_in=h_in.astype(np.float32).reshape(batch * S, C),
                            prep_out=h_out.astype(np.float32).reshape(batch * S, C), prep_node=np.int32(pid.value),
                            shape=np.array([S, Hq, Hkv, D, qkn]),
                            rope=np.array([rope["theta"], rope.get("scale", 1.0), rope.get("low_freq_factor", 1.0),
                                           rope.get("high_freq_factor", 4.0),
                                           rope.get("original_context_length", 8192.0)]))

    # ---------------------------------------------------------------- SGD
    sizes = [1000, 37, 4096]
    fp16_copy = [True, False, False]
    masters = [torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda() for n in sizes]
    vels = [torch.from_numpy((0.1 * rng.standard_normal(n)).astype(np.float32)).cuda() for n in sizes]
    grads = [torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda() for n in sizes]
    halves = [torch.zeros(n, dtype=torch.half, device="cuda") if h else None for n, h in zip(sizes, fp16_copy)]
    p0 = [m.cpu().numpy() for m in masters]
    v0 = [v.cpu().numpy() for v in vels]
    lr = torch.tensor([0.01], dtype=torch.float32, device="cuda")
    seed = torch.tensor([12345], dtype=torch.int32, device="cuda")
    PA = ctypes.c_void_p * 3
    assert L.ref_sgd(PA(*[m.data_ptr() for m in masters]), PA(*[h.data_ptr() if h is not None else 0 for h in halves]),
                     PA(*[v.data_ptr() for v in vels]), PA(*[g.data_ptr() for g in grads]),
                     (ctypes.c_int * 3)(*sizes), 3, P(lr), ctypes.c_float(0.9), ctypes.c_float(1e-4), P(seed),
                     None) == 0
    torch.cuda.synchronize()
    out = {"lr": np.float32(0.01), "momentum": np.float32(0.9), "wd": np.float32(1e-4),
           "seed_in": np.uint32(12345), "seed_out": np.uint32(seed.cpu().numpy().view(np.uint32)[0]),
           "fp16_copy": np.array(fp16_copy)}
    for i in range(3):
        out[f"p0_{i}"], out[f"v0_{i}"], out[f"g_{i}"] = p0[i], v0[i], grads[i].cpu().numpy()
        out[f"p1_{i}"], out[f"v1_{i}"] = masters[i].cpu().numpy(), vels[i].cpu().numpy()
        if halves[i] is not None:
            out[f"h1_{i}"] = halves[i].float().cpu().numpy()
    np.savez_compressed(os.path.join(outdir, "sgd.npz"), **out)
    print("golden vectors written to", outdir)


def qkv_prep_cases():
    """(file name, S, d_model, Hq, Hkv, D, QKNorm, RoPE keywords).  The scaled
    case uses a short original context and low theta so the Llama-3 frequency
    smoothing changes pairs that rotate visibly within S positions."""
    return [
        ("qkvprep_d64_qknorm_rope", 32, 128, 4, 2, 64, 1, {"theta": 10000.0}),
        ("qkvprep_d64_qknorm_rope_scaled", 48, 128, 4, 2, 64, 1,
         {"theta": 10000.0, "scale": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
          "original_context_length": 64.0}),
        ("qkvprep_d128_rope", 40, 128, 2, 1, 128, 0, {"theta": 500000.0}),
    ]


def qkv_prep_dsl(S, dm, Hq, Hkv, D, qkn, rope):
    kw = ", ".join(f"{k}={v:g}" for k, v in rope.items())
    pre = "QKNorm -> " if qkn else ""
    return f"""input: 1x{S}x{dm}
flow:
  n: RMSNorm -> {{
    q: FC({Hq * D}) -> {pre}RoPE({kw})
    k: FC({Hkv * D}) -> {pre}RoPE({kw})
    v: FC({Hkv * D})
  }} -> GQA(q={Hq}, kv={Hkv}, d={D}, causal=true)
"""


def tkm1_pack(tensors):
    parts = [np.array([0x544B4D31, len(tensors)], dtype=np.uint32).tobytes()]
    for t in tensors:
        t = np.ascontiguousarray(t, dtype=np.float32).ravel()
        parts.append(np.array([t.size], dtype=np.uint32).tobytes())
        parts.append(t.tobytes())
    return b"".join(parts)


def tkm1_unpack(blob):
    head = np.frombuffer(blob[:8], dtype=np.uint32)
    assert head[0] == 0x544B4D31
    out, off = [], 8
    for _ in range(int(head[1])):
        n = int(np.frombuffer(blob[off:off + 4], dtype=np.uint32)[0])
        off += 4
        out.append(np.frombuffer(blob[off:off + 4 * n], dtype=np.float32).copy())
        off += 4 * n
    return out


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(ROOT, "tests", "golden"))
