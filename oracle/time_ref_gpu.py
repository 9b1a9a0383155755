"""Times the reference's own GPU kernels on a B200 -- TEST INFRASTRUCTURE ONLY.

The reference (BSODsystem32/Tokamak) publishes no number for its GPU hot path,
so its kernels are timed here at this repository's benchmark shapes, built
unchanged from its sources by oracle/build_ref.py (oracle/_ref/libtkm_ref.so,
launchers in oracle/ref_gpu_harness.cu with the grids of its launch sites):

  k_gqa_flash_attn_tc_fwd / _bwd   src/tkm_gpu.cu:302-598 (fp16 WMMA; its
                                   backward computes dQ only, dK/dV are copies)
  k_softmax_loss_fwd_bwd_h         src/tkm_gpu.cu:632-682 (uint8 labels)
  k_softmax_fwd_h / _bwd_h         src/tkm_gpu.cu:600-630

Each kernel is timed with CUDA events on its stream after warm-up; the rate is
the algorithmic work of the shape (the same FLOP and byte counts bench.py
uses for this repository's kernels) divided by the time.  Prints one JSON
line per kernel.  Needs a GPU:  python oracle/time_ref_gpu.py
"""
import ctypes
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _time(fn, reps, warmup=2):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps / 1e3  # seconds per call


def main():
    path = os.path.join(HERE, "_ref", "libtkm_ref.so")
    if not os.path.exists(path):
        sys.exit(f"{path} is missing: build it with oracle/build_ref.py where the reference tree is present")
    L = ctypes.CDLL(path)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    dev = "cuda"
    g = torch.Generator(device=dev).manual_seed(11)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    out = []

    # attention: the headline shape of bench.py, fp16 (the reference's only 16-bit type)
    for (B, H, S, D, causal) in ((8, 16, 4096, 128, 1), (8, 16, 1024, 64, 1)):
        qkv = torch.randn(B, S, 3 * H * D, device=dev, generator=g).half()
        dout = torch.randn(B, S, H * D, device=dev, generator=g).half()
        o = torch.empty(B, S, H * D, device=dev, dtype=torch.half)
        lse = torch.empty(B * H, S, device=dev, dtype=torch.float32)
        dqkv = torch.empty_like(qkv)
        scale = ctypes.c_float(D ** -0.5)
        fwd = lambda: L.ref_attn_fwd(P(qkv), P(o), P(lse), B, S, H, H, D, scale, causal, stream)
        bwd = lambda: L.ref_attn_bwd(P(qkv), P(o), P(dout), P(lse), P(dqkv), B, S, H, H, D, scale, causal, stream)
        assert fwd() == 0 and bwd() == 0
        flops_fwd = 4.0 * B * H * S * S * D * (0.5 if causal else 1.0)
        tf, tb = _time(fwd, 3), _time(bwd, 3)
        out.append({"kernel": "reference k_gqa_flash_attn_tc_fwd", "B": B, "H": H, "S": S, "D": D, "causal": bool(causal),
                    "ms": tf * 1e3, "tflops": flops_fwd / tf / 1e12, "dtype": "f16"})
        out.append({"kernel": "reference k_gqa_flash_attn_tc_bwd (dQ only; dK/dV not computed)", "B": B, "H": H, "S": S,
                    "D": D, "causal": bool(causal), "ms": tb * 1e3,
                    "tflops_if_complete": 2.5 * flops_fwd / tb / 1e12, "dtype": "f16",
                    "note": "rate counts the work of a complete backward (2.5x forward), which this kernel does not do"})
        out.append({"kernel": "reference attention fwd+bwd", "B": B, "H": H, "S": S, "D": D, "causal": bool(causal),
                    "ms": (tf + tb) * 1e3, "tflops": 3.5 * flops_fwd / (tf + tb) / 1e12})
        del qkv, dout, o, lse, dqkv

    # softmax cross-entropy, fused forward + backward (configuration 3 shape)
    rows, cols = 8192, 32000
    logits = (2.0 * torch.randn(rows, cols, device=dev, generator=g)).half()
    labels = torch.randint(0, 256, (rows,), device=dev, generator=g, dtype=torch.uint8)
    dlog = torch.empty_like(logits)
    loss = torch.zeros(1, device=dev)
    correct = torch.zeros(1, device=dev, dtype=torch.int32)
    ce = lambda: L.ref_softmax_loss(P(logits), P(labels), P(dlog), P(loss), P(correct), rows, cols, 0,
                                    ctypes.c_float(0.0), stream)
    assert ce() == 0
    t = _time(ce, 3)
    out.append({"kernel": "reference k_softmax_loss_fwd_bwd_h", "rows": rows, "cols": cols, "ms": t * 1e3,
                "gbs": 4.0 * rows * cols / t / 1e9, "dtype": "f16",
                "bytes": "read logits + write d logits, 2 bytes each"})
    # standalone softmax forward and backward
    p = torch.empty_like(logits)
    dx = torch.empty_like(logits)
    sf = lambda: L.ref_softmax_fwd(P(logits), P(p), rows, cols, stream)
    sb = lambda: L.ref_softmax_bwd(P(p), P(logits), P(dx), rows, cols, stream)
    assert sf() == 0 and sb() == 0
    t = _time(sf, 3)
    out.append({"kernel": "reference k_softmax_fwd_h", "rows": rows, "cols": cols, "ms": t * 1e3,
                "gbs": 4.0 * rows * cols / t / 1e9, "dtype": "f16"})
    t = _time(sb, 3)
    out.append({"kernel": "reference k_softmax_bwd_h", "rows": rows, "cols": cols, "ms": t * 1e3,
                "gbs": 8.0 * rows * cols / t / 1e9, "dtype": "f16", "bytes": "read p, dp, dx; write dx"})
    for r in out:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
