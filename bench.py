"""Benchmark of the hot path: GQA attention forward + backward, bf16, causal,
B=8, H=16, S=4096, D=128 (headline shape) through the
C ABI of libtkm_b200.so.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = tkb_gqa_attn_fwd + tkb_gqa_attn_bwd over one batch.  Under torchrun
each rank runs the same per-GPU workload on its own GPU (weak scaling: the
(batch, head) units are independent, no collective on the data path); the
timed region is bracketed by barriers and synchronizes, and the elapsed time
is the max over ranks.  Rank 0 prints one JSON line.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, H, S, D = 8, 16, 4096, 128
CAUSAL = True
METRIC = "attn fwd+bwd TFLOP/s (bf16,S=4096,D=128,causal)"
UNIT = "TFLOP/s"


def attn_flops(b, h, s, d, causal=True):
    """Algorithmic FLOPs: fwd = 4*b*h*s^2*d (x1/2 causal); bwd = 2.5 x fwd."""
    fwd = 4.0 * b * h * s * s * d * (0.5 if causal else 1.0)
    return fwd, 2.5 * fwd


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            j = json.load(f)
        return j.get("bf16_tflops", 1590.0), j.get("bf16_tflops_sustained", 1400.0), j.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


def load_traffic():
    p = os.path.join(ROOT, "profiles", "attn_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


def cpu_reference(steps, warmup, sample_heads=None):
    """The reference path has no CPU implementation; time the C oracle (a
    restatement of its semantics, fp64 accumulation, OpenMP) on a bounded
    sample of the same workload: B=1, `sample_heads` heads, S=4096, D=128."""
    import numpy as np

    import oracle
    nt = oracle.num_threads()
    h = sample_heads or max(1, min(nt, 16))
    rng = np.random.default_rng(0)
    qkv = rng.standard_normal((1, S, 3 * h * D)).astype(np.float32)
    dout = rng.standard_normal((1, S, h * D)).astype(np.float32)
    sc = D ** -0.5
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        o, lse = oracle.attn_fwd(qkv, 1, S, h, h, D, sc, CAUSAL)
        oracle.attn_bwd(qkv, o, dout, lse, 1, S, h, h, D, sc, CAUSAL)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    f, b = attn_flops(1, h, S, D)
    return (f + b) / statistics.mean(times) / 1e12, nt, f"B=1, H={h} of 16 heads, S={S}, D={D}, causal, fwd+bwd", \
        statistics.mean(times)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        steps = max(1, min(args.steps, 6))
        warm = min(args.warmup, 1)
        v, cores, sample, t = cpu_reference(steps, warm)
        line = {"metric": METRIC, "value": v, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
                "steps": steps, "warmup": warm, "ms_per_step": t * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32 in, f64 accumulate", "data": "synthetic",
                "config": {"workload": "gqa_attention_fwd_bwd", "B": B, "H": H, "S": S, "D": D, "causal": CAUSAL,
                           "sample": sample},
                "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
                "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return 0

    import torch
    import torch.distributed as dist

    from tokamak_b200 import lib
    from tokamak_b200 import ops

    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    qkv = torch.randn(B, S, 3 * H * D, device=dev, generator=g).to(torch.bfloat16)
    dout = torch.randn(B, S, H * D, device=dev, generator=g).to(torch.bfloat16)
    sc = D ** -0.5
    L = lib()
    ws_bytes = L.tkb_gqa_attn_bwd_workspace(B, S, H, D, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty(B, S, H * D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B * H, S, dtype=torch.float32, device=dev)
    dqkv = torch.empty_like(qkv)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    import ctypes
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def fwd():
        ops.check(L.tkb_gqa_attn_fwd(P(qkv), P(out), P(lse), B, S, H, H, D, sc, 1, 1, ctypes.c_void_p(sp)), "fwd")

    def bwd():
        ops.check(L.tkb_gqa_attn_bwd(P(qkv), P(out), P(dout), P(lse), P(dqkv), P(ws), ws_bytes, B, S, H, H, D, sc,
                                     1, 1, ctypes.c_void_p(sp)), "bwd")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        fwd()
        bwd()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    n0 = L.tkb_launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        fwd()
        ev[i][1].record(stream)
        bwd()
        ev[i][2].record(stream)
    t_end.record(stream)
    barrier()
    launches = L.tkb_launch_count() - n0
    clocks = sampler.stop()
    ms = t_start.elapsed_time(t_end)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    code = ctypes.c_uint(0)
    ops.check(L.tkb_device_error(ctypes.byref(code), ctypes.c_void_p(sp)), "device error query")
    if code.value:
        raise RuntimeError(f"device error word 0x{code.value:x} after the timed region")
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()

    # e2e: host buffers in pinned memory, copies inside the timed region
    h_qkv = torch.empty(qkv.shape, dtype=qkv.dtype, pin_memory=True)
    h_dout = torch.empty(dout.shape, dtype=dout.dtype, pin_memory=True)
    h_qkv.copy_(qkv)
    h_dout.copy_(dout)
    h_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    h_dqkv = torch.empty(dqkv.shape, dtype=dqkv.dtype, pin_memory=True)
    e2e_steps = max(2, min(args.steps, 5))
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        qkv.copy_(h_qkv, non_blocking=True)
        dout.copy_(h_dout, non_blocking=True)
        fwd()
        bwd()
        h_out.copy_(out, non_blocking=True)
        h_dqkv.copy_(dqkv, non_blocking=True)
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()

    f_fl, b_fl = attn_flops(B, H, S, D, CAUSAL)
    step_fl = f_fl + b_fl
    value = step_fl * world * args.steps / (ms * 1e-3) / 1e12
    e2e_value = step_fl * world / (e2e_ms * 1e-3) / 1e12
    peak, peak_sus, hbm, src = load_peaks()
    bwd_tf = b_fl / (bwd_ms * 1e-3) / 1e12
    fwd_tf = f_fl / (fwd_ms * 1e-3) / 1e12
    dom = "bwd" if bwd_ms >= fwd_ms else "fwd"
    traffic = load_traffic().get(f"attn_{dom}_bytes_per_launch")
    result = None
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline:
            try:
                v, cores, sample, _ = cpu_reference(1, 0, sample_heads=None)
                cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}
            except Exception as e:  # the baseline never decides the run
                cpu = {"value": None, "unit": UNIT, "cores": None, "kind": "port", "sample": f"failed: {e}"}
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) Q,K,V,dO)",
            "config": {"workload": "gqa_attention_fwd_bwd", "B": B, "H": H, "Hkv": H, "S": S, "D": D,
                       "causal": CAUSAL, "per_gpu": "full workload on every rank",
                       "l2": "inputs larger than L2 (qkv 403 MB, dqkv 403 MB)",
                       "parallelism": f"replicas x{world} (independent batch/head units, no collective)"},
            "fwd_ms": fwd_ms, "bwd_ms": bwd_ms, "fwd_tflops": fwd_tf, "bwd_tflops": bwd_tf,
            "roofline": {"bound": "tensor", "kernel": f"tkb_gqa_attn_{dom}", "achieved": bwd_tf if dom == "bwd" else fwd_tf,
                         "peak": peak, "unit": "TFLOP/s",
                         "frac": (bwd_tf if dom == "bwd" else fwd_tf) / peak,
                         "frac_of_sustained": (bwd_tf if dom == "bwd" else fwd_tf) / peak_sus,
                         "peak_source": f"{src} bf16 burst (MEASURED_PEAKS.json)", "traffic": traffic,
                         "flops_per_launch": b_fl if dom == "bwd" else f_fl},
            "e2e": {"value": e2e_value, "unit": UNIT,
                    "h2d_bytes_per_step": qkv.numel() * 2 + dout.numel() * 2,
                    "d2h_bytes_per_step": out.numel() * 2 + dqkv.numel() * 2,
                    "path": "pinned host -> tkb_gqa_attn_fwd/bwd (C ABI) -> pinned host"},
            "cpu_baseline": cpu,
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        print(json.dumps(result))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
