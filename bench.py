"""Benchmark of the hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload attention|train|rows|longctx]

attention (default; BASELINE.json configs[1], headline shape): GQA attention
  forward + backward, bf16, causal, B=8, H=16, S=4096, D=128, through the C ABI
  of libtkm_b200.so.  One step = tkb_gqa_attn_fwd + tkb_gqa_attn_bwd.  Under
  torchrun every rank runs the same per-GPU workload (weak scaling, no
  collective on the data path).  The same JSON line carries two more records
  measured at the same N (skip them with --no-train / --no-longctx):
    "train"    the configs[3] data-parallel training step (below) with its
               NCCL gradient all-reduce timed alone (time, bus bandwidth);
    "longctx"  configs[4] at S=16384 with the KV-head groups sharded over
               the N ranks;
    "rows"     the rows workload (below) on every rank, per-GPU GB/s and
               each kernel's fraction of the HBM peak (skip with --no-rows).
train: one training step of the ~1B Llama-style decoder through
  the engine API of libtkm.so (bf16, batch 8 x 2048 tokens per GPU), the step
  captured as one CUDA graph; with N > 1 ranks the gradients are averaged by
  one NCCL all-reduce inside the graph (data parallel, weak scaling).
rows: the engine's generated plasma kernels (residual add, RMSNorm,
  SwiGLU epilogue) and the softmax cross-entropy at the configuration's shapes,
  timed per launch inside a training step; reported in HBM GB/s.
longctx: long-context GQA attention fwd+bwd, B=1, 64/8 heads,
  D=128, causal, S=16384 (or --seq 32768); KV-head groups sharded over ranks.
sweep: the attention sweep, B=8, H=16, S in {512..4096}, D in
  {64, 128}, causal and not; every point reported.

The timed region is bracketed by barriers and synchronizes, timed with CUDA
events on the launching stream, max over ranks.  Rank 0 prints one JSON line.
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


def load_rows_traffic():
    """DRAM bytes per launch of the generated row kernels (one ncu capture)."""
    p = os.path.join(ROOT, "profiles", "rows_traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("bytes_per_launch", {})
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
    ap.add_argument("--workload", default="attention", choices=["attention", "train", "rows", "longctx", "sweep", "gemm"])
    ap.add_argument("--seq", type=int, default=None, help="sequence length of the longctx / train workloads")
    ap.add_argument("--batch", type=int, default=None, help="sequences per GPU of the train workload")
    ap.add_argument("--profile", default=None, help="write the per-launch profile (train/rows) to this JSON file")
    ap.add_argument("--no-train", action="store_true", help="default line without the train object")
    ap.add_argument("--no-longctx", action="store_true", help="default line without the longctx object")
    ap.add_argument("--no-rows", action="store_true", help="default line without the rows object")
    ap.add_argument("--train-steps", type=int, default=10, help="timed steps of the train object")
    ap.add_argument("--dp-grad-dtype", default="fp32", choices=["bf16", "fp32"],
                    help="dtype the data-parallel gradients are averaged in (fp32: same-box step 95.6 vs 97.9 ms "
                         "for bf16 at 2 GPUs, whose rounding and widening passes cost more than the halved bytes save)")
    ap.add_argument("--gemm-shape", default=None, help="gemm workload: run only the shape with this name")
    ap.add_argument("--gemm", default=None, choices=["cublas", "tc"],
                    help="the engine's FC GEMMs: cuBLAS (default) or the tcgen05 kernel (sets TKM_GEMM)")
    args = ap.parse_args()
    if args.gemm:
        os.environ["TKM_GEMM"] = args.gemm
    if args.workload != "attention":
        return {"train": run_train, "rows": run_rows, "longctx": run_longctx, "sweep": run_sweep,
                "gemm": run_gemm}[args.workload](args)
    rank = int(os.environ.get("RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return 0
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            # torchrun sets OMP_NUM_THREADS=1 per rank; rank 0 runs alone here
            # and takes every host core it may use
            import oracle
            oracle.set_num_threads(len(os.sched_getaffinity(0)))
        steps, warm = ref_sample_counts(args)
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

    world, rank, local, dev = dist_setup()
    result = measure_attention(args, world, rank, local, dev)
    if not args.no_train:
        result["train"] = measure_train(args, world, rank, local, dev, configs_c4(args), args.train_steps,
                                        max(3, min(args.warmup, 5)))
    if not args.no_longctx:
        result["longctx"] = measure_longctx(args, world, rank, local, dev, args.seq or 16384, 5, 3)
    if not args.no_rows:
        result["rows"] = measure_rows(args, rank, 5, 3)[1]
    if rank == 0:
        print(json.dumps(result))
    dist_done(world)
    return 0


def ref_sample_counts(args):
    """Timed and warm-up samples of the CPU reference leg: at most 6 timed and
    3 warm-up samples of ~5 s each, in the reference arm and in the
    cpu_baseline of the default line alike."""
    return max(1, min(args.steps, 6)), min(args.warmup, 3)


def measure_attention(args, world, rank, local, dev):
    """The headline: GQA attention fwd+bwd at B=8, H=16, S=4096, D=128, causal,
    bf16, through the C ABI; every rank runs the full per-GPU workload
    (replicas, no collective).  Returns the JSON line (meaningful on rank 0)."""
    import ctypes

    import torch
    import torch.distributed as dist

    from tokamak_b200 import lib
    from tokamak_b200 import ops

    B_ = args.batch or B  # smaller batch for profiler captures; the bench line itself uses B=8
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    qkv = torch.randn(B_, S, 3 * H * D, device=dev, generator=g).to(torch.bfloat16)
    dout = torch.randn(B_, S, H * D, device=dev, generator=g).to(torch.bfloat16)
    sc = D ** -0.5
    L = lib()
    ws_bytes = L.tkb_gqa_attn_bwd_workspace_ex(B_, S, H, D, 1, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    out = torch.empty(B_, S, H * D, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B_ * H, S, dtype=torch.float32, device=dev)
    dqkv = torch.empty_like(qkv)
    stream = torch.cuda.current_stream()
    sp = stream.cuda_stream
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def fwd():
        ops.check(L.tkb_gqa_attn_fwd(P(qkv), P(out), P(lse), B_, S, H, H, D, sc, 1, 1, ctypes.c_void_p(sp)), "fwd")

    def bwd():
        ops.check(L.tkb_gqa_attn_bwd(P(qkv), P(out), P(dout), P(lse), P(dqkv), P(ws), ws_bytes, B_, S, H, H, D, sc,
                                     1, 1, ctypes.c_void_p(sp)), "bwd")

    for _ in range(args.warmup):
        fwd()
        bwd()
    dist_barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    n0 = L.tkb_launch_count()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    dist_barrier(world)
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
    dist_barrier(world)
    launches = L.tkb_launch_count() - n0
    clocks = sampler.stop()
    ms = t_start.elapsed_time(t_end)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    code = ctypes.c_uint(0)
    ops.check(L.tkb_device_error(ctypes.byref(code), ctypes.c_void_p(sp)), "device error query")
    if code.value:
        raise RuntimeError(f"device error word 0x{code.value:x} after the timed region")
    ms = dist_max(ms, world)

    # e2e: host buffers in pinned memory, copies inside the timed region
    h_qkv = torch.empty(qkv.shape, dtype=qkv.dtype, pin_memory=True)
    h_dout = torch.empty(dout.shape, dtype=dout.dtype, pin_memory=True)
    h_qkv.copy_(qkv)
    h_dout.copy_(dout)
    h_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    h_dqkv = torch.empty(dqkv.shape, dtype=dqkv.dtype, pin_memory=True)
    e2e_steps = max(2, min(args.steps, 5))
    # The batch goes through in per-sequence chunks (every (batch, head) unit
    # is independent, so the results are those of one call): chunk c's upload,
    # its fwd+bwd through the C ABI and chunk c-1's download run on three
    # streams at once, so PCIe (full duplex) and the kernels overlap.
    ws1 = L.tkb_gqa_attn_bwd_workspace_ex(1, S, H, D, 1, 1)
    up_s, down_s = torch.cuda.Stream(), torch.cuda.Stream()
    cs = ctypes.c_void_p(sp)

    def chunk_step(c):
        up = torch.cuda.Event()
        with torch.cuda.stream(up_s):
            qkv[c].copy_(h_qkv[c], non_blocking=True)
            dout[c].copy_(h_dout[c], non_blocking=True)
            up.record(up_s)
        stream.wait_event(up)
        lse_c = lse[c * H:(c + 1) * H]
        ops.check(L.tkb_gqa_attn_fwd(P(qkv[c]), P(out[c]), P(lse_c), 1, S, H, H, D, sc, 1, 1, cs), "fwd")
        ops.check(L.tkb_gqa_attn_bwd(P(qkv[c]), P(out[c]), P(dout[c]), P(lse_c), P(dqkv[c]), P(ws), ws1, 1, S, H, H,
                                     D, sc, 1, 1, cs), "bwd")
        done = torch.cuda.Event()
        done.record(stream)
        down_s.wait_event(done)
        with torch.cuda.stream(down_s):
            h_out[c].copy_(out[c], non_blocking=True)
            h_dqkv[c].copy_(dqkv[c], non_blocking=True)

    dist_barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    up_s.wait_event(e0)
    for _ in range(e2e_steps):
        for c in range(B_):
            chunk_step(c)
    tail = torch.cuda.Event()
    tail.record(down_s)
    stream.wait_event(tail)
    e1.record(stream)
    dist_barrier(world)
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    # the chunked path returns exactly the one-call results
    ref_dqkv = torch.empty_like(dqkv)
    ops.check(L.tkb_gqa_attn_fwd(P(qkv), P(out), P(lse), B_, S, H, H, D, sc, 1, 1, cs), "fwd")
    ops.check(L.tkb_gqa_attn_bwd(P(qkv), P(out), P(dout), P(lse), P(ref_dqkv), P(ws), ws_bytes, B_, S, H, H, D, sc,
                                 1, 1, cs), "bwd")
    torch.cuda.synchronize()
    e2e_identical = bool(torch.equal(ref_dqkv.cpu(), h_dqkv))
    del ref_dqkv
    e2e_ms = dist_max(e2e_ms, world)

    f_fl, b_fl = attn_flops(B_, H, S, D, CAUSAL)
    step_fl = f_fl + b_fl
    value = step_fl * world * args.steps / (ms * 1e-3) / 1e12
    e2e_value = step_fl * world / (e2e_ms * 1e-3) / 1e12
    peak, peak_sus, hbm, src = load_peaks()
    bwd_tf = b_fl / (bwd_ms * 1e-3) / 1e12
    fwd_tf = f_fl / (fwd_ms * 1e-3) / 1e12
    dom = "bwd" if bwd_ms >= fwd_ms else "fwd"
    traffic = load_traffic().get(f"attn_{dom}_bytes_per_launch")
    h2d, d2h = qkv.numel() * 2 + dout.numel() * 2, out.numel() * 2 + dqkv.numel() * 2
    del qkv, dout, out, lse, dqkv, ws, h_qkv, h_dout, h_out, h_dqkv
    torch.cuda.empty_cache()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            steps, warm = ref_sample_counts(args)
            v, cores, sample, _ = cpu_reference(steps, warm)
            cpu = {"value": v, "unit": UNIT, "cores": cores, "kind": "port",
                   "sample": f"{sample}; {warm} warm-up + {steps} timed samples, as the reference arm"}
        except Exception as e:  # the baseline never decides the run
            cpu = {"value": None, "unit": UNIT, "cores": None, "kind": "port", "sample": f"failed: {e}"}
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) Q,K,V,dO)",
        "config": {"workload": "gqa_attention_fwd_bwd", "B": B_, "H": H, "Hkv": H, "S": S, "D": D,
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
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": "pinned host -> per-sequence chunks: H2D, tkb_gqa_attn_fwd/bwd (C ABI), D2H on "
                        "three overlapped streams -> pinned host",
                "matches_one_call": e2e_identical},
        "cpu_baseline": cpu,
        "gpu_launches": int(launches),
        "clocks": clocks,
    }


# ----------------------------------------------------------------- helpers


def dist_setup():
    """(world, rank, local, device); NCCL process group for N > 1."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return world, rank, local, torch.device("cuda", local)


def dist_max(value, world):
    import torch
    import torch.distributed as dist
    if world == 1:
        return value
    t = torch.tensor([value], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.item()


def dist_barrier(world):
    import torch
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def dist_done(world):
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------- train (C4)


def train_cpu_baseline(cfg):
    """The engine step on the host: the float64 graph oracle (a restatement of
    the reference's semantics, numpy with the attention in the C oracle) on a
    bounded slice of configuration 4 -- the same layer shapes, one layer, one
    sequence of 256 tokens, vocabulary 32000."""
    import numpy as np
    from oracle.graph_oracle import oracle_for, reference_front_end
    from oracle.tkm_abi import bind
    from tokamak_b200 import configs, engine
    import oracle
    c = dict(cfg, layers=1, seq=256, batch=1)
    orc = oracle_for(configs.dsl_for(c), 1, reference_front_end() or bind(engine()))
    rng = np.random.default_rng(0)
    orc.set_params([rng.normal(0, 0.02, n) if k == 0 else (np.ones(n) if k == 1 else np.zeros(n))
                    for _, k, n in orc.tensors])
    x = rng.normal(0, 1, orc.rows(0) * orc.C[0])
    y = rng.integers(0, c["vocab"], c["seq"]).astype(np.int32)
    t0 = time.perf_counter()
    orc.run(x, y)
    dt = time.perf_counter() - t0
    return c["seq"] / dt, oracle.num_threads(), \
        f"1 layer of configuration 4 (d 2048, GQA 32/8x64, FFN 5632, vocab 32000), 1 x 256 tokens, fwd+bwd, float64"


def configs_c4(args):
    from tokamak_b200 import configs
    cfg = dict(configs.C4)
    if args.workload == "train":  # the overrides serve profiling runs of the train workload only
        if args.seq:
            cfg["seq"] = args.seq
        if args.batch:
            cfg["batch"] = args.batch
    return cfg


def measure_train(args, world, rank, local, dev, cfg, steps, warmup):
    """Configuration 4: one training step of the ~1B Llama-style decoder
    through the engine API (libtkm.so), bf16, the whole step one CUDA graph;
    at N ranks data parallel with the gradients averaged by NCCL all-reduces
    inside the graph (weak scaling: 8 x 2048 tokens per GPU).  Returns the
    `train` record (meaningful on rank 0)."""
    import ctypes
    import hashlib

    import numpy as np
    import torch
    import torch.distributed as dist

    from tokamak_b200 import configs, runtime
    B_, T, d, V = cfg["batch"], cfg["seq"], cfg["d_model"], cfg["vocab"]
    grad_dtype = runtime.DTYPE_BF16 if args.dp_grad_dtype == "bf16" else runtime.DTYPE_F32
    t_ign = time.perf_counter()
    rt = runtime.Runtime.from_dsl(configs.dsl_for(cfg), B_, runtime.DTYPE_BF16)
    rt.init_weights(1234, 0.02)
    if world > 1:
        obj = [runtime.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        rt.init_dp(obj[0], rank, world, grad_dtype)
    ignite_s = time.perf_counter() - t_ign
    # synthetic tokens: rows are the embeddings of uniform token ids (a
    # seeded N(0, 0.02) table), labels the next token
    g = np.random.default_rng(100 + rank)
    table = g.normal(0.0, 0.02, (V, d)).astype(np.float32)
    tokens = g.integers(0, V, (B_, T + 1))
    x = torch.from_numpy(table[tokens[:, :-1]].reshape(-1)).pin_memory()
    y = torch.from_numpy(tokens[:, 1:].reshape(-1).astype(np.int32)).pin_memory()
    del table
    L = runtime.lib()
    lr = 1e-4

    def step_e2e():
        loss = L.tkm_runtime_step_i32(rt.h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), lr)
        if not np.isfinite(loss):
            raise RuntimeError("train step failed: " + runtime.last_error())
        return loss

    first = step_e2e()  # uploads this rank's batch, runs eagerly, captures the step graph
    stream = torch.cuda.ExternalStream(rt.stream)
    for _ in range(max(0, warmup - 1)):
        rt.step_resident(lr)
    stream.synchronize()
    dist_barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_barrier(world)
    e0.record(stream)
    for _ in range(steps):
        rt.step_resident(lr)
    e1.record(stream)
    stream.synchronize()
    dist_barrier(world)
    clocks = sampler.stop()
    ms = dist_max(e0.elapsed_time(e1), world)

    # the gradient exchange alone (all ranks together, between steps)
    allreduce = None
    if world > 1:
        dist_barrier(world)
        ar_ms, ar_bytes = rt.dp_allreduce_time(5)
        ar_ms = dist_max(ar_ms, world)
        algbw = ar_bytes / (ar_ms * 1e-3) / 1e9
        allreduce = {"ms": ar_ms, "bytes_per_rank": ar_bytes, "dtype": args.dp_grad_dtype,
                     "algbw_GBs": algbw, "busbw_GBs": algbw * 2 * (world - 1) / world,
                     "link_ref_GBs": 770.0, "collective": "ncclAllReduce(avg), ~16 buckets in reverse layer order",
                     "overlap": "issued on a second stream as the backward completes each bucket; "
                                "the SGD update waits for the last"}

    # end to end: pinned host embeddings + labels uploaded every step, loss read
    # back; as many steps as the resident loop, so that one slow host call
    # (seen up to 150 ms against 88) weighs as little as in the resident rate
    e2e_steps = max(4, steps)
    host_ms = []
    dist_barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    last = first
    for _ in range(e2e_steps):
        h0 = time.perf_counter()
        last = step_e2e()
        host_ms.append((time.perf_counter() - h0) * 1e3)
    t1.record(stream)
    stream.synchronize()
    e2e_ms = dist_max(t0.elapsed_time(t1) / e2e_steps, world)
    # what one step's upload costs when every rank uploads at once
    dbuf = torch.empty(x.numel(), dtype=torch.float32, device=dev)
    dist_barrier(world)
    u0, u1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    u0.record()
    dbuf.copy_(x, non_blocking=True)
    u1.record()
    torch.cuda.synchronize()
    up_ms = dist_max(u0.elapsed_time(u1), world)
    del dbuf
    tokens_step = B_ * T
    value = tokens_step * world * steps / (ms * 1e-3)
    e2e_value = tokens_step * world / (e2e_ms * 1e-3)
    # data parallel: every rank must hold the same weights after the steps
    digest = hashlib.sha256(rt.save_weights()).hexdigest()
    digests = [None] * world
    if world > 1:
        dist.all_gather_object(digests, digest)
    else:
        digests = [digest]
    prof = None
    if rank == 0 and args.profile and args.workload == "train":
        prof = rt.profile(iters=2)
        with open(args.profile, "w") as f:
            json.dump(prof, f)
    # model FLOPs of one step: every GEMM (forward 2, backward 4 per MAC) plus attention
    L_, q, kv, hd, F = cfg["layers"], cfg["q_heads"], cfg["kv_heads"], cfg["head_dim"], cfg["ffn"]
    gemm_macs = L_ * d * (q * hd + 2 * kv * hd + q * hd + 3 * F) + d * V
    attn = L_ * 4.0 * B_ * q * T * T * hd * 0.5 * 3.5
    step_flops = 6.0 * tokens_step * gemm_macs + attn
    peak, peak_sus, hbm, src = load_peaks()
    achieved = step_flops / (ms / steps * 1e-3) / 1e12
    rt.close()
    torch.cuda.empty_cache()
    rec = {
        "metric": "train tokens/sec (Llama-style ~1B, bf16, data parallel)", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
        "tokens_per_s_per_gpu": value / world, "higher_is_better": True, "scaling": "weak",
        "dtype": "bf16", "data": "synthetic (seeded uniform token ids, N(0,0.02) embeddings and weights)",
        "config": {"workload": "llama_1b_train_step", "layers": L_, "d_model": d, "heads": f"{q}/{kv}x{hd}",
                   "ffn": F, "vocab": V, "seq_len": T, "micro_batch": B_, "global_batch": B_ * world,
                   "parallelism": f"dp{world}", "graph": "whole step captured as one CUDA graph",
                   "grad_allreduce_dtype": args.dp_grad_dtype if world > 1 else None,
                   "gemm": "tcgen05 kernel" if os.environ.get("TKM_GEMM") == "tc" else "cuBLAS",
                   "l2": "working set far above L2 (activations ~40 GB)"},
        "ignite_s": ignite_s, "loss_first_step": first, "loss_last": last, "host_cpus": host_cpus(),
        "dp_weights_identical_across_ranks": len(set(digests)) == 1, "weights_sha256": digests[0][:16],
        "allreduce": allreduce,
        "roofline": {"bound": "tensor", "kernel": "whole step (GEMM + attention FLOPs)", "achieved": achieved,
                     "peak": peak_sus, "unit": "TFLOP/s", "frac": achieved / peak_sus,
                     "peak_source": f"{src} bf16 sustained (MEASURED_PEAKS.json)", "traffic": None,
                     "flops_per_step_per_gpu": step_flops},
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": x.numel() * 4 + y.numel() * 4,
                "d2h_bytes_per_step": 4, "path": "pinned host -> tkm_runtime_step_i32 (engine C API) -> loss",
                "host_ms_per_call": host_ms, "upload_ms_all_ranks_at_once": up_ms},
        "clocks": clocks,
    }
    if prof:
        by_kind = {}
        for e in prof:
            by_kind[e["kind"]] = by_kind.get(e["kind"], 0.0) + e["ms"]
        rec["profile_ms_by_kind"] = by_kind
        rec["gpu_launches"] = len(prof)
    return rec


def host_cpus():
    """CPUs this process may use and the container's CPU quota (cgroup v2
    cpu.max), recorded beside the end-to-end numbers they can limit."""
    out = {"os_cpus": os.cpu_count()}
    try:
        out["affinity"] = len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        pass
    try:
        with open("/sys/fs/cgroup/cpu.max") as f:
            out["cgroup_cpu_max"] = f.read().strip()
    except OSError:
        pass
    return out


def run_train(args):
    world, rank, local, dev = dist_setup()
    cfg = configs_c4(args)
    line = measure_train(args, world, rank, local, dev, cfg, args.steps, args.warmup)
    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            try:
                v, cores, sample = train_cpu_baseline(cfg)
                cpu = {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample}
            except Exception as e:
                cpu = {"value": None, "unit": "tokens/s", "cores": None, "kind": "port", "sample": f"failed: {e}"}
        line["vs_baseline"] = None
        line["cpu_baseline"] = cpu
        line.setdefault("gpu_launches", None)
        print(json.dumps(line))
    dist_done(world)
    return 0


# ------------------------------------------------------------- rows (C3)


def rows_cpu_baseline():
    """The row kernels on the host: the C oracle (a restatement of the
    reference's semantics, fp32 in, fp64 accumulation, OpenMP) on a bounded
    sample of the same shapes -- 2048 rows of Add+RMSNorm [x4096] and SwiGLU
    [x11008], 1024 rows of softmax CE [x32000] -- as algorithmic bf16 bytes
    (the byte counts the GPU line uses) over the summed time."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(0)
    n = 2048
    x = rng.standard_normal((n, 4096)).astype(np.float32)
    r = rng.standard_normal((n, 4096)).astype(np.float32)
    g = np.ones(4096, np.float32)
    gu = rng.standard_normal((n, 2 * 11008)).astype(np.float32)
    lg = (2.0 * rng.standard_normal((n // 2, 32000))).astype(np.float32)
    lab = rng.integers(0, 32000, n // 2).astype(np.int32)
    work = [(lambda: oracle.add_rmsnorm_fwd(x, r, g), 4 * n * 4096 * 2),
            (lambda: oracle.swiglu_fwd(gu), 3 * n * 11008 * 2),
            (lambda: oracle.softmax_loss(lg, lab), 2 * (n // 2) * 32000 * 2)]
    tot_b, tot_t = 0, 0.0
    for fn, nb in work:
        fn()
        t0 = time.perf_counter()
        fn()
        tot_t += time.perf_counter() - t0
        tot_b += nb
    return tot_b / tot_t / 1e9, oracle.num_threads(), \
        "2048 x 4096 Add+RMSNorm fwd, 2048 x 11008 SwiGLU fwd, 1024 x 32000 softmax CE fwd+bwd"


def measure_rows(args, rank, steps, warmup):
    """Generated plasma kernels at configuration 2's shapes, timed per launch
    by the engine's profiler inside a bf16 training step of the graph
    [16384 x 4096] -> FC -> Bias+Add(residual) -> RMSNorm -> twin FC(11008)
    -> Bias+SiLU * Bias -> FC, and the softmax cross-entropy over
    [8192 x 32000] logits.  Returns (per-kernel rows, the `rows` record)."""
    from tokamak_b200 import runtime
    nrows = (args.seq if args.workload == "rows" else None) or 16384
    chain = f"""input: 1x{nrows}x4096
flow:
  r: {{
    branch: FC(4096)
    skip: Identity
  }} -> Add
  f: RMSNorm -> {{
    gate: FC(11008) -> SiLU
    up: FC(11008)
  }} -> Mul -> FC(10) -> SoftmaxCE
"""
    ce = f"""input: 1x{nrows // 2}x512
flow:
  h: FC(32000) -> SoftmaxCE
"""
    import numpy as np
    out = []
    for dsl in (chain, ce):
        rt = runtime.Runtime.from_dsl(dsl, 1, runtime.DTYPE_BF16)
        rt.init_weights(7, 0.02)
        x = np.random.default_rng(1).normal(0, 1, rt.input_elements).astype(np.float32)
        for _ in range(warmup):
            rt.step(x, None, 0.0)
        prof = rt.profile(iters=steps)
        out += [e for e in prof if e["kind"] in ("plasma", "softmax/loss")]
        rt.close()
    peak, peak_sus, hbm, src = load_peaks()
    rows = []
    for e in out:
        gbs = e["bytes"] / (e["ms"] * 1e-3) / 1e9
        rows.append({"name": e["name"], "ms": e["ms"], "bytes": e["bytes"], "GB/s": gbs, "frac": gbs / hbm})
    tot_b = sum(r["bytes"] for r in rows)
    tot_ms = sum(r["ms"] for r in rows)
    agg = tot_b / (tot_ms * 1e-3) / 1e9
    dom = max(rows, key=lambda r: r["ms"])
    rec = {"metric": "fused row kernels achieved HBM GB/s (bf16, per GPU)", "value": agg, "unit": "GB/s",
           "ms_per_step": tot_ms, "steps": steps, "warmup": warmup,
           "config": {"workload": "plasma_rows", "shapes": "16384x4096 add+RMSNorm, 16384x11008 SwiGLU, 8192x32000 CE",
                      "l2": "every tensor larger than L2"},
           "kernels": [{k: (round(v, 5) if isinstance(v, float) else v) for k, v in r.items()} for r in rows],
           "roofline": {"bound": "hbm", "kernel": dom["name"], "achieved": dom["GB/s"], "peak": hbm, "unit": "GB/s",
                        "frac": dom["GB/s"] / hbm, "peak_source": f"{src} HBM copy (MEASURED_PEAKS.json)",
                        "traffic": load_rows_traffic().get(dom["name"])}}
    return rows, rec


def run_rows(args):
    """The rows workload alone (see measure_rows); with --profile the
    per-kernel rows are also written to that file."""
    world, rank, local, dev = dist_setup()
    rows, rec = measure_rows(args, rank, max(3, args.steps), max(3, args.warmup))
    agg, tot_ms, dom_rf = rec["value"], rec["ms_per_step"], rec["roofline"]
    if args.profile and rank == 0:
        with open(args.profile, "w") as f:
            json.dump(rows, f, indent=1)
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        v, cores, sample = rows_cpu_baseline()
        cpu = {"value": v, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps({
            "metric": "fused row kernels achieved HBM GB/s (bf16)", "value": agg * world, "unit": "GB/s",
            "n_gpus": world, "steps": max(3, args.steps), "warmup": max(3, args.warmup), "ms_per_step": tot_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": rec["config"], "kernels": rows, "roofline": dom_rf,
            "e2e": None, "cpu_baseline": cpu, "gpu_launches": len(rows)}))
    dist_done(world)
    return 0


# ---------------------------------------------------------- longctx (C5)


def measure_longctx(args, world, rank, local, dev, S_, steps, warmup):
    """Configuration 5: long-context GQA attention fwd+bwd, B=1, 64/8 heads,
    D=128, causal, bf16; the 8 KV-head groups (each with its 8 query heads)
    sharded over the ranks with no collective (strong scaling: the total work
    is fixed).  Returns the `longctx` record (meaningful on rank 0)."""
    import ctypes

    import torch

    from tokamak_b200 import lib, ops
    Hq_all, Hkv_all, D_ = 64, 8, 128
    if Hkv_all % world:
        raise SystemExit("KV-head groups (8) must divide over the ranks")
    Hkv = Hkv_all // world
    Hq = Hq_all // world
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    qkv = torch.randn(1, S_, (Hq + 2 * Hkv) * D_, device=dev, generator=g).to(torch.bfloat16)
    dout = torch.randn(1, S_, Hq * D_, device=dev, generator=g).to(torch.bfloat16)
    out = torch.empty(1, S_, Hq * D_, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(Hq, S_, dtype=torch.float32, device=dev)
    dqkv = torch.empty_like(qkv)
    L = lib()
    ws_bytes = L.tkb_gqa_attn_bwd_workspace_ex(1, S_, Hq, D_, 1, 1)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    sc = D_ ** -0.5
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731

    def step():
        ops.check(L.tkb_gqa_attn_fwd(P(qkv), P(out), P(lse), 1, S_, Hq, Hkv, D_, sc, 1, 1, sp), "fwd")
        ops.check(L.tkb_gqa_attn_bwd(P(qkv), P(out), P(dout), P(lse), P(dqkv), P(ws), ws_bytes, 1, S_, Hq, Hkv, D_,
                                     sc, 1, 1, sp), "bwd")

    for _ in range(warmup):
        step()
    dist_barrier(world)
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    n0 = L.tkb_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_barrier(world)
    e0.record()
    for _ in range(steps):
        step()
    e1.record()
    dist_barrier(world)
    clocks = sampler.stop()
    launches = int(L.tkb_launch_count() - n0)
    ms = dist_max(e0.elapsed_time(e1), world)
    f, b = attn_flops(1, Hq, S_, D_, True)
    value = (f + b) * world * steps / (ms * 1e-3) / 1e12
    peak, peak_sus, hbm, src = load_peaks()
    del qkv, dout, out, lse, dqkv, ws
    torch.cuda.empty_cache()
    return {
        "metric": "long-context GQA attn fwd+bwd TFLOP/s (bf16, causal)", "value": value, "unit": "TFLOP/s",
        "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms / steps,
        "higher_is_better": True, "scaling": "strong", "dtype": "bf16", "data": "synthetic (seeded N(0,1))",
        "config": {"workload": "gqa_attention_long_context", "B": 1, "Hq": Hq_all, "Hkv": Hkv_all, "S": S_, "D": D_,
                   "causal": True, "per_gpu": f"{Hq} query / {Hkv} KV heads",
                   "parallelism": f"KV-head groups sharded x{world} (no collective)",
                   "dS_workspace": ws_bytes > L.tkb_gqa_attn_bwd_workspace(1, S_, Hq, D_, 1)},
        "per_gpu_tflops": value / world,
        "roofline": {"bound": "tensor", "achieved": value / world, "peak": peak, "unit": "TFLOP/s",
                     "frac": value / world / peak, "peak_source": f"{src} bf16 burst (MEASURED_PEAKS.json)",
                     "traffic": None},
        "gpu_launches": launches, "clocks": clocks}


def run_longctx(args):
    world, rank, local, dev = dist_setup()
    line = measure_longctx(args, world, rank, local, dev, args.seq or 16384, args.steps, args.warmup)
    if rank == 0:
        line.update({"vs_baseline": None, "e2e": None, "cpu_baseline": None})
        print(json.dumps(line))
    dist_done(world)
    return 0


# ------------------------------------------------------------ gemm (C4 GEMMs)


GEMM_SHAPES = [
    # (name, M, N, K, a_trans, b_trans, C fp32): one layer of configuration 4 and the LM head, 16384 tokens
    ("qkv fwd", 16384, 3072, 2048, False, False, False),
    ("qkv dX", 16384, 2048, 3072, False, True, False),
    ("qkv dW", 2048, 3072, 16384, True, False, True),
    ("o-proj fwd", 16384, 2048, 2048, False, False, False),
    ("gate|up fwd", 16384, 11264, 2048, False, False, False),
    ("gate|up dX", 16384, 2048, 11264, False, True, False),
    ("gate|up dW", 2048, 11264, 16384, True, False, True),
    ("down fwd", 16384, 2048, 5632, False, False, False),
    ("down dX", 16384, 5632, 2048, False, True, False),
    ("down dW", 5632, 2048, 16384, True, False, True),
    ("lm-head fwd", 16384, 32000, 2048, False, False, False),
]


def run_gemm(args):
    """The GEMMs of one configuration-4 layer and the LM head (16384 tokens)
    on the tcgen05 kernel (tkb_gemm, and tkb_gemm_swiglu for the twin FC)
    and on cuBLAS (torch.matmul, bf16) in the same process: TFLOP/s of each,
    every launch timed alone with CUDA events after a 256 MB L2 flush."""
    import torch

    from tokamak_b200 import lib, ops
    world, rank, local, dev = dist_setup()
    torch.backends.cuda.matmul.allow_tf32 = False
    L = lib()
    peak, peak_sus, hbm, src = load_peaks()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    reps = max(5, args.steps)

    def timed(fn):
        for _ in range(max(3, args.warmup)):
            fn()
        ts = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1))
        return statistics.median(ts)

    n0 = L.tkb_launch_count()
    rows = []
    g = torch.Generator(device=dev).manual_seed(3)
    for name, M, N, K, at, bt, f32 in GEMM_SHAPES:
        if args.gemm_shape and name != args.gemm_shape:
            continue
        A = (0.05 * torch.randn(*((K, M) if at else (M, K)), device=dev, generator=g)).bfloat16()
        Bm = (0.05 * torch.randn(*((N, K) if bt else (K, N)), device=dev, generator=g)).bfloat16()
        C = torch.empty(M, N, dtype=torch.float32 if f32 else torch.bfloat16, device=dev)
        a_op = A.T if at else A
        b_op = Bm.T if bt else Bm
        ours = timed(lambda: ops.gemm(A, Bm, at, bt, out=C))
        cublas = timed(lambda: torch.matmul(a_op, b_op))
        fl = 2.0 * M * N * K
        rows.append({"name": name, "M": M, "N": N, "K": K, "ms": ours, "tflops": fl / (ours * 1e-3) / 1e12,
                     "cublas_ms": cublas, "cublas_tflops": fl / (cublas * 1e-3) / 1e12})
        del A, Bm, C
    if args.gemm_shape:
        if rank == 0:
            print(json.dumps({"metric": "bf16 GEMM TFLOP/s (one shape)", "kernels": rows,
                              "gpu_launches": int(L.tkb_launch_count() - n0)}))
        dist_done(world)
        return 0
    # the twin FC with its SwiGLU epilogue against cuBLAS GEMM + torch SwiGLU
    F = 5632
    A = (0.05 * torch.randn(16384, 2048, device=dev, generator=g)).bfloat16()
    W = (0.05 * torch.randn(2048, 2 * F, device=dev, generator=g)).bfloat16()
    ours = timed(lambda: ops.gemm_swiglu(A, W, F))

    def cublas_swiglu():
        gu = torch.matmul(A, W)
        return torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]
    ref = timed(cublas_swiglu)
    fl = 2.0 * 16384 * 2 * F * 2048
    rows.append({"name": "gate|up fwd + SwiGLU epilogue", "M": 16384, "N": 2 * F, "K": 2048, "ms": ours,
                 "tflops": fl / (ours * 1e-3) / 1e12, "cublas_ms": ref, "cublas_tflops": fl / (ref * 1e-3) / 1e12,
                 "cublas_path": "torch.matmul + torch SiLU*up"})
    # the LM head with its softmax CE (configuration 4: 16384 rows, d 2048, vocab 32000): fused
    # (tkb_lmhead_ce: statistics pass + gradient pass, no logits buffer) against cuBLAS GEMM
    # + bias + tkb_softmax_loss (the unfused path's kernels)
    Rh, dh, Vh = 16384, 2048, 32000
    X = (0.5 * torch.randn(Rh, dh, device=dev, generator=g)).bfloat16()
    Wh = (0.02 * torch.randn(dh, Vh, device=dev, generator=g)).bfloat16()
    bh = torch.zeros(Vh, device=dev)
    yh = torch.randint(0, Vh, (Rh,), device=dev, generator=g, dtype=torch.int32)
    fused = timed(lambda: ops.lmhead_ce(X, Wh, yh, bh))

    def unfused():
        logits = torch.matmul(X, Wh) + bh.bfloat16()
        return ops.softmax_loss(logits, yh, 0, 2.0)
    ref_ce = timed(unfused)
    fl = 2.0 * Rh * dh * Vh
    ce_row = {"name": "lm-head + softmax CE (fused, two GEMM passes, no logits buffer)", "M": Rh, "N": Vh, "K": dh,
              "ms": fused, "unfused_ms": ref_ce,
              "unfused_path": "cuBLAS GEMM + bias + tkb_softmax_loss (logits [16384 x 32000] bf16 written and read)",
              "logits_buffer_bytes_saved": Rh * Vh * 2}
    del X, Wh, bh, yh
    launches = int(L.tkb_launch_count() - n0)
    tot_fl = sum(2.0 * r["M"] * r["N"] * r["K"] for r in rows[:-1])
    tot_ms = sum(r["ms"] for r in rows[:-1])
    tot_cb = sum(r["cublas_ms"] for r in rows[:-1])
    value = tot_fl / (tot_ms * 1e-3) / 1e12
    dom = max(rows[:-1], key=lambda r: r["ms"])
    rows.append(ce_row)
    if rank == 0:
        print(json.dumps({
            "metric": "bf16 GEMM TFLOP/s (configuration-4 layer GEMMs + LM head)", "value": value,
            "unit": "TFLOP/s", "n_gpus": world, "steps": reps, "warmup": max(3, args.warmup),
            "ms_per_step": tot_ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic N(0, 0.05)", "config": {"workload": "gemm_c4", "l2": "256 MB flush before every launch"},
            "cublas_tflops_same_shapes": tot_fl / (tot_cb * 1e-3) / 1e12, "kernels": rows,
            "gemm_tflops_vs_cublas": value / (tot_fl / (tot_cb * 1e-3) / 1e12),
            "roofline": {"bound": "tensor", "kernel": dom["name"], "achieved": dom["tflops"], "peak": peak,
                         "unit": "TFLOP/s", "frac": dom["tflops"] / peak,
                         "peak_source": f"{src} bf16 burst (MEASURED_PEAKS.json)", "traffic": None},
            "e2e": None, "cpu_baseline": None, "gpu_launches": launches}))
    dist_done(world)
    return 0


# ---------------------------------------------------------- sweep (C2)


def run_sweep(args):
    """The attention sweep of configuration 2: B=8, H=16, S in {512, 1024,
    2048, 4096}, D in {64, 128}, causal and not, bf16, fwd+bwd through the C
    ABI (tkb_gqa_attn_fwd + tkb_gqa_attn_bwd with the dS workspace), each point
    timed with CUDA events over --steps steps after --warmup.  One JSON line:
    the headline point is `value`, every point is listed under "points" with
    its TFLOP/s and fraction of the bf16 burst peak."""
    import ctypes

    import torch

    from tokamak_b200 import lib, ops
    world, rank, local, dev = dist_setup()
    L = lib()
    sp = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    peak, peak_sus, hbm, src = load_peaks()
    Bs, Hs = 8, 16
    points = []
    n0 = L.tkb_launch_count()
    sampler = ClockSampler(local)
    sampler.start()
    for D_ in (64, 128):
        for S_ in (512, 1024, 2048, 4096):
            for causal in (1, 0):
                g = torch.Generator(device=dev).manual_seed(5 + rank)
                qkv = torch.randn(Bs, S_, 3 * Hs * D_, device=dev, generator=g).to(torch.bfloat16)
                dout = torch.randn(Bs, S_, Hs * D_, device=dev, generator=g).to(torch.bfloat16)
                out = torch.empty(Bs, S_, Hs * D_, dtype=torch.bfloat16, device=dev)
                lse = torch.empty(Bs * Hs, S_, dtype=torch.float32, device=dev)
                dqkv = torch.empty_like(qkv)
                ws_bytes = L.tkb_gqa_attn_bwd_workspace_ex(Bs, S_, Hs, D_, causal, 1)
                ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
                sc = D_ ** -0.5

                def fwd():
                    ops.check(L.tkb_gqa_attn_fwd(P(qkv), P(out), P(lse), Bs, S_, Hs, Hs, D_, sc, causal, 1, sp), "fwd")

                def bwd():
                    ops.check(L.tkb_gqa_attn_bwd(P(qkv), P(out), P(dout), P(lse), P(dqkv), P(ws), ws_bytes, Bs, S_,
                                                 Hs, Hs, D_, sc, causal, 1, sp), "bwd")
                for _ in range(args.warmup):
                    fwd()
                    bwd()
                ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
                dist_barrier(world)
                ev[0].record()
                for _ in range(args.steps):
                    fwd()
                ev[1].record()
                for _ in range(args.steps):
                    bwd()
                ev[2].record()
                dist_barrier(world)
                tf = dist_max(ev[0].elapsed_time(ev[1]), world) / args.steps
                tb = dist_max(ev[1].elapsed_time(ev[2]), world) / args.steps
                f, b = attn_flops(Bs, Hs, S_, D_, bool(causal))
                tot = (f + b) / ((tf + tb) * 1e-3) / 1e12
                points.append({"S": S_, "D": D_, "causal": bool(causal), "fwd_ms": tf, "bwd_ms": tb,
                               "fwd_tflops": f / (tf * 1e-3) / 1e12, "bwd_tflops": b / (tb * 1e-3) / 1e12,
                               "tflops": tot, "frac": tot / peak})
                del qkv, dout, out, lse, dqkv, ws
    clocks = sampler.stop()
    head = next(p_ for p_ in points if p_["S"] == 4096 and p_["D"] == 128 and p_["causal"])
    if rank == 0:
        print(json.dumps({
            "metric": "attn fwd+bwd TFLOP/s sweep (bf16, B=8, H=16)", "value": head["tflops"] * world,
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": head["fwd_ms"] + head["bwd_ms"], "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) Q,K,V,dO)",
            "config": {"workload": "gqa_attention_sweep", "B": Bs, "H": Hs, "S": [512, 1024, 2048, 4096],
                       "D": [64, 128], "causal": [True, False], "value_point": "S=4096, D=128, causal",
                       "parallelism": f"replicas x{world} (no collective)"},
            "points": points,
            "roofline": {"bound": "tensor", "achieved": head["tflops"], "peak": peak, "unit": "TFLOP/s",
                         "frac": head["frac"], "peak_source": f"{src} bf16 burst (MEASURED_PEAKS.json)",
                         "traffic": None},
            "e2e": None, "cpu_baseline": None, "gpu_launches": int(L.tkb_launch_count() - n0), "clocks": clocks}))
    dist_done(world)
    return 0


if __name__ == "__main__":
    sys.exit(main())
