"""Data-parallel training step on CPU ranks (torch.distributed, gloo,
world_size 2), with the engine's NCCL all-reduce stubbed on the host.

Each rank runs the float64 graph oracle on its own micro-batch, packs the
gradients into the engine's gradient-pool layout (tensors in registration
order, 64-value slots), averages them bucket by bucket over gloo following
the engine's own bucket plan (tkm_dp_plan_buckets, the host logic of
tkm_runtime_init_dp), and applies the reference SGD update.  Every rank must
end with the same weights, equal to one process stepping on the whole batch
(the loss is a mean over rows, so the average of the ranks' gradients is the
gradient of the global batch).  Nothing here needs a GPU.
"""
import hashlib
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

WORLD = 2
CFG = dict(layers=1, d_model=128, q_heads=2, kv_heads=1, head_dim=64, ffn=256, vocab=96, seq=16, theta=10000)
B_LOCAL = 2
LR = 0.05


def _oracle(batch):
    from oracle.graph_oracle import oracle_for
    from oracle.tkm_abi import bind
    from tokamak_b200 import configs, engine
    orc = oracle_for(configs.dsl_for(CFG), batch, bind(engine()))
    rng = np.random.default_rng(5)
    orc.set_params([rng.normal(0, 0.05, n) if k == 0 else
                    (1.0 + rng.normal(0, 0.05, n) if k == 1 else rng.normal(0, 0.05, n))
                    for _, k, n in orc.tensors])
    return orc


def _batch():
    rng = np.random.default_rng(11)
    x = rng.normal(0, 1, (WORLD * B_LOCAL, CFG["seq"], CFG["d_model"]))
    y = rng.integers(0, CFG["vocab"], (WORLD * B_LOCAL, CFG["seq"])).astype(np.int32)
    return x, y


def _pool_layout(orc, grads):
    """(slot offset per tensor with a gradient, pool size): the engine's
    gradient pool, one 64-value-aligned slot per updated tensor."""
    off, pos = {}, 0
    for t, (_, _, n) in enumerate(orc.tensors):
        if t in grads:
            off[t] = pos
            pos += (n + 63) // 64 * 64
    return off, pos


def _rank_main(rank, port, outdir, target):
    import torch.distributed as dist
    from datetime import timedelta

    from tokamak_b200 import runtime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        orc = _oracle(B_LOCAL)
        x, y = _batch()
        sl = slice(rank * B_LOCAL, (rank + 1) * B_LOCAL)
        res = orc.run(x[sl].ravel(), y[sl].ravel())
        grads = res["grads"]
        off, total = _pool_layout(orc, grads)
        pool = np.zeros(total, np.float64)
        for t, o in off.items():
            pool[o:o + grads[t].size] = grads[t].ravel()
        plan = runtime.plan_buckets([n for _, _, n in orc.tensors], [nd for nd, _, _ in orc.tensors],
                                    [t in grads for t in range(len(orc.tensors))], target)
        # the stubbed all-reduce: ncclAvg over the ranks, bucket by bucket, in the engine's order
        for _, start, length in plan:
            buf = torch.from_numpy(pool[start:start + length].copy())
            dist.all_reduce(buf, op=dist.ReduceOp.SUM)
            pool[start:start + length] = buf.numpy() / WORLD
        avg = {t: pool[o:o + grads[t].size].reshape(grads[t].shape) for t, o in off.items()}
        new_p, _ = orc.sgd_update(avg, LR)
        flat = np.concatenate([p.ravel() for p in new_p]).astype(np.float32)
        np.save(os.path.join(outdir, f"rank{rank}.npy"), flat)
        np.save(os.path.join(outdir, f"plan{rank}.npy"), np.array(plan, dtype=np.int64).reshape(-1, 3))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("target", [64, 1 << 30])
def test_data_parallel_step_on_gloo_ranks(tmp_path, target):
    """target 64: one bucket per node boundary (many buckets); 2^30: a single bucket."""
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(_free_port(), str(tmp_path), target), nprocs=WORLD, join=True,
                       start_method="spawn")
    ranks = [np.load(tmp_path / f"rank{r}.npy") for r in range(WORLD)]
    digests = {hashlib.sha256(r.tobytes()).hexdigest() for r in ranks}
    assert len(digests) == 1, "ranks ended with different weights"

    # one process, whole batch
    orc = _oracle(WORLD * B_LOCAL)
    x, y = _batch()
    res = orc.run(x.ravel(), y.ravel())
    new_p, _ = orc.sgd_update(res["grads"], LR)
    ref = np.concatenate([p.ravel() for p in new_p]).astype(np.float32)
    assert np.allclose(ranks[0], ref, rtol=1e-6, atol=1e-7), np.abs(ranks[0] - ref).max()

    plan = np.load(tmp_path / "plan0.npy")
    if target == 64:
        assert len(plan) > 3
    else:
        assert len(plan) == 1


def test_bucket_plan_covers_every_slot_once():
    """tkm_dp_plan_buckets: buckets are contiguous, exchanged from the end of
    the pool to its start, cut only where a node's tensors end, and cover
    every gradient slot exactly once (tensors without a gradient own none)."""
    from tokamak_b200 import runtime
    rng = np.random.default_rng(3)
    for trial in range(50):
        nt = int(rng.integers(1, 40))
        nodes = np.sort(rng.integers(1, 20, nt))
        sizes = rng.integers(1, 5000, nt)
        has = rng.random(nt) < 0.8
        target = int(rng.integers(1, 20000))
        plan = runtime.plan_buckets(sizes, nodes, has, target, cap=8)
        total = int(sum((s + 63) // 64 * 64 for s, h in zip(sizes, has) if h))
        if total == 0:
            assert plan == []
            continue
        assert 1 <= len(plan) <= 8
        end = total
        for node, start, length in plan:  # exchange order: back to front, no gap, no overlap
            assert start + length == end and length > 0
            end = start
        assert end == 0
        # every cut but the last falls where a node's tensors begin
        slot, starts = 0, {}
        for t in range(nt):
            if has[t]:
                starts.setdefault(int(nodes[t]), slot)
                slot += (int(sizes[t]) + 63) // 64 * 64
        for node, start, _ in plan[:-1]:
            assert starts[node] == start
