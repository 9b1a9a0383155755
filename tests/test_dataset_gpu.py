"""Device-resident dataset epochs (tkm_dataset_create / _i32 / _tokens +
tkm_runtime_train_epoch): the epoch graph that gathers each batch on the
device, sets the learning rate from the warm-up + cosine table and runs the
captured step must train exactly like the host-gathered path (same kernels,
same inputs, same order): bit-identical weights and the same average loss.
The reference builds the same feature at src/tkm_gpu.cu:1803-1967."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _rt(dsl, batch, seed=3):
    from tokamak_b200 import runtime
    rt = runtime.Runtime.from_dsl(dsl, batch, runtime.DTYPE_BF16)
    rt.init_weights(seed, 0.05)
    return rt


def _pair(dsl, batch, monkeypatch):
    """(resident runtime, host-gathered runtime) with the same weights."""
    a = _rt(dsl, batch)
    b = _rt(dsl, batch)
    b.load_weights(a.save_weights())
    return a, b


def _epochs(rt_res, rt_host, make, monkeypatch, order, epochs=2):
    from tokamak_b200 import runtime
    monkeypatch.delenv("TKM_DATASET_RESIDENT", raising=False)
    ds_a = make(rt_res)
    monkeypatch.setenv("TKM_DATASET_RESIDENT", "0")
    ds_b = make(rt_host)
    monkeypatch.delenv("TKM_DATASET_RESIDENT", raising=False)
    assert ds_a.resident and not ds_b.resident
    step = 0
    for e in range(epochs):
        o = None if order is None else order(e)
        la = ds_a.train_epoch(o, peak_lr=0.05, min_lr_ratio=0.1, step0=step, total_steps=20, warmup=2)
        lb = ds_b.train_epoch(o, peak_lr=0.05, min_lr_ratio=0.1, step0=step, total_steps=20, warmup=2)
        assert np.isfinite(la)
        assert abs(la - lb) <= 1e-6 * abs(lb), (e, la, lb)
        step += 1
    wa, wb = runtime.tkm1_unpack(rt_res.save_weights()), runtime.tkm1_unpack(rt_host.save_weights())
    for t, (x, y) in enumerate(zip(wa, wb)):
        assert np.array_equal(x, y), t
    ds_a.close()
    ds_b.close()


def test_resident_epoch_uint8_labels(monkeypatch):
    """The reference's API: images + one uint8 label per sample."""
    from tokamak_b200 import runtime
    dsl = "input: 1x1x64\nflow:\n  h: FC(32) -> ReLU -> FC(10) -> SoftmaxCE\n"
    B, n = 16, 100
    rng = np.random.default_rng(1)
    x = rng.normal(0, 1, (n, 64)).astype(np.float32)
    y = rng.integers(0, 10, n).astype(np.uint8)
    a, b = _pair(dsl, B, monkeypatch)
    _epochs(a, b, lambda rt: runtime.Dataset(rt, x, y), monkeypatch,
            lambda e: np.random.default_rng(e).permutation(n).astype(np.uint32))


def test_resident_epoch_int32_row_labels(monkeypatch):
    """A small Llama-style decoder with one int32 label per token row."""
    from tokamak_b200 import configs, runtime
    cfg = dict(configs.C1, layers=1, d_model=128, q_heads=2, kv_heads=1, head_dim=64, ffn=256, vocab=512, seq=32)
    dsl = configs.dsl_for(cfg)
    B, n = 4, 18
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, (n, cfg["seq"], cfg["d_model"])).astype(np.float32)
    y = rng.integers(0, cfg["vocab"], (n, cfg["seq"])).astype(np.int32)
    a, b = _pair(dsl, B, monkeypatch)
    _epochs(a, b, lambda rt: runtime.Dataset(rt, x, y), monkeypatch, None)


def test_resident_token_sequences_match_gathered_rows(monkeypatch):
    """Token sequences over an embedding table, gathered on the device, train
    exactly like the same rows and next-token labels gathered on the host."""
    from tokamak_b200 import configs, runtime
    cfg = dict(configs.C1, layers=1, d_model=128, q_heads=2, kv_heads=1, head_dim=64, ffn=256, vocab=512, seq=32)
    dsl = configs.dsl_for(cfg)
    B, n, V = 4, 12, cfg["vocab"]
    rng = np.random.default_rng(4)
    table = rng.normal(0, 0.5, (V, cfg["d_model"])).astype(np.float32)
    tokens = rng.integers(0, V, (n, cfg["seq"] + 1)).astype(np.int32)
    a, b = _pair(dsl, B, monkeypatch)
    _epochs(a, b, lambda rt: runtime.Dataset(rt, None, tokens=tokens, embed=table), monkeypatch,
            lambda e: np.random.default_rng(10 + e).permutation(n).astype(np.uint32))
    # the same sequences as explicit rows and labels on a third runtime
    c = _rt(dsl, B)
    d = _rt(dsl, B)
    d.load_weights(c.save_weights())
    rows = table[tokens[:, :-1]]
    labels = tokens[:, 1:].copy()
    ds_c = runtime.Dataset(c, None, tokens=tokens, embed=table)
    ds_d = runtime.Dataset(d, rows, labels)
    assert ds_c.resident and ds_d.resident
    lc = ds_c.train_epoch(None, 0.05, 0.1, 0, 10, 0)
    ld = ds_d.train_epoch(None, 0.05, 0.1, 0, 10, 0)
    assert lc == ld
    for x, y in zip(runtime.tkm1_unpack(c.save_weights()), runtime.tkm1_unpack(d.save_weights())):
        assert np.array_equal(x, y)


def test_dataset_rejects_bad_labels_tokens_and_order():
    from tokamak_b200 import TkbError, configs, runtime
    dsl = "input: 1x1x64\nflow:\n  h: FC(10) -> SoftmaxCE\n"
    rt = _rt(dsl, 8)
    x = np.zeros((16, 64), np.float32)
    with pytest.raises(TkbError):
        runtime.Dataset(rt, x, np.full(16, 12, np.uint8))  # label >= 10 classes
    with pytest.raises(TkbError):
        runtime.Dataset(rt, x, np.full(16, -1, np.int32))
    ds = runtime.Dataset(rt, x, np.zeros(16, np.uint8))
    with pytest.raises(TkbError):
        ds.train_epoch(np.full(16, 99, np.uint32))  # order entry outside the dataset
    cfg = dict(configs.C1, layers=1, d_model=128, q_heads=2, kv_heads=1, head_dim=64, ffn=256, vocab=512, seq=32)
    rt2 = _rt(configs.dsl_for(cfg), 2)
    with pytest.raises(TkbError):
        runtime.Dataset(rt2, None, tokens=np.full((2, 33), 600, np.int32),
                        embed=np.zeros((512, 128), np.float32))  # token outside the table
