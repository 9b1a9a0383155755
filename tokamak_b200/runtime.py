"""Python binding of the Tokamak engine API (include/tkm.h, libtkm.so).

Mirrors the reference's runtime calls (tkm_load_string, tkm_runtime_step,
tkm_runtime_forward, tkm_save_weights_buffer, tkm_get_grad_sample, ...) with
numpy arrays in place of raw host pointers.  Everything runs in libtkm.so;
this module only marshals buffers and raises on failure.
"""
import ctypes
import os

import numpy as np

from . import TkbError, engine

DTYPE_F32, DTYPE_BF16 = 0, 1

_c = ctypes
_vp, _i, _f, _sz = _c.c_void_p, _c.c_int, _c.c_float, _c.c_size_t
_SIGS = {
    "tkm_last_error": ([], _c.c_char_p),
    "tkm_load_string": ([_c.c_char_p, _i], _vp),
    "tkm_load_string_ex": ([_c.c_char_p, _i, _i], _vp),
    "tkm_load_file": ([_c.c_char_p, _i], _vp),
    "tkm_load_buffer": ([_c.c_char_p, _sz, _i], _vp),
    "tkm_runtime_ignite": ([_vp, _c.c_char_p], _vp),
    "tkm_runtime_ignite_inference": ([_vp, _c.c_char_p], _vp),
    "tkm_runtime_ignite_ex": ([_vp, _c.c_char_p, _i, _i], _vp),
    "tkm_runtime_step": ([_vp, _vp, _vp, _f], _f),
    "tkm_runtime_step_i32": ([_vp, _vp, _vp, _f], _f),
    "tkm_runtime_eval": ([_vp, _vp, _vp, _i], _i),
    "tkm_runtime_forward": ([_vp, _vp, _vp, _sz], _sz),
    "tkm_runtime_input_elements": ([_vp], _sz),
    "tkm_runtime_output_elements": ([_vp], _sz),
    "tkm_runtime_weight_bytes": ([_vp], _sz),
    "tkm_runtime_input_grad": ([_vp, _vp, _sz], _sz),
    "tkm_runtime_logits": ([_vp, _vp, _sz], _sz),
    "tkm_runtime_param_grad": ([_vp, _i, _vp, _sz], _sz),
    "tkm_runtime_param_count": ([_vp], _i),
    "tkm_save_weights_buffer": ([_vp, _vp, _sz, _c.POINTER(_sz)], _i),
    "tkm_load_weights_buffer": ([_vp, _vp, _sz], _i),
    "tkm_save_weights": ([_vp, _c.c_char_p], _i),
    "tkm_load_weights": ([_vp, _c.c_char_p], _i),
    "tkm_runtime_free": ([_vp], None),
    "tkm_get_grad_sample": ([_vp, _i, _i], _f),
    "tkm_perturb_tensor": ([_vp, _i, _i, _f], None),
    "tkm_eval_current_loss": ([_vp], _f),
    "tkm_nccl_unique_id": ([_vp], _i),
    "tkm_runtime_init_dp": ([_vp, _vp, _i, _i], _i),
    "tkm_runtime_init_dp_ex": ([_vp, _vp, _i, _i, _i], _i),
    "tkm_runtime_dp_allreduce_time": ([_vp, _i, _c.POINTER(_f)], _sz),
    "tkm_dp_plan_buckets": ([_i, _c.POINTER(_sz), _c.POINTER(_i), _c.POINTER(_i), _sz, _i, _c.POINTER(_i),
                             _c.POINTER(_sz), _c.POINTER(_sz)], _i),
    "tkm_codegen_cuda_string": ([_vp], _vp),
    "tkm_runtime_profile": ([_vp, _i, _vp, _i], _i),
    "tkm_runtime_init_weights": ([_vp, _c.c_ulonglong, _f], _i),
    "tkm_runtime_stream": ([_vp], _vp),
    "tkm_runtime_optimizer_bytes": ([_vp], _sz),
    "tkm_dataset_create": ([_vp, _vp, _vp, _sz], _vp),
    "tkm_dataset_create_i32": ([_vp, _vp, _vp, _sz], _vp),
    "tkm_dataset_create_tokens": ([_vp, _vp, _i, _vp, _sz], _vp),
    "tkm_dataset_free": ([_vp], None),
    "tkm_dataset_is_resident": ([_vp], _i),
    "tkm_runtime_train_epoch": ([_vp, _vp, _vp, _f, _f, _sz, _sz, _sz, _c.POINTER(_f)], _i),
    "tkm_save_optimizer_buffer": ([_vp, _vp, _sz, _c.POINTER(_sz)], _i),
    "tkm_load_optimizer_buffer": ([_vp, _vp, _sz], _i),
}


class ProfileEntry(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 64), ("node", ctypes.c_int), ("kind", ctypes.c_int),
                ("backward", ctypes.c_int), ("bytes", ctypes.c_double), ("flops", ctypes.c_double),
                ("ms", ctypes.c_float)]


PROFILE_KINDS = {0: "plasma", 1: "gemm", 2: "attention", 3: "softmax/loss", 4: "sgd", 5: "collective"}

_BOUND = None


def lib():
    global _BOUND
    if _BOUND is None:
        L = engine()
        for name, (args, res) in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _BOUND = L
    return _BOUND


def last_error():
    return (lib().tkm_last_error() or b"").decode(errors="replace")


def _ptr(a):
    return a.ctypes.data_as(_vp) if a is not None else None


def nccl_unique_id():
    buf = (ctypes.c_char * 128)()
    if not lib().tkm_nccl_unique_id(ctypes.cast(buf, _vp)):
        raise TkbError("tkm_nccl_unique_id: " + last_error())
    return bytes(buf)


class Runtime:
    """One engine runtime (owns device state until close())."""

    def __init__(self, handle):
        if not handle:
            raise TkbError("runtime creation failed: " + last_error())
        self.h = _vp(handle)

    @classmethod
    def from_dsl(cls, text, batch, dtype=DTYPE_BF16):
        rt = cls(lib().tkm_load_string_ex(text.encode(), int(batch), int(dtype)))
        rt.batch = int(batch)
        return rt

    @classmethod
    def from_file(cls, path, batch):
        return cls(lib().tkm_load_file(os.fsencode(path), int(batch)))

    def close(self):
        if self.h:
            lib().tkm_runtime_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def input_elements(self):
        return lib().tkm_runtime_input_elements(self.h)

    @property
    def output_elements(self):
        return lib().tkm_runtime_output_elements(self.h)

    def step(self, x, labels=None, lr=0.0):
        """One training step.  uint8 labels follow the reference's convention
        (one per sample); int32 labels give one label per loss row."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        assert x.size == self.input_elements, (x.size, self.input_elements)
        if labels is not None and np.asarray(labels).dtype == np.int32:
            y = np.ascontiguousarray(labels, dtype=np.int32)
            loss = lib().tkm_runtime_step_i32(self.h, _ptr(x), _ptr(y), float(lr))
        else:
            y = None if labels is None else np.ascontiguousarray(labels, dtype=np.uint8)
            loss = lib().tkm_runtime_step(self.h, _ptr(x), _ptr(y), float(lr))
        if np.isnan(loss) and last_error():
            raise TkbError("step: " + last_error())
        return float(loss)

    def forward(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(self.output_elements, dtype=np.float32)
        n = lib().tkm_runtime_forward(self.h, _ptr(x), _ptr(out), out.size)
        if n == 0:
            raise TkbError("forward: " + last_error())
        return out

    def eval(self, x, labels_u8, count):
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.ascontiguousarray(labels_u8, dtype=np.uint8)
        return lib().tkm_runtime_eval(self.h, _ptr(x), _ptr(y), int(count))

    def logits(self, n):
        out = np.empty(n, dtype=np.float32)
        if lib().tkm_runtime_logits(self.h, _ptr(out), n) != n:
            raise TkbError("logits: " + last_error())
        return out

    def input_grad(self):
        out = np.empty(self.input_elements, dtype=np.float32)
        if lib().tkm_runtime_input_grad(self.h, _ptr(out), out.size) != out.size:
            raise TkbError("input_grad: " + last_error())
        return out

    def param_count(self):
        return lib().tkm_runtime_param_count(self.h)

    def param_grad(self, index, n):
        out = np.empty(n, dtype=np.float32)
        if lib().tkm_runtime_param_grad(self.h, int(index), _ptr(out), n) != n:
            raise TkbError(f"param_grad {index}: " + last_error())
        return out

    def save_weights(self):
        n = lib().tkm_runtime_weight_bytes(self.h)
        buf = np.empty(n, dtype=np.uint8)
        size = _sz()
        if not lib().tkm_save_weights_buffer(self.h, _ptr(buf), n, ctypes.byref(size)):
            raise TkbError("save_weights: " + last_error())
        return buf.tobytes()

    def load_weights(self, blob):
        arr = np.frombuffer(blob, dtype=np.uint8)
        if not lib().tkm_load_weights_buffer(self.h, _ptr(arr), arr.size):
            raise TkbError("load_weights: " + last_error())

    def save_optimizer(self):
        """SGD momentum state (TKMV layout, beside the TKM1 weights)."""
        n = lib().tkm_runtime_optimizer_bytes(self.h)
        buf = np.empty(max(n, 1), dtype=np.uint8)
        size = _sz()
        if not n or not lib().tkm_save_optimizer_buffer(self.h, _ptr(buf), n, ctypes.byref(size)):
            raise TkbError("save_optimizer: " + last_error())
        return buf[:n].tobytes()

    def load_optimizer(self, blob):
        arr = np.frombuffer(blob, dtype=np.uint8)
        if not lib().tkm_load_optimizer_buffer(self.h, _ptr(arr), arr.size):
            raise TkbError("load_optimizer: " + last_error())

    def grad_sample(self, node, idx):
        return float(lib().tkm_get_grad_sample(self.h, int(node), int(idx)))

    def perturb(self, node, idx, delta):
        lib().tkm_perturb_tensor(self.h, int(node), int(idx), float(delta))

    def eval_current_loss(self):
        return float(lib().tkm_eval_current_loss(self.h))

    def init_weights(self, seed, std):
        if not lib().tkm_runtime_init_weights(self.h, int(seed), float(std)):
            raise TkbError("init_weights: " + last_error())

    @property
    def stream(self):
        """cudaStream_t of the runtime (as an integer)."""
        return lib().tkm_runtime_stream(self.h) or 0

    def step_resident(self, lr):
        """One step on the inputs and labels already on the device (no upload,
        no loss read-back, no host synchronisation)."""
        lib().tkm_runtime_step(self.h, None, None, float(lr))

    def profile(self, iters=3, capacity=4096):
        """Per-launch device times of `iters` eager training steps, as dicts."""
        arr = (ProfileEntry * capacity)()
        n = lib().tkm_runtime_profile(self.h, int(iters), ctypes.cast(arr, _vp), capacity)
        if n <= 0:
            raise TkbError("profile: " + last_error())
        out = []
        for e in arr[:n]:
            out.append({"name": e.name.decode(), "node": e.node, "kind": PROFILE_KINDS.get(e.kind, "?"),
                        "backward": bool(e.backward), "bytes": e.bytes, "flops": e.flops, "ms": e.ms})
        return out

    def init_dp(self, uid, rank, world, grad_dtype=DTYPE_F32):
        """Join a data-parallel group (NCCL); grad_dtype: the dtype gradients
        are averaged in across the ranks (DTYPE_F32 or DTYPE_BF16)."""
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        if not lib().tkm_runtime_init_dp_ex(self.h, ctypes.cast(buf, _vp), int(rank), int(world), int(grad_dtype)):
            raise TkbError("init_dp: " + last_error())

    def dp_allreduce_time(self, iters=5):
        """(milliseconds of one round of every gradient bucket's all-reduce,
        bytes each rank sends into it), timed alone between steps."""
        ms = _f(0.0)
        n = lib().tkm_runtime_dp_allreduce_time(self.h, int(iters), ctypes.byref(ms))
        if not n:
            raise TkbError("dp_allreduce_time: " + last_error())
        return float(ms.value), int(n)


class Dataset:
    """A training dataset of the engine (tkm_dataset_create*).  Keeps the
    host arrays alive for its lifetime (the engine copies them)."""

    def __init__(self, rt, inputs, labels=None, tokens=None, embed=None):
        L = lib()
        self.rt = rt
        if tokens is not None:
            self._keep = (np.ascontiguousarray(embed, np.float32), np.ascontiguousarray(tokens, np.int32))
            h = L.tkm_dataset_create_tokens(rt.h, _ptr(self._keep[0]), int(self._keep[0].shape[0]),
                                            _ptr(self._keep[1]), int(self._keep[1].shape[0]))
        else:
            x = np.ascontiguousarray(inputs, np.float32)
            n = int(x.size // (rt.input_elements // self._batch(rt)))
            if np.asarray(labels).dtype == np.uint8:
                y = np.ascontiguousarray(labels, np.uint8)
                h = L.tkm_dataset_create(rt.h, _ptr(x), _ptr(y), n)
            else:
                y = np.ascontiguousarray(labels, np.int32)
                h = L.tkm_dataset_create_i32(rt.h, _ptr(x), _ptr(y), n)
            self._keep = (x, y)
        if not h:
            raise TkbError("dataset creation failed: " + last_error())
        self.h = _vp(h)

    @staticmethod
    def _batch(rt):
        return rt.batch

    @property
    def resident(self):
        return bool(lib().tkm_dataset_is_resident(self.h))

    def train_epoch(self, order=None, peak_lr=0.01, min_lr_ratio=0.1, step0=0, total_steps=100, warmup=0):
        o = None if order is None else np.ascontiguousarray(order, np.uint32)
        avg = _f(0.0)
        if not lib().tkm_runtime_train_epoch(self.rt.h, self.h, _ptr(o), float(peak_lr), float(min_lr_ratio),
                                             int(step0), int(total_steps), int(warmup), ctypes.byref(avg)):
            raise TkbError("train_epoch: " + last_error())
        return float(avg.value)

    def close(self):
        if self.h:
            lib().tkm_dataset_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def plan_buckets(sizes, nodes, has_grad, target_elems, cap=64):
    """The engine's data-parallel gradient buckets (tkm_dp_plan_buckets) for
    tensors in registration order: a list of (start node, first value, value
    count) in exchange order, over the 64-value-aligned gradient slots."""
    n = len(sizes)
    a_n = (_sz * max(n, 1))(*[int(x) for x in sizes])
    a_node = (_i * max(n, 1))(*[int(x) for x in nodes])
    a_has = (_i * max(n, 1))(*[1 if x else 0 for x in has_grad])
    bn, bo, bl = (_i * cap)(), (_sz * cap)(), (_sz * cap)()
    k = lib().tkm_dp_plan_buckets(n, a_n, a_node, a_has, int(target_elems), int(cap), bn, bo, bl)
    return [(bn[i], bo[i], bl[i]) for i in range(k)]


def tkm1_pack(tensors):
    """Serialise float32 arrays in the TKM1 checkpoint layout (magic, count,
    then per tensor: count of values, values)."""
    parts = [np.array([0x544B4D31, len(tensors)], dtype=np.uint32).tobytes()]
    for t in tensors:
        t = np.ascontiguousarray(t, dtype=np.float32).ravel()
        parts.append(np.array([t.size], dtype=np.uint32).tobytes())
        parts.append(t.tobytes())
    return b"".join(parts)


def tkm1_unpack(blob):
    head = np.frombuffer(blob[:8], dtype=np.uint32)
    assert head[0] == 0x544B4D31, "not a TKM1 checkpoint"
    out, off = [], 8
    for _ in range(int(head[1])):
        n = int(np.frombuffer(blob[off:off + 4], dtype=np.uint32)[0])
        off += 4
        out.append(np.frombuffer(blob[off:off + 4 * n], dtype=np.float32).copy())
        off += 4 * n
    return out
