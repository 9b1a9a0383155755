"""CPU oracle of a whole Tokamak training step -- TEST INFRASTRUCTURE ONLY.

Interprets a compiled TkmGraph (node table after fusion, as the reference's
tkm_optimize_and_bind produces it) node by node in float64 numpy and returns
the loss, every activation, d(loss)/d(input) and the gradient of every
learnable tensor, then applies the reference's SGD.  Imported only by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg.

Semantics followed (reference file:line):
  - tensor registration / TKM1 order: src/tkm_gpu.cu:901-1031 (per node in id
    order, dead nodes included: GEMM weight [K][N], then bias, gain, shift);
  - FC: out = in @ W, W stored [K][N] (src/tkm_gpu.cu:1207-1216);
  - fluid operators: src/tkm_registry.c:258-466 (pointwise definitions);
  - RMSNorm / LN / BN / L2Norm: src/tkm_registry.c:190-256 with the row
    statistics over the whole row (the reference's reduction is only right up
    to 64 channels); LN/BN variance as mean((x - mean)^2);
  - residual Add and the twin `[gate|up]` Mul: src/tkm_codegen.c:484-625 and
    the twin rule src/tkm_registry.c:653-686;
  - QKV prep (bias, QKNorm, RoPE): src/tkm_codegen.c:43-70, 211-295 through
    oracle/tkm_oracle.c (pinned against the reference's golden vectors);
  - GQA attention, softmax and the softmax losses: oracle/tkm_oracle.c;
  - SGD: src/tkm_gpu.cu:684-720 (weight decay on GEMM weights only, Nesterov
    momentum 0.9, wd 1e-4).
Drop is not interpreted (its random mask belongs to the device generator).
"""
import math

import numpy as np

from . import attn_bwd, attn_fwd, qkv_prep_bwd, qkv_prep_fwd, sgd, softmax_bwd, softmax_fwd, softmax_loss

# operator enum values of include/tkm.h
OP = {name: i for i, name in enumerate([
    "NONE", "INPUT", "CONV", "FC", "FC_TWIN_FUSED", "FC_QKV_FUSED", "GQA_ATTN", "MIXPOOL", "AVGPOOL", "FLATTEN",
    "BORDER_REFLECT", "RAND_SHIFT", "RAND_ROTATE", "RAND_SCALE", "RAND_FLIPX", "RAND_FLIPY", "RAND_ELASTIC",
    "RAND_NOISE", "RAND_CUTOUT", "RAND_BRIGHTNESS", "RAND_CONTRAST", "RAND_SATURATION", "RAND_HUE",
    "RAND_GRAYSCALE", "RAND_CHANNEL_SCALE", "RAND_SOLARIZE", "RAND_ERASING", "BN", "LN", "RMSNORM", "L2NORM",
    "QKNORM", "BIAS", "SILU", "RELU", "RELU2", "LEAKY_RELU", "ELU", "GELU", "MISH", "HARDSWISH", "HARDSIGMOID",
    "TANH", "SIGMOID", "SWISH_BETA", "SIN", "COSGATE", "SOFTCAP", "CLAMP", "SCALE", "LAYERSCALE", "DYT", "PRELU",
    "XATLU", "ROPE", "DROP", "ADD", "MUL", "SOFTMAX", "SOFTMAX_CE", "SOFTMAX_FOCAL", "SOFTMAX_MSE", "USER_FLUID",
    "COUNT"])}
RES_BIAS, RES_WEIGHT, RES_BETA = 1, 2, 4
FC_OPS = (OP["FC"], OP["FC_TWIN_FUSED"], OP["FC_QKV_FUSED"])
LOSS_OPS = (OP["SOFTMAX_CE"], OP["SOFTMAX_FOCAL"], OP["SOFTMAX_MSE"])


def _sig(x):
    return 0.5 * (1.0 + np.tanh(0.5 * x))


def _softplus20(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))


_GELU_K = math.sqrt(2.0 / math.pi)


def pointwise(op, x, f, w=None):
    """(y, dy/dx, dy/dw or None) of a pointwise operator; w = per-channel gain."""
    if op == OP["SILU"]:
        s = _sig(x)
        return x * s, s * (1 + x * (1 - s)), None
    if op == OP["RELU"]:
        return np.maximum(x, 0), (x > 0).astype(x.dtype), None
    if op == OP["RELU2"]:
        r = np.maximum(x, 0)
        return r * r, np.where(x > 0, 2 * x, 0.0), None
    if op == OP["LEAKY_RELU"]:
        return np.where(x > 0, x, x * f), np.where(x > 0, 1.0, f), None
    if op == OP["ELU"]:
        return np.where(x > 0, x, f * np.expm1(np.minimum(x, 0))), np.where(x > 0, 1.0, f * np.exp(np.minimum(x, 0))), None
    if op == OP["GELU"]:
        u = _GELU_K * (x + 0.044715 * x ** 3)
        t = np.tanh(u)
        return 0.5 * x * (1 + t), 0.5 * (1 + t) + 0.5 * x * (1 - t * t) * _GELU_K * (1 + 3 * 0.044715 * x * x), None
    if op == OP["MISH"]:
        t = np.tanh(_softplus20(x))
        return x * t, t + x * (1 - t * t) * _sig(x), None
    if op == OP["HARDSWISH"]:
        return x * np.clip(x + 3, 0, 6) / 6, np.where(x <= -3, 0.0, np.where(x >= 3, 1.0, (2 * x + 3) / 6)), None
    if op == OP["HARDSIGMOID"]:
        return np.clip((x + 3) / 6, 0, 1), np.where((x > -3) & (x < 3), 1 / 6, 0.0), None
    if op == OP["TANH"]:
        t = np.tanh(x)
        return t, 1 - t * t, None
    if op == OP["SIGMOID"]:
        s = _sig(x)
        return s, s * (1 - s), None
    if op == OP["SWISH_BETA"]:
        s = _sig(f * x)
        return x * s, s * (1 + f * x * (1 - s)), None
    if op == OP["SIN"]:
        return np.sin(f * x), f * np.cos(f * x), None
    if op == OP["COSGATE"]:
        return x * np.cos(x), np.cos(x) - x * np.sin(x), None
    if op == OP["SOFTCAP"]:
        t = np.tanh(x / f)
        return f * t, 1 - t * t, None
    if op == OP["CLAMP"]:
        return np.clip(x, -f, f), ((x > -f) & (x < f)).astype(x.dtype), None
    if op == OP["SCALE"]:
        return x * f, np.full_like(x, f), None
    if op == OP["LAYERSCALE"]:
        return x * w, np.broadcast_to(w, x.shape), x
    if op == OP["DYT"]:
        t = np.tanh(f * x)
        return t * w, w * f * (1 - t * t), t
    if op == OP["PRELU"]:
        return np.where(x > 0, x, x * w * f), np.where(x > 0, 1.0, w * f), np.where(x > 0, 0.0, x * f)
    if op == OP["XATLU"]:
        s = _sig(x)
        return x * (w * s + 1 - w), (1 - w) + w * s * (1 + x * (1 - s)), x * (s - 1)
    raise NotImplementedError(f"operator {op}")


def formula(expr, x, fval):
    """Evaluate a registry formula (x, fval, pi, exp log ln sqrt sin cos tanh
    abs max min pow) elementwise."""
    env = {"x": x, "fval": fval, "pi": math.pi, "exp": np.exp, "log": np.log, "ln": np.log, "sqrt": np.sqrt,
           "sin": np.sin, "cos": np.cos, "tanh": np.tanh, "abs": np.abs, "max": np.maximum, "min": np.minimum,
           "pow": np.power, "__builtins__": {}}
    return np.asarray(eval(expr, env, {}), dtype=np.float64) * np.ones_like(x)  # noqa: S307 (registry formulas)


def loss_fwd_bwd(logits, labels, kind, gamma):
    """Softmax losses of src/tkm_gpu.cu:632-682 in float64: mean over rows of
    -log(max(p_y, 1e-7)) (kind 0), of -(1-p_y)^gamma log p_y (kind 1, focal),
    of sum_c (p_c - onehot_c)^2 / C (kind 2, Brier); d logits carries the
    reference's 1/rows scaling and its focal gradient factor."""
    rows, C = logits.shape
    z = logits - logits.max(axis=1, keepdims=True)
    p = np.exp(z)
    p /= p.sum(axis=1, keepdims=True)
    onehot = np.zeros_like(p)
    onehot[np.arange(rows), labels] = 1.0
    py = np.maximum(p[np.arange(rows), labels], 1e-7)
    if kind == 0:
        per_row = -np.log(py)
        grad = p - onehot
    elif kind == 1:
        w = (1.0 - py) ** gamma
        per_row = -w * np.log(py)
        scale = w - gamma * py * (1.0 - py) ** (gamma - 1.0) * np.log(py)
        grad = scale[:, None] * (p - onehot)
    else:
        diff = p - onehot
        per_row = (diff * diff).sum(axis=1) / C
        dot = (p * diff).sum(axis=1, keepdims=True)
        grad = (2.0 / C) * p * (diff - dot)
    return float(per_row.sum() / rows), grad / rows


def _norm_fwd(x, eps, centered):
    m = x.mean(axis=1, keepdims=True) if centered else 0.0
    d = x - m
    var = (d * d).mean(axis=1, keepdims=True)
    r = 1.0 / np.sqrt(var + eps)
    return d * r, r


def _norm_bwd(dxh, xh, r, centered):
    m2 = (dxh * xh).mean(axis=1, keepdims=True)
    m1 = dxh.mean(axis=1, keepdims=True) if centered else 0.0
    return r * (dxh - m1 - xh * m2)


class GraphOracle:
    """Float64 interpreter of one compiled graph.

    `graph` is an oracle.tkm_abi.Graph; `specs` maps spec index -> (dsl_name,
    res_flags, fwd_expr, bwd_expr, op) of the registry that compiled it."""

    def __init__(self, graph, specs):
        self.g = graph
        self.B = graph.batch_size
        self.specs = specs
        self.n = graph.num_nodes
        self.nodes = [graph.nodes[i] for i in range(self.n)]
        self.C = [nd.C for nd in self.nodes]
        self.H = [nd.H for nd in self.nodes]
        self.W = [nd.W for nd in self.nodes]
        for i, nd in enumerate(self.nodes):  # width fix-up of the reference's ignite
            if self.C[i] == 0 and nd.in0 >= 0:
                p = self.nodes[nd.in0]
                self.H[i], self.W[i] = self.H[nd.in0], self.W[nd.in0]
                self.C[i] = p.c_out if p.c_out > 0 else self.C[nd.in0]
        self.tensors = []  # (node, kind, size); kind 0 matrix, 1 gain, 2 shift, 3 bias
        self.tidx = {}
        for i, nd in enumerate(self.nodes):
            C = self.C[i]
            if C <= 0:
                continue
            flags = self.flags(i)
            if nd.op in FC_OPS:
                self._add(i, 0, self.C[nd.in0] * C)
            elif nd.op == OP["CONV"]:
                self._add(i, 0, 9 * self.C[nd.in0] * C)
            if flags & RES_BIAS:
                self._add(i, 3, C)
            if flags & RES_WEIGHT:
                self._add(i, 1, C)
            if flags & RES_BETA:
                self._add(i, 2, C)
        self.params = None

    def _add(self, node, kind, size):
        self.tidx[(node, kind)] = len(self.tensors)
        self.tensors.append((node, kind, size))

    def flags(self, i):
        """resource flags of node i's registry entry (found by operator, or by
        spec index for formula operators, as tkm_find_spec_by_node does)"""
        nd = self.nodes[i]
        if nd.op == OP["USER_FLUID"]:
            return self.specs[nd.spec_id][1] if nd.spec_id >= 0 else 0
        for name, flags, fe, be, op in self.specs.values():
            if op == nd.op:
                return flags
        return 0

    def rows(self, i):
        return self.B * self.H[i] * self.W[i]

    def default_params(self):
        out = []
        for node, kind, size in self.tensors:
            out.append(np.full(size, 1.0 if kind == 1 else 0.0))
        return out

    def set_params(self, arrays):
        assert len(arrays) == len(self.tensors)
        self.params = [np.asarray(a, dtype=np.float64).ravel().copy() for a in arrays]

    def P(self, node, kind):
        return self.params[self.tidx[(node, kind)]]

    # ------------------------------------------------------------ pointwise
    def _fluid(self, i, x):
        """y and a backward closure dy -> (dx, {tensor index: grad})."""
        nd = self.nodes[i]
        op = nd.op
        f = float(nd.fval)
        if op == OP["BIAS"]:
            t = self.tidx[(i, 3)]
            return x + self.params[t], lambda dy: (dy, {t: dy.sum(0)})
        if op == OP["USER_FLUID"]:
            _, _, fe, be, _ = self.specs[nd.spec_id]
            y = formula(fe, x, f)
            d = formula(be, x, f)
            return y, lambda dy: (dy * d, {})
        if op in (OP["RMSNORM"], OP["L2NORM"], OP["LN"], OP["BN"]):
            centered = op in (OP["LN"], OP["BN"])
            xh, r = _norm_fwd(x, f, centered)
            y = xh.copy()
            tg = self.tidx.get((i, 1)) if self.flags(i) & RES_WEIGHT else None
            tb = self.tidx.get((i, 2)) if self.flags(i) & RES_BETA else None
            if tg is not None:
                y = y * self.params[tg]
            if tb is not None:
                y = y + self.params[tb]

            def back(dy):
                grads = {}
                dxh = dy
                if tg is not None:
                    grads[tg] = (dy * xh).sum(0)
                    dxh = dy * self.params[tg]
                if tb is not None:
                    grads[tb] = dy.sum(0)
                return _norm_bwd(dxh, xh, r, centered), grads
            return y, back
        if op == OP["DROP"]:
            raise NotImplementedError("Drop draws device random numbers; the oracle does not interpret it")
        w = None
        tw = None
        if self.flags(i) & RES_WEIGHT:
            tw = self.tidx[(i, 1)]
            w = self.params[tw]
        y, d, dw = pointwise(op, x, f, w)

        def back(dy):
            g = {}
            if tw is not None:
                g[tw] = (dy * dw).sum(0)
            return dy * d, g
        return y, back

    # ---------------------------------------------------------------- step
    def run(self, x, labels=None, train=True):
        """Forward (and backward when train): returns a dict with 'loss',
        'acts' (node -> array), 'dinput', 'grads' (tensor index -> array)."""
        B = self.B
        vals = {0: np.asarray(x, dtype=np.float64).reshape(self.rows(0), self.C[0])}
        tape = []
        loss = None
        dlogits = None
        for i in range(1, self.n):
            nd = self.nodes[i]
            if nd.dead:
                continue
            op = nd.op
            if op in FC_OPS:
                W = self.P(i, 0).reshape(self.C[nd.in0], self.C[i])
                a = vals[nd.in0]
                vals[i] = a @ W
                tape.append((i, "fc"))
            elif op == OP["ADD"]:
                vals[i] = vals[nd.in0] + vals[nd.in1]
                tape.append((i, "add"))
            elif op == OP["MUL"] and nd.left_len > 0:
                fc = vals[nd.in0]
                F = self.C[i]
                left, right = fc[:, :F], fc[:, F:]
                lb, rb = [], []
                for k in range(nd.left_len):
                    left, b = self._fluid(nd.left_nodes[k], left)
                    lb.append(b)
                for k in range(nd.right_len):
                    right, b = self._fluid(nd.right_nodes[k], right)
                    rb.append(b)
                vals[i] = left * right
                tape.append((i, ("twin", left, right, lb, rb)))
            elif op == OP["QKNORM"] and nd.q_c > 0:
                S = self.H[i] * self.W[i]
                hd = nd.head_dim
                args = dict(S=S, Hq=nd.q_heads, Hkv=nd.kv_heads, D=hd, qknorm=nd.has_qknorm, rope=nd.has_rope,
                            theta=nd.rope_theta, scale=nd.rope_scale, low=nd.rope_low_freq_factor,
                            high=nd.rope_high_freq_factor, octx=nd.rope_original_context_length)
                xin = vals[nd.in0].astype(np.float32)
                bias = self.P(i, 3).astype(np.float32)
                gain = self.P(i, 1).astype(np.float32)
                out, istd = qkv_prep_fwd(np.ascontiguousarray(xin), bias, gain, **args)
                vals[i] = out.astype(np.float64)
                tape.append((i, ("prep", xin, bias, gain, istd, args)))
            elif op == OP["GQA_ATTN"]:
                S = self.H[i] * self.W[i]
                qkv = np.ascontiguousarray(vals[nd.in0].astype(np.float32))
                sc = 1.0 / math.sqrt(nd.head_dim)
                out, lse = attn_fwd(qkv, B, S, nd.q_heads, nd.kv_heads, nd.head_dim, sc, nd.causal)
                vals[i] = out.reshape(self.rows(i), self.C[i]).astype(np.float64)
                tape.append((i, ("attn", qkv, out, lse, S, sc)))
            elif op == OP["SOFTMAX"]:
                p = softmax_fwd(np.ascontiguousarray(vals[nd.in0].astype(np.float32)))
                vals[i] = p.astype(np.float64)
                tape.append((i, ("softmax", p)))
            elif op in LOSS_OPS:
                kind = {OP["SOFTMAX_CE"]: 0, OP["SOFTMAX_FOCAL"]: 1, OP["SOFTMAX_MSE"]: 2}[op]
                lg = vals[nd.in0]
                lab = np.zeros(lg.shape[0], np.int64) if labels is None else np.asarray(labels, np.int64)
                loss, dl = loss_fwd_bwd(lg, lab, kind, float(nd.fval))
                dlogits = (nd.in0, dl)
            elif op == OP["FLATTEN"]:
                vals[i] = vals[nd.in0].reshape(self.rows(i), self.C[i])
                tape.append((i, "flatten"))
            elif nd.cat in (4, 5):  # CAT_NORM, CAT_FLUID chain members
                y, back = self._fluid(i, vals[nd.in0])
                vals[i] = y
                tape.append((i, ("fluid", back)))
            else:
                raise NotImplementedError(f"node {i} op {op}")
        res = {"loss": loss, "acts": vals}
        if not train:
            return res
        grads = {}
        d = {}

        def acc(node, g):
            d[node] = d[node] + g if node in d else g

        def acc_t(t, g):
            grads[t] = grads[t] + g if t in grads else g

        if dlogits is not None:
            acc(*dlogits)
        for i, item in reversed(tape):
            nd = self.nodes[i]
            if i not in d:
                continue
            dy = d.pop(i)
            if item == "fc":
                W = self.P(i, 0).reshape(self.C[nd.in0], self.C[i])
                acc_t(self.tidx[(i, 0)], (vals[nd.in0].T @ dy).ravel())
                acc(nd.in0, dy @ W.T)
            elif item == "add":
                acc(nd.in0, dy)
                acc(nd.in1, dy)
            elif item == "flatten":
                acc(nd.in0, dy.reshape(self.rows(nd.in0), self.C[nd.in0]))
            elif item[0] == "fluid":
                dx, g = item[1](dy)
                for t, v in g.items():
                    acc_t(t, v)
                acc(nd.in0, dx)
            elif item[0] == "twin":
                _, left, right, lb, rb = item
                dl, dr = dy * right, dy * left
                for b in reversed(lb):
                    dl, g = b(dl)
                    for t, v in g.items():
                        acc_t(t, v)
                for b in reversed(rb):
                    dr, g = b(dr)
                    for t, v in g.items():
                        acc_t(t, v)
                acc(nd.in0, np.concatenate([dl, dr], axis=1))
            elif item[0] == "prep":
                _, xin, bias, gain, istd, args = item
                din, db, dg = qkv_prep_bwd(np.ascontiguousarray(dy.astype(np.float32)), xin, bias, gain, istd, **args)
                acc_t(self.tidx[(i, 3)], db.astype(np.float64))
                if nd.has_qknorm:
                    g = np.zeros(self.C[i])
                    g[:dg.size] = dg
                    acc_t(self.tidx[(i, 1)], g)
                acc(nd.in0, din.astype(np.float64))
            elif item[0] == "attn":
                _, qkv, out, lse, S, sc = item
                dout = np.ascontiguousarray(dy.astype(np.float32).reshape(out.shape))
                dqkv = attn_bwd(qkv, out, dout, lse, self.B, S, nd.q_heads, nd.kv_heads, nd.head_dim, sc, nd.causal)
                acc(nd.in0, dqkv.reshape(qkv.shape[0], -1).astype(np.float64))
            elif item[0] == "softmax":
                p = item[1]
                dx = softmax_bwd(p, np.ascontiguousarray(dy.astype(np.float32)), np.zeros_like(p))
                acc(nd.in0, dx.astype(np.float64))
        res["dinput"] = d.get(0, np.zeros_like(vals[0]))
        res["grads"] = grads
        return res

    def sgd_update(self, grads, lr, vel=None):
        """One reference SGD step on every tensor the graph reads; returns the
        new parameters and velocities (tensors without a gradient keep theirs)."""
        new_p, new_v = [], []
        for t, (node, kind, size) in enumerate(self.tensors):
            p = self.params[t].astype(np.float32)
            v = np.zeros(size, np.float32) if vel is None else vel[t].astype(np.float32)
            if t in grads:
                p, v = sgd(p, v, grads[t].astype(np.float32), lr, apply_wd=(kind == 0))
            new_p.append(p)
            new_v.append(v)
        return new_p, new_v


def specs_of(lib):
    """spec index -> (dsl_name, res_flags, fwd_expr, bwd_expr, op) of a loaded libtkm."""
    out = {}
    for i in range(lib.tkm_get_spec_count()):
        s = lib.tkm_find_spec_by_index(i).contents
        out[i] = (s.dsl_name.decode(), s.res_flags,
                  s.fwd_expr.decode() if s.fwd_expr else None, s.bwd_expr.decode() if s.bwd_expr else None, s.op)
    return out


def reference_front_end():
    """The reference's own host library (oracle/_ref/libtkm_ref_host.so) when it
    was built, else None."""
    import ctypes
    import os
    from .tkm_abi import bind
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libtkm_ref_host.so")
    if not os.path.exists(path):
        return None
    return bind(ctypes.CDLL(path))


def oracle_for(dsl, batch, front_end=None):
    """Compile `dsl` with the reference's front end (or the given one) and
    return a GraphOracle for it."""
    from .tkm_abi import compile_graph
    lib = front_end or reference_front_end()
    if lib is None:
        raise RuntimeError("no front end: build oracle/_ref or pass one")
    g = compile_graph(lib, dsl, batch)
    return GraphOracle(g, specs_of(lib))
