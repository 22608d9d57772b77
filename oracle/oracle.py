"""ctypes wrapper of the C oracle (oxf_oracle.h).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline / reference arm, as the checker or the timed CPU
baseline. Never imported by the product package.

PARITY UNPINNED against the reference (see oxf_oracle.h): pinned instead by
hand-derived known answers and independent numpy fixtures (tests/golden/).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SO = HERE / "_build" / "liboxf_oracle.so"

F32 = np.float32
GEMM_F32, GEMM_TF32_RNA, GEMM_TF32_RZ = 0, 1, 2
IDENTITY, GELU, RELU, SILU = 0, 1, 2, 3
NORM_RMS, NORM_LAYER = 0, 1

_lib = None


def build() -> Path:
    """Compiles the oracle with its Makefile (gcc)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return SO


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not SO.exists():
            build()
        h = C.CDLL(str(SO))
        fp = C.POINTER(C.c_float)
        sz = C.c_size_t
        sigs = {
            "oxo_set_threads": (C.c_int, [C.c_int]),
            "oxo_get_threads": (C.c_int, []),
            "oxo_tf32_rna": (C.c_float, [C.c_float]),
            "oxo_tf32_rz": (C.c_float, [C.c_float]),
            "oxo_gemm": (None, [fp, fp, fp, sz, sz, sz, C.c_int, C.c_int, C.c_int, C.c_float,
                                C.c_float]),
            "oxo_gemm_mt": (None, [fp, fp, fp, sz, sz, sz, C.c_int, C.c_int, C.c_int, C.c_float,
                                   C.c_float]),
            "oxo_gemm_f64": (None, [fp, fp, C.POINTER(C.c_double), sz, sz, sz, C.c_int,
                                    C.c_int]),
            "oxo_binary": (None, [fp, fp, fp, sz, C.c_int]),
            "oxo_binary_assign": (None, [fp, fp, sz, C.c_int]),
            "oxo_binary_assign_by_rows": (None, [fp, fp, sz, sz, C.c_int]),
            "oxo_act_forward": (C.c_float, [C.c_int, C.c_float]),
            "oxo_act_derivative": (C.c_float, [C.c_int, C.c_float]),
            "oxo_activate": (None, [fp, sz, C.c_int]),
            "oxo_sum_rows": (None, [fp, fp, sz, sz]),
            "oxo_sum_cols": (None, [fp, fp, sz, sz]),
            "oxo_transpose": (None, [fp, fp, sz, sz]),
            "oxo_fill_seq": (None, [fp, sz, C.c_int]),
            "oxo_fill_random": (None, [fp, sz, C.c_uint32]),
            "oxo_unary": (C.c_float, [C.c_int, C.c_float, C.c_float]),
            "oxo_map_sum": (C.c_float, [fp, sz, C.c_int, C.c_float]),
            "oxo_dot": (C.c_float, [fp, fp, sz]),
            "oxo_matrix_slice": (None, [fp, fp, sz, sz, sz, sz, sz]),
            "oxo_exchange_sgd": (None, [C.c_void_p, C.c_void_p, C.c_int, sz, sz, C.c_float]),
            "oxo_causal_mask": (None, [fp, sz, sz, sz]),
            "oxo_softmax_rows": (None, [fp, sz, sz, C.c_float, sz]),
            "oxo_layer_norm_rows": (None, [fp, sz, sz, C.c_float, fp, fp]),
            "oxo_rms_norm_rows": (None, [fp, sz, sz, C.c_float, fp]),
            "oxo_softmax_backward": (None, [fp, fp, fp, sz, sz, C.c_float]),
            "oxo_layer_norm_backward": (None, [fp, fp, fp, sz, sz, C.c_float]),
            "oxo_rms_norm_backward": (None, [fp, fp, fp, sz, sz, C.c_float]),
            "oxo_loss_rows": (None, [fp, fp, fp, sz, sz]),
            "oxo_mse_grad": (None, [fp, fp, fp, sz, sz]),
        }
        for name, (res, args) in sigs.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _define_structs(h)
        _lib = h
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.dtype == F32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _c(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=F32)


def set_threads(n: int) -> int:
    return lib().oxo_set_threads(n)


# ---------------------------------------------------------------- kernels
def gemm(A, B, a_trans=False, b_trans=False, rounding=GEMM_F32, alpha=1.0, threads=True):
    A, B = _c(A), _c(B)
    M = A.shape[1] if a_trans else A.shape[0]
    K = A.shape[0] if a_trans else A.shape[1]
    N = B.shape[0] if b_trans else B.shape[1]
    assert (B.shape[1] if b_trans else B.shape[0]) == K
    Cm = np.zeros((M, N), F32)
    f = lib().oxo_gemm_mt if threads else lib().oxo_gemm
    f(_p(A), _p(B), _p(Cm), M, N, K, int(a_trans), int(b_trans), rounding, alpha, 0.0)
    return Cm


def gemm_f64(A, B, a_trans=False, b_trans=False):
    A, B = _c(A), _c(B)
    M = A.shape[1] if a_trans else A.shape[0]
    K = A.shape[0] if a_trans else A.shape[1]
    N = B.shape[0] if b_trans else B.shape[1]
    Cm = np.zeros((M, N), np.float64)
    lib().oxo_gemm_f64(_p(A), _p(B), Cm.ctypes.data_as(C.POINTER(C.c_double)), M, N, K,
                       int(a_trans), int(b_trans))
    return Cm


def tf32_rna(x: float) -> float:
    return lib().oxo_tf32_rna(x)


def tf32_rz(x: float) -> float:
    return lib().oxo_tf32_rz(x)


def binary(a, b, op):
    a, b = _c(a), _c(b)
    out = np.empty_like(a)
    lib().oxo_binary(_p(a), _p(b), _p(out), a.size, op)
    return out


def binary_assign_by_rows(m, row, op):
    m = _c(m).copy()
    row = _c(row)
    lib().oxo_binary_assign_by_rows(_p(m), _p(row), m.shape[0], m.shape[1], op)
    return m


def act_forward(act, x):
    x = _c(x).copy()
    lib().oxo_activate(_p(x), x.size, act)
    return x


def act_derivative(act, x):
    x = _c(x)
    f = lib().oxo_act_derivative
    return np.array([f(act, float(v)) for v in x.ravel()], F32).reshape(x.shape)


def sum_rows(m):
    m = _c(m)
    out = np.empty(m.shape[0], F32)
    lib().oxo_sum_rows(_p(m), _p(out), m.shape[0], m.shape[1])
    return out


def sum_cols(m):
    m = _c(m)
    out = np.empty(m.shape[1], F32)
    lib().oxo_sum_cols(_p(m), _p(out), m.shape[0], m.shape[1])
    return out


def transpose(m):
    m = _c(m)
    out = np.empty((m.shape[1], m.shape[0]), F32)
    lib().oxo_transpose(_p(m), _p(out), m.shape[0], m.shape[1])
    return out


def fill_seq(n, ascending=True):
    out = np.empty(n, F32)
    lib().oxo_fill_seq(_p(out), n, int(bool(ascending)))
    return out


def fill_random(n, seed):
    out = np.empty(n, F32)
    lib().oxo_fill_random(_p(out), n, int(seed) & 0xFFFFFFFF)
    return out


def map_sum(x, op, param=0.0):
    x = _c(x)
    return float(lib().oxo_map_sum(_p(x), x.size, op, param))


def exchange_sgd(params: list, grads: list, offset: int, count: int, lr: float) -> list:
    """Every rank's parameters after the data-parallel update of
    [offset, offset+count) (oxo_exchange_sgd); inputs are not modified."""
    ps = [_c(p).copy() for p in params]
    gs = [_c(g) for g in grads]
    W = len(ps)
    pp = (C.c_void_p * W)(*[p.ctypes.data for p in ps])
    gp = (C.c_void_p * W)(*[g.ctypes.data for g in gs])
    lib().oxo_exchange_sgd(pp, gp, W, offset, count, lr)
    return ps


def dot(x, y):
    x, y = _c(x), _c(y)
    return float(lib().oxo_dot(_p(x), _p(y), x.size))


def matrix_slice(m, tile_rows, tile_cols, tiles_per_row, n_tiles):
    m = _c(m)
    out = np.empty(n_tiles * tile_rows * tile_cols, F32)
    lib().oxo_matrix_slice(_p(m), _p(out), out.size, m.shape[1], tile_rows, tile_cols,
                           tiles_per_row)
    return out


def causal_mask(m, period=0):
    m = _c(m).copy()
    lib().oxo_causal_mask(_p(m), m.shape[0], m.shape[1], period)
    return m


def softmax_rows(m, scale=1.0, causal_period=0):
    m = _c(m).copy()
    lib().oxo_softmax_rows(_p(m), m.shape[0], m.shape[1], scale, causal_period)
    return m


def layer_norm_rows(m, eps=1e-5, gamma=None, beta=None):
    m = _c(m).copy()
    g = _c(gamma) if gamma is not None else None
    b = _c(beta) if beta is not None else None
    lib().oxo_layer_norm_rows(_p(m), m.shape[0], m.shape[1], eps, _p(g), _p(b))
    return m


def rms_norm_rows(m, eps=1e-5, gamma=None):
    m = _c(m).copy()
    g = _c(gamma) if gamma is not None else None
    lib().oxo_rms_norm_rows(_p(m), m.shape[0], m.shape[1], eps, _p(g))
    return m


def softmax_backward(p, dy, scale=1.0):
    p, dy = _c(p), _c(dy)
    dx = np.empty_like(p)
    lib().oxo_softmax_backward(_p(p), _p(dy), _p(dx), p.shape[0], p.shape[1], scale)
    return dx


def layer_norm_backward(x, dy, eps=1e-5):
    x, dy = _c(x), _c(dy)
    dx = np.empty_like(x)
    lib().oxo_layer_norm_backward(_p(x), _p(dy), _p(dx), x.shape[0], x.shape[1], eps)
    return dx


def rms_norm_backward(x, dy, eps=1e-5):
    x, dy = _c(x), _c(dy)
    dx = np.empty_like(x)
    lib().oxo_rms_norm_backward(_p(x), _p(dy), _p(dx), x.shape[0], x.shape[1], eps)
    return dx


def loss_rows(y, t):
    y, t = _c(y), _c(t)
    out = np.empty(y.shape[0], F32)
    lib().oxo_loss_rows(_p(y), _p(t), _p(out), y.shape[0], y.shape[1])
    return out


def mse_grad(y, t):
    y, t = _c(y), _c(t)
    out = np.empty_like(y)
    lib().oxo_mse_grad(_p(y), _p(t), _p(out), y.shape[0], y.shape[1])
    return out


# ---------------------------------------------------------------- executors
class Linear(C.Structure):
    _fields_ = [("w", C.POINTER(C.c_float)), ("b", C.POINTER(C.c_float)), ("in_", C.c_size_t),
                ("out", C.c_size_t), ("act", C.c_int)]


class Mlp(C.Structure):
    _fields_ = [("layers", C.POINTER(Linear)), ("n_layers", C.c_size_t), ("res_start", C.c_int),
                ("res_end", C.c_int)]


class Transformer(C.Structure):
    _fields_ = [("seq", C.c_size_t), ("hidden", C.c_size_t), ("out", C.c_size_t),
                ("norm", C.c_int), ("q", Linear), ("k", Linear), ("v", Linear),
                ("position", C.POINTER(C.c_float)), ("ffn", Mlp), ("o", Linear)]


def _define_structs(h):
    fp = C.POINTER(C.c_float)
    sigs = {
        "oxo_linear_forward": (None, [C.POINTER(Linear), fp, fp, fp, fp, C.c_size_t, C.c_int]),
        "oxo_mlp_forward": (None, [C.POINTER(Mlp), fp, fp, C.POINTER(fp), C.c_size_t, C.c_int]),
        "oxo_mlp_backward": (None, [C.POINTER(Mlp), C.POINTER(fp), fp, fp, C.c_size_t, C.c_float,
                                    C.c_int]),
        "oxo_transformer_forward": (None, [C.POINTER(Transformer), fp, fp, C.c_int, C.c_int]),
        "oxo_transformer_train_step": (None, [C.POINTER(Transformer), fp, fp, fp, fp, fp,
                                              C.c_float, fp, C.c_int]),
        "oxo_transformer_param_count": (C.c_size_t, [C.POINTER(Transformer)]),
        "oxo_transformer_forward_heads": (None, [C.POINTER(Transformer), fp, fp, C.c_int,
                                                 C.c_int, C.c_int]),
        "oxo_transformer_train_step_heads": (None, [C.POINTER(Transformer), fp, fp, fp, fp, fp,
                                                    C.c_float, fp, C.c_int, C.c_int]),
        "oxo_attention_forward_heads": (None, [fp, fp, fp, fp, fp, C.c_size_t, C.c_size_t,
                                               C.c_size_t, C.c_size_t, C.c_int, C.c_int]),
        "oxo_attention_backward_heads": (None, [fp, fp, fp, fp, fp, fp, fp, fp, C.c_size_t,
                                                C.c_size_t, C.c_size_t, C.c_size_t, C.c_int]),
    }
    for name, (res, args) in sigs.items():
        f = getattr(h, name)
        f.restype = res
        f.argtypes = args


class LinearParams:
    """Host copy of one Linear layer: W [in,out], optional bias [out]."""

    def __init__(self, w, b=None, act=IDENTITY):
        self.w = _c(w).copy()
        self.b = None if b is None else _c(b).copy()
        self.act = act

    def struct(self) -> Linear:
        return Linear(_p(self.w), _p(self.b) if self.b is not None else None, self.w.shape[0],
                      self.w.shape[1], self.act)

    def params(self):
        return [self.w] + ([self.b] if self.b is not None else [])


def linear_forward(layer: LinearParams, x, residual=None, rounding=GEMM_F32):
    x = _c(x)
    rows = x.shape[0]
    y = np.empty((rows, layer.w.shape[1]), F32)
    pre = np.empty_like(y)
    s = layer.struct()
    r = _c(residual) if residual is not None else None
    lib().oxo_linear_forward(C.byref(s), _p(x), _p(r), _p(y), _p(pre), rows, rounding)
    return y, pre


class MlpParams:
    def __init__(self, layers, res_range=None):
        self.layers = list(layers)
        self.res = res_range

    def struct(self):
        arr = (Linear * len(self.layers))(*[l.struct() for l in self.layers])
        rs, re = self.res if self.res is not None else (-1, -1)
        return Mlp(arr, len(self.layers), rs, re), arr

    def params(self):
        return [p for l in self.layers for p in l.params()]


def mlp_forward(m: MlpParams, x, rounding=GEMM_F32):
    x = _c(x)
    rows = x.shape[0]
    y = np.empty((rows, m.layers[-1].w.shape[1]), F32)
    s, keep = m.struct()
    lib().oxo_mlp_forward(C.byref(s), _p(x), _p(y), None, rows, rounding)
    return y


def mlp_train_step(m: MlpParams, x, dy, lr, rounding=GEMM_F32):
    """Forward (taping layer inputs) then backward with immediate SGD
    (mlp.rs:121-168). Updates m's arrays in place; returns (y, dx)."""
    x = _c(x)
    rows = x.shape[0]
    y = np.empty((rows, m.layers[-1].w.shape[1]), F32)
    tape = [np.empty((rows, l.w.shape[0]), F32) for l in m.layers]
    s, keep = m.struct()
    tp = (C.POINTER(C.c_float) * len(tape))(*[_p(t) for t in tape])
    lib().oxo_mlp_forward(C.byref(s), _p(x), _p(y), tp, rows, rounding)
    dx = np.empty_like(x)
    lib().oxo_mlp_backward(C.byref(s), tp, _p(_c(dy)), _p(dx), rows, lr, rounding)
    return y, dx


class TransformerParams:
    """Host copy of a single-block transformer in cursor order
    (inference.rs:52-66): q, k, v, position, ffn layers, output."""

    def __init__(self, q, k, v, position, ffn: MlpParams, o, norm, seq):
        self.q, self.k, self.v, self.o = q, k, v, o
        self.position = _c(position).copy()
        self.ffn = ffn
        self.norm = norm
        self.seq = seq

    def struct(self):
        f, keep = self.ffn.struct()
        t = Transformer(self.seq, self.position.shape[1], self.o.w.shape[1], self.norm,
                        self.q.struct(), self.k.struct(), self.v.struct(), _p(self.position), f,
                        self.o.struct())
        return t, keep

    def params(self):
        return (self.q.params() + self.k.params() + self.v.params() + [self.position] +
                self.ffn.params() + self.o.params())

    def flat(self):
        return np.concatenate([p.ravel() for p in self.params()])

    def copy(self):
        import copy
        return copy.deepcopy(self)


def transformer_forward(t: TransformerParams, x, causal=False, rounding=GEMM_F32, heads=1):
    """Inference forward of one sequence; heads > 1 splits the attention
    into that many heads (oxo_attention_forward_heads)."""
    x = _c(x)
    y = np.empty((t.seq, t.o.w.shape[1]), F32)
    s, keep = t.struct()
    if heads == 1:
        lib().oxo_transformer_forward(C.byref(s), _p(x), _p(y), int(causal), rounding)
    else:
        lib().oxo_transformer_forward_heads(C.byref(s), _p(x), _p(y), int(causal), rounding,
                                            int(heads))
    return y


def transformer_train_step(t: TransformerParams, x, target, lr, grads=None, rounding=GEMM_F32,
                           heads=1):
    """One reference training step on one sequence. Returns (y, row_loss, dx).
    If `grads` (flat, cursor order) is given, parameter gradients are added
    to it. heads > 1: multi-head attention."""
    x, target = _c(x), _c(target)
    y = np.empty((t.seq, t.o.w.shape[1]), F32)
    loss = np.empty(t.seq, F32)
    dx = np.empty_like(x)
    s, keep = t.struct()
    g = _p(grads) if grads is not None else None
    if heads == 1:
        lib().oxo_transformer_train_step(C.byref(s), _p(x), _p(target), _p(y), _p(loss), _p(dx),
                                         lr, g, rounding)
    else:
        lib().oxo_transformer_train_step_heads(C.byref(s), _p(x), _p(target), _p(y), _p(loss),
                                               _p(dx), lr, g, rounding, int(heads))
    return y, loss, dx


def attention_heads(q, k, v, heads, causal=False, rounding=GEMM_F32):
    """The attention core alone: (att [S, Hv], P [heads, S, S])."""
    q, k, v = _c(q), _c(k), _c(v)
    S, D = q.shape
    Hv = v.shape[1]
    att = np.empty((S, Hv), F32)
    p = np.empty((heads, S, S), F32)
    lib().oxo_attention_forward_heads(_p(q), _p(k), _p(v), _p(p), _p(att), S, D, Hv, heads,
                                      int(causal), rounding)
    return att, p


def attention_heads_backward(q, k, v, p, dr, heads, rounding=GEMM_F32):
    """Gradients (dq, dk, dv) of the attention core given dL/d(att) = dr."""
    q, k, v, p, dr = _c(q), _c(k), _c(v), _c(p), _c(dr)
    S, D = q.shape
    Hv = v.shape[1]
    dq, dk, dv = np.empty_like(q), np.empty_like(k), np.empty_like(v)
    lib().oxo_attention_backward_heads(_p(q), _p(k), _p(v), _p(p), _p(dr), _p(dq), _p(dk),
                                       _p(dv), S, D, Hv, heads, rounding)
    return dq, dk, dv
