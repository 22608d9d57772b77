"""Tensor-level wrappers of the kernel C ABI (include/oxf.h).

Device memory and streams come from PyTorch (plumbing only); every call goes
through liboxf.so and fails loudly on error. Tensors must be contiguous
float32 CUDA tensors; results are written in place or into `out`.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import CSlice, GemmDesc, Slice, check, lib


def _stream(stream=None):
    if stream is None:
        stream = torch.cuda.current_stream()
    return C.c_void_p(stream.cuda_stream)


def _f32(t: torch.Tensor, name: str = "tensor") -> torch.Tensor:
    if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous()):
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor")
    return t


def cs(t: torch.Tensor | None) -> CSlice:
    if t is None:
        return CSlice(None, 0)
    _f32(t)
    return CSlice(t.data_ptr(), t.numel())


def ms(t: torch.Tensor) -> Slice:
    _f32(t)
    return Slice(t.data_ptr(), t.numel())


def ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(_f32(t).data_ptr())


# ---------------------------------------------------------------- elementwise
def binary(a, b, out, op, stream=None):
    check(lib().oxf_slice_binary(cs(a), cs(b), ms(out), op, _stream(stream)))
    return out


def binary_assign(target, rhs, op, stream=None):
    check(lib().oxf_slice_binary_assign(ms(target), cs(rhs), op, _stream(stream)))
    return target


def unary(x, op, param=0.0, stream=None):
    check(lib().oxf_slice_unary(ms(x), op, float(param), _stream(stream)))
    return x


def sgd_update(w, g, lr, stream=None):
    check(lib().oxf_sgd_update(ms(w), cs(g), float(lr), _stream(stream)))
    return w


def mse_grad(y, t, out, stream=None):
    check(lib().oxf_mse_grad(cs(y), cs(t), ms(out), y.shape[-1], _stream(stream)))
    return out


def loss_rows(y, t, out, stream=None):
    check(lib().oxf_loss_rows(cs(y), cs(t), ms(out), y.shape[-1], _stream(stream)))
    return out


def mse_loss_grad(y, t, row_loss, dy, stream=None):
    check(lib().oxf_mse_loss_grad(cs(y), cs(t), ms(row_loss), ms(dy), y.shape[-1],
                                  _stream(stream)))
    return row_loss, dy


def slice_sum(x, out, stream=None):
    check(lib().oxf_slice_sum(cs(x), ptr(out), _stream(stream)))
    return out


def slice_max(x, out, stream=None):
    check(lib().oxf_slice_max(cs(x), ptr(out), _stream(stream)))
    return out


def map_sum(x, op, param, out, stream=None):
    """slice_map_sum: out[0] = sum of the unary op applied to x."""
    check(lib().oxf_slice_map_sum(cs(x), op, float(param), ptr(out), _stream(stream)))
    return out


def dot(x, y, out, stream=None):
    """Vector::dot: out[0] = sum_i x[i] * y[i], one reduction launch."""
    check(lib().oxf_slice_dot(cs(x), cs(y), ptr(out), _stream(stream)))
    return out


def fill(x, value, stream=None):
    check(lib().oxf_slice_set(ms(x), float(value), _stream(stream)))
    return x


def fill_seq(x, ascending=True, stream=None):
    check(lib().oxf_slice_set_seq(ms(x), int(bool(ascending)), _stream(stream)))
    return x


def fill_random(x, seed, stream=None):
    check(lib().oxf_slice_set_random(ms(x), int(seed) & 0xFFFFFFFF, _stream(stream)))
    return x


def matrix_slice(m, out, tile_rows, tile_cols, tiles_per_row, stream=None):
    """matrix_slice: tiles of m (2-D) concatenated into out (1-D or any
    contiguous shape holding a whole number of tiles)."""
    check(lib().oxf_matrix_slice(cs(m), ms(out), m.shape[-1], tile_rows, tile_cols, tiles_per_row,
                                 _stream(stream)))
    return out


def sum_rows(m, out, stream=None):
    check(lib().oxf_matrix_sum_rows(cs(m), ms(out), m.shape[-1], _stream(stream)))
    return out


def sum_cols(m, out, accumulate=False, stream=None):
    check(lib().oxf_matrix_sum_cols(cs(m), ms(out), m.shape[-1], int(accumulate),
                                    _stream(stream)))
    return out


# ---------------------------------------------------------------- row kernels
def softmax_rows(m, scale=1.0, causal_period=0, stream=None):
    check(lib().oxf_matrix_softmax_rows(ms(m), m.shape[-1], float(scale), int(causal_period),
                                        _stream(stream)))
    return m


def layer_norm_rows(m, eps=1e-5, gamma=None, beta=None, stream=None):
    check(lib().oxf_matrix_layer_norm_rows(ms(m), m.shape[-1], float(eps), ptr(gamma), ptr(beta),
                                           _stream(stream)))
    return m


def rms_norm_rows(m, eps=1e-5, gamma=None, stream=None):
    check(lib().oxf_rms_norm_assign(ms(m), m.shape[-1], float(eps), ptr(gamma), _stream(stream)))
    return m


def norm_rows(x, out, norm_type, eps=1e-5, gamma=None, beta=None, stream=None):
    check(lib().oxf_norm_rows(cs(x), ms(out), x.shape[-1], int(norm_type), float(eps), ptr(gamma),
                              ptr(beta), _stream(stream)))
    return out


def norm_rows_backward(x, dy, out, norm_type, eps=1e-5, stream=None):
    check(lib().oxf_norm_rows_backward(cs(x), cs(dy), ms(out), x.shape[-1], int(norm_type),
                                       float(eps), _stream(stream)))
    return out


def binary_broadcast(a, b, out, op, stream=None):
    check(lib().oxf_slice_binary_broadcast(cs(a), cs(b), ms(out), op, _stream(stream)))
    return out


def mul_act_derivative(g, pre, act, stream=None):
    check(lib().oxf_slice_mul_act_derivative(ms(g), cs(pre), int(act), _stream(stream)))
    return g


def softmax_backward(p, dy, out, scale=1.0, stream=None):
    check(lib().oxf_softmax_rows_backward(cs(p), cs(dy), ms(out), p.shape[-1], float(scale),
                                          _stream(stream)))
    return out


def layer_norm_backward(x, dy, out, eps=1e-5, stream=None):
    check(lib().oxf_layer_norm_backward(cs(x), cs(dy), ms(out), x.shape[-1], float(eps),
                                        _stream(stream)))
    return out


def rms_norm_backward(x, dy, out, eps=1e-5, stream=None):
    check(lib().oxf_matrix_rms_norm_backward(cs(x), cs(dy), ms(out), x.shape[-1], float(eps),
                                             _stream(stream)))
    return out


def binary_assign_by_rows(m, row, op, stream=None):
    check(lib().oxf_matrix_binary_assign_by_rows(ms(m), cs(row), m.shape[-1], op,
                                                 _stream(stream)))
    return m


def causal_mask(m, stream=None):
    check(lib().oxf_matrix_causal_mask(ms(m), m.shape[-1], _stream(stream)))
    return m


def transpose(m, out, stream=None):
    check(lib().oxf_matrix_transpose(cs(m), ms(out), m.shape[0], m.shape[1], _stream(stream)))
    return out


# ---------------------------------------------------------------- GEMM
def matrix_multiply(a, b, out, stream=None):
    """module.rs:179-191 argument order: out[rows,cols] = a[rows,len]·b[len,cols]."""
    check(lib().oxf_matrix_multiply(cs(a), cs(b), ms(out), a.shape[1], a.shape[0], b.shape[1],
                                    _stream(stream)))
    return out


def matrix_multiply_fp32(a, b, out, stream=None):
    """module.rs:165-177 argument order; f32 products on the CUDA cores."""
    check(lib().oxf_matrix_multiply_fp32(cs(a), cs(b), ms(out), a.shape[1], a.shape[0], b.shape[1],
                                         _stream(stream)))
    return out


def matrix_multiply_refalgo(a, b, out, stream=None):
    check(lib().oxf_matrix_multiply_refalgo(cs(a), cs(b), ms(out), a.shape[1], a.shape[0],
                                            b.shape[1], _stream(stream)))
    return out


def gemm(a, b, out, *, a_trans=False, b_trans=False, alpha=1.0, beta=0.0, bias=None,
         residual=None, pre_out=None, aux=None, act=_lib.ACT_IDENTITY, grad_act=_lib.ACT_IDENTITY,
         accumulate=False, split_k=0, precision=_lib.PREC_TF32, workspace=None, reduce_batch=False,
         variant=0, stream=None):
    """out = epilogue(alpha * op(a)·op(b)); 2-D or batched 3-D operands.

    a: [M,K] (or [K,M] with a_trans), b: [K,N] (or [N,K] with b_trans); a
    leading batch dimension on any operand makes it per-batch (a 2-D operand
    is shared across the batch). Matrices may be row-strided views (unit
    stride along rows); leading dimensions and batch strides come from the
    tensors' strides."""
    def dims(t):
        return (t.shape[0], t.shape[1], t.shape[2]) if t.dim() == 3 else (1, t.shape[0], t.shape[1])

    def lds(t, name):
        """(leading dimension, batch stride) in elements."""
        if not (t.is_cuda and t.dtype == torch.float32) or t.dim() not in (2, 3):
            raise ValueError(f"{name} must be a 2-D or 3-D float32 CUDA tensor")
        if t.numel() == 0:
            return t.shape[-1], 0
        if t.shape[-1] > 1 and t.stride(-1) != 1:
            raise ValueError(f"{name} must have unit stride along its rows")
        ld = t.stride(-2) if t.shape[-2] > 1 else t.shape[-1]
        return ld, (t.stride(0) if t.dim() == 3 else 0)

    ba, ar, ac = dims(a)
    bb, br, bc = dims(b)
    bo, M, N = dims(out)
    batch = max(ba, bb, bo)
    K = ar if a_trans else ac
    d = GemmDesc()
    lib().oxf_gemm_desc_init(C.byref(d), M, N, K, int(a_trans), int(b_trans), a.data_ptr(),
                             b.data_ptr(), out.data_ptr())
    d.batch = batch
    d.lda, d.stride_a = lds(a, "a")
    d.ldb, d.stride_b = lds(b, "b")
    d.ldc, d.stride_c = lds(out, "out")
    d.alpha, d.beta = float(alpha), float(beta)
    if bias is not None:
        d.bias = _f32(bias).data_ptr()
    for name, t, ldn, sn in (("residual", residual, "ldr", "stride_r"),
                             ("pre_out", pre_out, "ldp", "stride_p"),
                             ("aux", aux, "ldx", "stride_x")):
        if t is not None:
            setattr(d, name, t.data_ptr())
            ld, st = lds(t, name)
            setattr(d, ldn, ld)
            setattr(d, sn, st)
    d.act, d.grad_act = int(act), int(grad_act)
    d.accumulate, d.split_k, d.precision = int(accumulate), int(split_k), int(precision)
    d.reduce_batch = int(reduce_batch)
    d.variant = int(variant)
    if reduce_batch:
        d.stride_c = 0
    if precision == _lib.PREC_TF32X3:
        need = lib().oxf_gemm_workspace_size(C.byref(d))
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            raise ValueError(f"TF32X3 needs a workspace of {need} bytes")
        d.workspace, d.workspace_bytes = workspace.data_ptr(), need
    check(lib().oxf_gemm(C.byref(d), _stream(stream)))
    return out


def gemm_workspace_bytes(M, N, K, a_trans=False, b_trans=False, batch=1, batched_a=False,
                         batched_b=False, precision=_lib.PREC_TF32X3) -> int:
    d = GemmDesc()
    lib().oxf_gemm_desc_init(C.byref(d), M, N, K, int(a_trans), int(b_trans), None, None, None)
    d.batch = batch
    d.stride_a = 1 if batched_a else 0
    d.stride_b = 1 if batched_b else 0
    d.precision = precision
    return int(lib().oxf_gemm_workspace_size(C.byref(d)))


def attention_stats_floats(batch: int, seq: int) -> int:
    return int(lib().oxf_attention_stats_floats(int(batch), int(seq)))


def attention_forward(q, k, v, out, scores, stats, scale, residual=None, causal=False,
                      stream=None):
    """out = residual + softmax(scale * Q·Kᵀ [causal]) · V per sequence
    (oxf_attention_forward). q, k: [batch, seq, d_qk]; v, out, residual:
    [batch, seq, d_v]; scores: [batch, seq, seq] workspace; stats:
    attention_stats_floats(batch, seq) floats of workspace."""
    batch, seq, dqk = q.shape
    dv = v.shape[-1]
    for name, tns in (("q", q), ("k", k), ("v", v), ("out", out), ("scores", scores),
                      ("stats", stats), ("residual", residual)):
        if tns is not None:
            _f32(tns, name)
    if stats.numel() < attention_stats_floats(batch, seq):
        raise ValueError("stats workspace too small")
    check(lib().oxf_attention_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                      residual.data_ptr() if residual is not None else None,
                                      out.data_ptr(), scores.data_ptr(), stats.data_ptr(), batch,
                                      seq, dqk, dv, float(scale), int(causal), _stream(stream)))
    return out


def attention_heads_forward(q, k, v, out, heads, residual=None, causal=False, stream=None):
    """Multi-head attention in one fused kernel (oxf_attention_heads_forward):
    out[..., j*w:(j+1)*w] = residual + softmax(Q_j·K_jᵀ/sqrt(w))·V_j, w =
    d/heads. q, k: [batch, seq, d_qk]; v, out, residual: [batch, seq, d_v]."""
    batch, seq, dqk = q.shape
    dv = v.shape[-1]
    for name, tns in (("q", q), ("k", k), ("v", v), ("out", out), ("residual", residual)):
        if tns is not None:
            _f32(tns, name)
    check(lib().oxf_attention_heads_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                            residual.data_ptr() if residual is not None else None,
                                            out.data_ptr(), batch, seq, dqk, dv, int(heads),
                                            int(causal), _stream(stream)))
    return out


def device_error() -> int:
    code = C.c_uint32(0)
    check(lib().oxf_device_error(C.byref(code)))
    return int(code.value)
