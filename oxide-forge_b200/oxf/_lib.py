"""ctypes binding of liboxf.so (include/oxf.h and include/oxf_host.h).

This is the binding a Python host (tests, bench, the data-parallel driver)
uses to reach the sm_100a kernels. It mirrors how a Rust crate would bind the
same header through FFI. Loading fails loudly if the library is missing:
there is no CPU fallback anywhere in the product path.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent.parent
LIB_PATH = Path(os.environ.get("OXF_LIB", _PKG / "liboxf.so"))

OK, INVALID_ARG, UNSUPPORTED_SHAPE, CUDA_ERROR, TIMEOUT, DEVICE_CHECK, IO, STATE = range(8)
STATUS_NAMES = {0: "OK", 1: "INVALID_ARG", 2: "UNSUPPORTED_SHAPE", 3: "CUDA_ERROR",
                4: "TIMEOUT", 5: "DEVICE_CHECK", 6: "IO", 7: "STATE"}

ADD, SUB, MUL, DIV = 0, 1, 2, 3
ACT_IDENTITY, ACT_GELU, ACT_RELU, ACT_SILU = 0, 1, 2, 3
UNARY_SCALE, UNARY_ADD_SCALAR, UNARY_ACT_FORWARD, UNARY_ACT_DERIV, UNARY_HALF_SQUARE = range(5)
PREC_TF32, PREC_TF32X3, PREC_F32 = 0, 1, 2
NORM_RMS, NORM_LAYER = 0, 1


class OxfError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


class CSlice(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("len", C.c_size_t)]


class Slice(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("len", C.c_size_t)]


class GemmDesc(C.Structure):
    _fields_ = [
        ("M", C.c_int), ("N", C.c_int), ("K", C.c_int), ("batch", C.c_int),
        ("a_trans", C.c_int), ("b_trans", C.c_int),
        ("A", C.c_void_p), ("lda", C.c_longlong), ("stride_a", C.c_longlong),
        ("B", C.c_void_p), ("ldb", C.c_longlong), ("stride_b", C.c_longlong),
        ("C", C.c_void_p), ("ldc", C.c_longlong), ("stride_c", C.c_longlong),
        ("alpha", C.c_float), ("beta", C.c_float),
        ("bias", C.c_void_p),
        ("residual", C.c_void_p), ("ldr", C.c_longlong), ("stride_r", C.c_longlong),
        ("pre_out", C.c_void_p), ("ldp", C.c_longlong), ("stride_p", C.c_longlong),
        ("aux", C.c_void_p), ("ldx", C.c_longlong), ("stride_x", C.c_longlong),
        ("act", C.c_int), ("grad_act", C.c_int), ("accumulate", C.c_int),
        ("split_k", C.c_int), ("precision", C.c_int),
        ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t),
        ("reduce_batch", C.c_int), ("variant", C.c_int),
    ]


# oxf_gemm_plan (oxf.h): the path oxf_gemm takes and its tile, splits, raster.
GEMM_PATH_NONE, GEMM_PATH_SIMT, GEMM_PATH_TINY, GEMM_PATH_ONE_CTA, GEMM_PATH_CTA_PAIR = range(5)


class GemmPlanInfo(C.Structure):
    _fields_ = [
        ("path", C.c_int), ("tile_m", C.c_int), ("tile_n", C.c_int), ("stages", C.c_int),
        ("staging", C.c_int), ("splits", C.c_int), ("group_m", C.c_int), ("zero_c", C.c_int),
        ("units", C.c_longlong),
    ]


# Peer exchange (oxf.h): limits, device error codes, descriptor and handle.
EXCHANGE_MAX_RANKS = 8
EXCHANGE_MAX_BLOCKS = 1024
EXCHANGE_SIGNAL_BYTES = 2 * EXCHANGE_MAX_BLOCKS * EXCHANGE_MAX_RANKS * 4
DEVERR_EXCHANGE_START, DEVERR_EXCHANGE_END = 0x201, 0x202
DEVERR_ROW_PARAMS = 0x301


class IpcHandle(C.Structure):
    _fields_ = [("handle", C.c_ubyte * 64), ("offset", C.c_uint64)]


class ExchangeDesc(C.Structure):
    _fields_ = [
        ("rank", C.c_int), ("world", C.c_int),
        ("params", C.c_void_p * EXCHANGE_MAX_RANKS),
        ("grads", C.c_void_p * EXCHANGE_MAX_RANKS),
        ("signals", C.c_void_p * EXCHANGE_MAX_RANKS),
        ("epoch", C.c_uint32), ("blocks", C.c_int), ("timeout_us", C.c_uint32),
    ]


_lib = None

# name -> (restype, argtypes)
_SIGS = {
    "oxf_last_error_string": (C.c_char_p, []),
    "oxf_version": (C.c_char_p, []),
    "oxf_kernel_launches": (C.c_ulonglong, []),
    "oxf_device_error": (C.c_int, [C.POINTER(C.c_uint32)]),
    "oxf_slice_binary": (C.c_int, [CSlice, CSlice, Slice, C.c_int, C.c_void_p]),
    "oxf_slice_binary_assign": (C.c_int, [Slice, CSlice, C.c_int, C.c_void_p]),
    "oxf_slice_unary": (C.c_int, [Slice, C.c_int, C.c_float, C.c_void_p]),
    "oxf_sgd_update": (C.c_int, [Slice, CSlice, C.c_float, C.c_void_p]),
    "oxf_mse_grad": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_void_p]),
    "oxf_loss_rows": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_void_p]),
    "oxf_mse_loss_grad": (C.c_int, [CSlice, CSlice, Slice, Slice, C.c_size_t, C.c_void_p]),
    "oxf_slice_sum": (C.c_int, [CSlice, C.c_void_p, C.c_void_p]),
    "oxf_slice_max": (C.c_int, [CSlice, C.c_void_p, C.c_void_p]),
    "oxf_slice_map_sum": (C.c_int, [CSlice, C.c_int, C.c_float, C.c_void_p, C.c_void_p]),
    "oxf_slice_dot": (C.c_int, [CSlice, CSlice, C.c_void_p, C.c_void_p]),
    "oxf_slice_set": (C.c_int, [Slice, C.c_float, C.c_void_p]),
    "oxf_wait_timeout_selftest": (C.c_int, [C.c_uint32, C.c_void_p, C.c_void_p]),
    "oxf_slice_set_seq": (C.c_int, [Slice, C.c_int, C.c_void_p]),
    "oxf_slice_set_random": (C.c_int, [Slice, C.c_uint32, C.c_void_p]),
    "oxf_matrix_slice": (C.c_int, [CSlice, Slice, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                                   C.c_void_p]),
    "oxf_matrix_sum_rows": (C.c_int, [CSlice, Slice, C.c_size_t, C.c_void_p]),
    "oxf_matrix_sum_cols": (C.c_int, [CSlice, Slice, C.c_size_t, C.c_int, C.c_void_p]),
    "oxf_matrix_softmax_rows": (C.c_int, [Slice, C.c_size_t, C.c_float, C.c_size_t, C.c_void_p]),
    "oxf_matrix_layer_norm_rows": (C.c_int, [Slice, C.c_size_t, C.c_float, C.c_void_p,
                                             C.c_void_p, C.c_void_p]),
    "oxf_rms_norm_assign": (C.c_int, [Slice, C.c_size_t, C.c_float, C.c_void_p, C.c_void_p]),
    "oxf_norm_rows": (C.c_int, [CSlice, Slice, C.c_size_t, C.c_int, C.c_float, C.c_void_p,
                                C.c_void_p, C.c_void_p]),
    "oxf_norm_rows_backward": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_int, C.c_float,
                                         C.c_void_p]),
    "oxf_slice_binary_broadcast": (C.c_int, [CSlice, CSlice, Slice, C.c_int, C.c_void_p]),
    "oxf_slice_mul_act_derivative": (C.c_int, [Slice, CSlice, C.c_int, C.c_void_p]),
    "oxf_softmax_rows_backward": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_float,
                                            C.c_void_p]),
    "oxf_layer_norm_backward": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_float,
                                          C.c_void_p]),
    "oxf_matrix_rms_norm_backward": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_float,
                                               C.c_void_p]),
    "oxf_matrix_binary_assign_by_rows": (C.c_int, [Slice, CSlice, C.c_size_t, C.c_int,
                                                   C.c_void_p]),
    "oxf_matrix_causal_mask": (C.c_int, [Slice, C.c_size_t, C.c_void_p]),
    "oxf_matrix_transpose": (C.c_int, [CSlice, Slice, C.c_size_t, C.c_size_t, C.c_void_p]),
    "oxf_gemm_desc_init": (None, [C.POINTER(GemmDesc), C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "oxf_gemm_workspace_size": (C.c_size_t, [C.POINTER(GemmDesc)]),
    "oxf_gemm": (C.c_int, [C.POINTER(GemmDesc), C.c_void_p]),
    "oxf_gemm_tf32x3_noalloc": (C.c_int, [C.POINTER(GemmDesc), C.c_void_p]),
    "oxf_gemm_plan": (C.c_int, [C.POINTER(GemmDesc), C.c_int, C.POINTER(GemmPlanInfo)]),
    "oxf_attention_stats_floats": (C.c_size_t, [C.c_int, C.c_int]),
    "oxf_attention_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int,
                                        C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p]),
    "oxf_attention_heads_forward": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                              C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                              C.c_int, C.c_int, C.c_void_p]),
    "oxf_matrix_multiply": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_size_t, C.c_size_t,
                                      C.c_void_p]),
    "oxf_matrix_multiply_fp32": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_size_t,
                                          C.c_size_t, C.c_void_p]),
    "oxf_matrix_multiply_refalgo": (C.c_int, [CSlice, CSlice, Slice, C.c_size_t, C.c_size_t,
                                              C.c_size_t, C.c_void_p]),
    "oxf_exchange_sgd": (C.c_int, [C.POINTER(ExchangeDesc), C.c_size_t, C.c_size_t, C.c_float,
                                   C.c_void_p]),
    "oxf_ipc_export": (C.c_int, [C.c_void_p, C.POINTER(IpcHandle)]),
    "oxf_ipc_open": (C.c_int, [C.POINTER(IpcHandle), C.POINTER(C.c_void_p)]),
    "oxf_ipc_close": (C.c_int, [C.POINTER(IpcHandle), C.c_void_p]),
}


def lib() -> C.CDLL:
    """Loads liboxf.so once (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: run `python oxide-forge_b200/build.py` "
                "(there is no CPU fallback)")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGS.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        from . import _host_sigs
        _host_sigs.bind(h)
        _lib = h
    return _lib


def check(status: int) -> None:
    if status != OK:
        msg = lib().oxf_last_error_string().decode(errors="replace")
        raise OxfError(status, msg)


def exported_symbols() -> list[str]:
    return sorted(_SIGS)
