"""ctypes signatures of the host-layer C ABI (include/oxf_host.h)."""
from __future__ import annotations

import ctypes as C

MAX_LAYERS = 16


class LayerSpec(C.Structure):
    _fields_ = [("in_", C.c_int), ("out", C.c_int), ("act", C.c_int), ("bias", C.c_int)]


class MlpSpec(C.Structure):
    _fields_ = [("n_layers", C.c_int), ("layers", LayerSpec * MAX_LAYERS),
                ("res_start", C.c_int), ("res_end", C.c_int)]


class TransformerSpec(C.Structure):
    _fields_ = [("seq", C.c_int), ("hidden", C.c_int), ("norm", C.c_int), ("q", LayerSpec),
                ("k", LayerSpec), ("v", LayerSpec), ("ffn", MlpSpec), ("out", LayerSpec)]


_h = C.c_void_p
_fp = C.c_void_p
_sz = C.c_size_t
SIGS: dict = {
    "oxf_transformer_create": (C.c_int, [C.POINTER(TransformerSpec), C.c_int, C.c_void_p,
                                         C.POINTER(C.c_void_p)]),
    "oxf_transformer_destroy": (C.c_int, [_h]),
    "oxf_transformer_param_count": (_sz, [_h]),
    "oxf_transformer_params": (C.c_void_p, [_h]),
    "oxf_transformer_grads": (C.c_void_p, [_h]),
    "oxf_transformer_stream": (C.c_void_p, [_h]),
    "oxf_transformer_set_params_host": (C.c_int, [_h, _fp]),
    "oxf_transformer_get_params_host": (C.c_int, [_h, _fp]),
    "oxf_transformer_forward": (C.c_int, [_h, _fp, C.c_int, C.c_int, _fp]),
    "oxf_transformer_train_forward": (C.c_int, [_h, _fp, C.c_int]),
    "oxf_transformer_set_target": (C.c_int, [_h, _fp]),
    "oxf_transformer_set_output_gradient": (C.c_int, [_h, _fp]),
    "oxf_transformer_backward_stage": (C.c_int, [_h, C.c_int]),
    "oxf_transformer_bucket": (C.c_int, [_h, C.c_int, C.POINTER(_sz), C.POINTER(_sz)]),
    "oxf_transformer_zero_grads": (C.c_int, [_h]),
    "oxf_transformer_sgd": (C.c_int, [_h, C.c_float]),
    "oxf_transformer_set_heads": (C.c_int, [_h, C.c_int]),
    "oxf_transformer_heads": (C.c_int, [_h]),
    "oxf_transformer_output": (C.c_int, [_h, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p),
                                         C.POINTER(C.c_void_p)]),
    "oxf_transformer_train_step_host": (C.c_int, [_h, _fp, _fp, C.c_int, C.c_float,
                                                  C.POINTER(C.c_float)]),
    "oxf_transformer_set_timing": (C.c_int, [_h, C.c_int]),
    "oxf_transformer_read_timing": (C.c_int, [_h, C.POINTER(C.c_double), C.POINTER(C.c_double),
                                              C.POINTER(C.c_int)]),
    "oxf_mlp_create": (C.c_int, [C.POINTER(MlpSpec), _sz, C.c_void_p, C.POINTER(C.c_void_p)]),
    "oxf_mlp_destroy": (C.c_int, [_h]),
    "oxf_mlp_param_count": (_sz, [_h]),
    "oxf_mlp_params": (C.c_void_p, [_h]),
    "oxf_mlp_grads": (C.c_void_p, [_h]),
    "oxf_mlp_forward": (C.c_int, [_h, _fp, _fp, _sz]),
    "oxf_mlp_backward": (C.c_int, [_h, _fp, _fp, _sz]),
    "oxf_mlp_zero_grads": (C.c_int, [_h]),
    "oxf_mlp_sgd": (C.c_int, [_h, C.c_float]),
    "oxf_runtime_create": (C.c_int, [C.c_int, C.c_void_p, C.POINTER(C.c_void_p)]),
    "oxf_runtime_destroy": (C.c_int, [_h]),
    "oxf_runtime_stream": (C.c_void_p, [_h]),
    "oxf_runtime_sync": (C.c_int, [_h]),
    "oxf_runtime_reserve_buffers": (C.c_int, [_h, _sz, _sz]),
    "oxf_runtime_pooled_buffers": (C.c_int, [_h, C.POINTER(_sz)]),
    "oxf_linear_create": (C.c_int, [_h, C.POINTER(LayerSpec), _fp, _fp, C.POINTER(C.c_void_p)]),
    "oxf_linear_destroy": (C.c_int, [_h]),
    "oxf_linear_params": (C.c_int, [_h, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "oxf_linear_forward": (C.c_int, [_h, _fp, _sz, _fp, _fp, _fp, C.c_void_p]),
    "oxf_linear_backward": (C.c_int, [_h, _fp, _fp, _fp, _sz, _fp, _fp, C.c_void_p]),
    "oxf_linear_learn": (C.c_int, [_h, _fp, _fp, _fp, _sz, C.c_float, C.c_void_p]),
    "oxf_linear_input_gradient": (C.c_int, [_h, _fp, _sz, _fp, C.c_void_p]),
    "oxf_checkpoint_write_linear": (C.c_int, [C.c_char_p, C.POINTER(LayerSpec), _fp, _sz]),
    "oxf_checkpoint_write_mlp": (C.c_int, [C.c_char_p, C.POINTER(MlpSpec), _fp, _sz]),
    "oxf_checkpoint_write_transformer": (C.c_int, [C.c_char_p, C.POINTER(TransformerSpec), _fp,
                                                   _sz]),
    "oxf_checkpoint_read_linear": (C.c_int, [C.c_char_p, C.POINTER(LayerSpec), _fp, _sz,
                                             C.POINTER(_sz)]),
    "oxf_checkpoint_read_mlp": (C.c_int, [C.c_char_p, C.POINTER(MlpSpec), _fp, _sz,
                                          C.POINTER(_sz)]),
    "oxf_checkpoint_read_transformer": (C.c_int, [C.c_char_p, C.POINTER(TransformerSpec), _fp,
                                                  _sz, C.POINTER(_sz)]),
    "oxf_transformer_dump": (C.c_int, [_h, C.c_char_p]),
    "oxf_transformer_load": (C.c_int, [C.c_char_p, C.c_int, C.c_void_p,
                                       C.POINTER(C.c_void_p)]),
    "oxf_mlp_dump": (C.c_int, [_h, C.c_char_p]),
    "oxf_mlp_load": (C.c_int, [C.c_char_p, _sz, C.c_void_p, C.POINTER(C.c_void_p)]),
    "oxf_exchange_create": (C.c_int, [C.c_int, C.c_int, _fp, _fp, _sz, C.POINTER(C.c_void_p)]),
    "oxf_exchange_handles": (C.c_int, [_h, C.c_void_p]),
    "oxf_exchange_connect": (C.c_int, [_h, C.c_void_p]),
    "oxf_exchange_step": (C.c_int, [_h, _sz, _sz, C.c_float, C.c_int, C.c_void_p]),
    "oxf_exchange_set_timeout": (C.c_int, [_h, C.c_uint32]),
    "oxf_exchange_destroy": (C.c_int, [_h]),
}


def bind(h: C.CDLL) -> None:
    for name, (res, args) in SIGS.items():
        f = getattr(h, name)
        f.restype = res
        f.argtypes = args
