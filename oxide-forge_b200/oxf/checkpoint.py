"""Checkpoint format version 1 of the reference (src/net/checkpoint/
model.rs, io.rs): `<name>.toml` metadata plus `<name>.bin` little-endian f32
parameters in cursor order. Reading and writing run in liboxf.so
(host/checkpoint.cpp); these are thin wrappers.

Host forms take and return numpy parameter arrays and need no GPU:
    dump_linear / load_linear, dump_mlp / load_mlp,
    dump_transformer_params / load_transformer_params.
Engine forms move an engine's device parameter arena:
    dump_transformer(model, path) / load_transformer(path, max_batch),
    dump_mlp_engine(model, path) / load_mlp_engine(path, max_rows).
Errors raise oxf._lib.OxfError with the reference's validation messages.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from ._host_sigs import LayerSpec, MlpSpec, TransformerSpec
from ._lib import check, lib


def _p(path) -> bytes:
    return os.fsencode(os.fspath(path))


def _layer(spec: LayerSpec):
    from .models import Layer
    return Layer(spec.in_, spec.out, spec.act, bool(spec.bias))


def _mlp_config(spec: MlpSpec):
    from .models import MlpConfig
    layers = [_layer(spec.layers[i]) for i in range(spec.n_layers)]
    res = (spec.res_start, spec.res_end) if spec.res_start >= 0 else None
    return MlpConfig(layers, res)


def _transformer_config(spec: TransformerSpec):
    """TransformerConfig of a checkpoint's spec. The Python config describes
    Q/K/V with one activation and bias flag and K = Q width; other specs
    load through the C ABI but have no Python config."""
    from .models import TransformerConfig
    q, k, v, o = spec.q, spec.k, spec.v, spec.out
    uniform = (q.act == k.act == v.act and q.bias == k.bias == v.bias == o.bias and
               q.out == k.out and v.out == spec.hidden)
    if not uniform:
        raise NotImplementedError("checkpoint Q/K/V layers differ in activation or bias; "
                                  "use the C ABI (oxf_checkpoint_read_transformer)")
    return TransformerConfig(spec.seq, spec.hidden, _mlp_config(spec.ffn), o.out, spec.norm,
                             qkv_dim=None if q.out == spec.hidden else q.out, qkv_act=q.act,
                             out_act=o.act, bias=bool(q.bias))


def _params(flat) -> np.ndarray:
    return np.ascontiguousarray(flat, np.float32).ravel()


def _read(fn, path, spec):
    n = C.c_size_t()
    check(fn(_p(path), C.byref(spec), None, 0, C.byref(n)))
    out = np.empty(n.value, np.float32)
    check(fn(_p(path), None, out.ctypes.data, out.size, C.byref(n)))
    return out


# ---------------------------------------------------------------- host forms
def dump_linear(path, layer, params) -> None:
    """dump_linear (model.rs:53-71): layer is a models.Layer."""
    flat = _params(params)
    spec = layer.spec()
    check(lib().oxf_checkpoint_write_linear(_p(path), C.byref(spec), flat.ctypes.data, flat.size))


def load_linear(path):
    """load_linear (model.rs:73-76) -> (models.Layer, parameters)."""
    spec = LayerSpec()
    flat = _read(lib().oxf_checkpoint_read_linear, path, spec)
    return _layer(spec), flat


def dump_mlp(path, cfg, params) -> None:
    """dump_mlp (model.rs:78-88): cfg is a models.MlpConfig."""
    flat = _params(params)
    spec = cfg.spec()
    check(lib().oxf_checkpoint_write_mlp(_p(path), C.byref(spec), flat.ctypes.data, flat.size))


def load_mlp(path):
    """load_mlp (model.rs:90-94) -> (models.MlpConfig, parameters)."""
    spec = MlpSpec()
    flat = _read(lib().oxf_checkpoint_read_mlp, path, spec)
    return _mlp_config(spec), flat


def dump_transformer_params(path, cfg, params) -> None:
    """dump_transformer (model.rs:138-148) of a models.TransformerConfig
    and its cursor-order parameters."""
    flat = _params(params)
    spec = cfg.spec()
    check(lib().oxf_checkpoint_write_transformer(_p(path), C.byref(spec), flat.ctypes.data,
                                                 flat.size))


def load_transformer_params(path):
    """load_transformer's metadata and data (model.rs:150-172) ->
    (models.TransformerConfig, parameters)."""
    spec = TransformerSpec()
    flat = _read(lib().oxf_checkpoint_read_transformer, path, spec)
    return _transformer_config(spec), flat


# ---------------------------------------------------------------- engine forms
def dump_transformer(model, path) -> None:
    """dump_transformer / dump_training_transformer of a models.Transformer."""
    check(lib().oxf_transformer_dump(model._h, _p(path)))


def load_transformer(path, max_batch: int = 1, stream=None):
    """load_transformer / load_training_transformer -> models.Transformer
    holding the checkpoint's parameters."""
    import torch
    from .models import Transformer
    spec = TransformerSpec()
    n = C.c_size_t()
    check(lib().oxf_checkpoint_read_transformer(_p(path), C.byref(spec), None, 0, C.byref(n)))
    cfg = _transformer_config(spec)
    if stream is None:
        stream = torch.cuda.current_stream()
    h = C.c_void_p()
    check(lib().oxf_transformer_load(_p(path), max_batch, C.c_void_p(stream.cuda_stream),
                                     C.byref(h)))
    return Transformer(cfg, max_batch, stream, _handle=h)


def dump_mlp_engine(model, path) -> None:
    """dump_mlp / dump_training_mlp of a models.Mlp."""
    check(lib().oxf_mlp_dump(model._h, _p(path)))


def load_mlp_engine(path, max_rows: int, stream=None):
    """load_mlp / load_training_mlp -> models.Mlp holding the checkpoint's
    parameters."""
    import torch
    from .models import Mlp
    spec = MlpSpec()
    n = C.c_size_t()
    check(lib().oxf_checkpoint_read_mlp(_p(path), C.byref(spec), None, 0, C.byref(n)))
    if stream is None:
        stream = torch.cuda.current_stream()
    h = C.c_void_p()
    check(lib().oxf_mlp_load(_p(path), max_rows, C.c_void_p(stream.cuda_stream), C.byref(h)))
    return Mlp(_mlp_config(spec), max_rows, stream, _handle=h)
