"""Python driver of the host executors (include/oxf_host.h).

`Transformer` and `Mlp` wrap the C++ engines; their parameter and gradient
arenas are exposed as zero-copy torch views (via __cuda_array_interface__)
in checkpoint cursor order, so a data-parallel driver can all-reduce the
gradient buckets with torch.distributed. All compute runs in liboxf.so on
the engine's stream (by default torch's current stream).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib, kernels
from ._host_sigs import LayerSpec, MlpSpec, TransformerSpec
from ._lib import check, lib


class _DeviceArray:
    """Borrowed device memory exposed through __cuda_array_interface__."""

    def __init__(self, ptr: int, shape, owner):
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape), "typestr": "<f4",
            "data": (int(ptr), False), "version": 3, "strides": None}
        self._owner = owner


def device_view(ptr: int, shape, owner=None) -> torch.Tensor:
    if int(np.prod(shape)) == 0:
        return torch.empty(shape, device="cuda")
    return torch.as_tensor(_DeviceArray(ptr, shape, owner), device="cuda")


@dataclass
class Layer:
    """One Linear (linear.rs:72-86): weights [in, out], optional bias."""
    in_: int
    out: int
    act: int = _lib.ACT_IDENTITY
    bias: bool = False

    def spec(self) -> LayerSpec:
        return LayerSpec(self.in_, self.out, self.act, int(self.bias))

    def shapes(self):
        return [(self.in_, self.out)] + ([(self.out,)] if self.bias else [])

    def count(self) -> int:
        return self.in_ * self.out + (self.out if self.bias else 0)


@dataclass
class MlpConfig:
    layers: list
    res_range: tuple | None = None

    def spec(self) -> MlpSpec:
        s = MlpSpec()
        s.n_layers = len(self.layers)
        for i, l in enumerate(self.layers):
            s.layers[i] = l.spec()
        s.res_start, s.res_end = self.res_range if self.res_range else (-1, -1)
        return s

    def shapes(self):
        return [sh for l in self.layers for sh in l.shapes()]


@dataclass
class TransformerConfig:
    seq: int
    hidden: int
    ffn: MlpConfig
    out: int
    norm: int = _lib.NORM_LAYER
    qkv_dim: int | None = None
    qkv_act: int = _lib.ACT_IDENTITY
    out_act: int = _lib.ACT_IDENTITY
    bias: bool = False

    def layers(self):
        d = self.qkv_dim or self.hidden
        q = Layer(self.hidden, d, self.qkv_act, self.bias)
        k = Layer(self.hidden, d, self.qkv_act, self.bias)
        v = Layer(self.hidden, self.hidden, self.qkv_act, self.bias)
        o = Layer(self.hidden, self.out, self.out_act, self.bias)
        return q, k, v, o

    def spec(self) -> TransformerSpec:
        q, k, v, o = self.layers()
        return TransformerSpec(self.seq, self.hidden, self.norm, q.spec(), k.spec(), v.spec(),
                               self.ffn.spec(), o.spec())

    def shapes(self):
        """Cursor order (inference.rs:52-66): q, k, v, position, ffn, out."""
        q, k, v, o = self.layers()
        return (q.shapes() + k.shapes() + v.shapes() + [(self.seq, self.hidden)] +
                self.ffn.shapes() + o.shapes())

    def param_count(self) -> int:
        return int(sum(np.prod(s) for s in self.shapes()))


def transformer_config(seq, hidden, ffn, out=None, norm=_lib.NORM_LAYER, bias=False,
                       ffn_act=_lib.ACT_GELU) -> TransformerConfig:
    """The configurations' transformer shape: FFN hidden -> ffn (GELU) -> hidden."""
    mlp = MlpConfig([Layer(hidden, ffn, ffn_act, bias), Layer(ffn, hidden, _lib.ACT_IDENTITY, bias)])
    return TransformerConfig(seq, hidden, mlp, out or hidden, norm, bias=bias)


def init_transformer_params(cfg: TransformerConfig, seed: int = 0,
                            pos_std: float = 0.02) -> np.ndarray:
    """Xavier-uniform weights (bound sqrt(6/(fan_in+fan_out))), position
    N(0, pos_std), biases 0.01*N(0,1); from a seeded host RNG."""
    rng = np.random.default_rng(seed)
    out = []
    for i, sh in enumerate(cfg.shapes()):
        if len(sh) == 1:
            out.append(0.01 * rng.standard_normal(sh))
        elif sh == (cfg.seq, cfg.hidden) and i == _position_index(cfg):
            out.append(pos_std * rng.standard_normal(sh))
        else:
            b = np.sqrt(6.0 / (sh[0] + sh[1]))
            out.append(rng.uniform(-b, b, sh))
    return np.concatenate([a.astype(np.float32).ravel() for a in out])


def _position_index(cfg: TransformerConfig) -> int:
    q, k, v, _ = cfg.layers()
    return len(q.shapes()) + len(k.shapes()) + len(v.shapes())


def split_params(cfg, flat: np.ndarray) -> list:
    """Flat cursor-order arena -> list of arrays with cfg.shapes()."""
    res, off = [], 0
    for sh in cfg.shapes():
        n = int(np.prod(sh))
        res.append(np.asarray(flat[off:off + n]).reshape(sh))
        off += n
    return res


class Transformer:
    """Batched single-block Post-Norm transformer (inference + training)."""

    def __init__(self, cfg: TransformerConfig, max_batch: int = 1, stream=None, _handle=None,
                 heads: int = 1):
        self.cfg = cfg
        self.max_batch = max_batch
        if stream is None:
            stream = torch.cuda.current_stream()
        self._stream = stream
        h = _handle
        if h is None:
            h = C.c_void_p()
            spec = cfg.spec()
            check(lib().oxf_transformer_create(C.byref(spec), max_batch,
                                               C.c_void_p(stream.cuda_stream), C.byref(h)))
        self._h = h
        self.n = int(lib().oxf_transformer_param_count(h))
        assert self.n == cfg.param_count(), (self.n, cfg.param_count())
        if heads != 1:
            self.set_heads(heads)
        self.params = device_view(lib().oxf_transformer_params(h), (self.n,), self)
        self.grads = device_view(lib().oxf_transformer_grads(h), (self.n,), self)

    # ---------------------------------------------------------------- params
    def set_params(self, flat) -> None:
        flat = np.ascontiguousarray(flat, np.float32)
        assert flat.size == self.n
        check(lib().oxf_transformer_set_params_host(self._h, flat.ctypes.data))

    def get_params(self) -> np.ndarray:
        out = np.empty(self.n, np.float32)
        check(lib().oxf_transformer_get_params_host(self._h, out.ctypes.data))
        return out

    def bucket(self, stage: int) -> tuple[int, int]:
        off, cnt = C.c_size_t(), C.c_size_t()
        check(lib().oxf_transformer_bucket(self._h, stage, C.byref(off), C.byref(cnt)))
        return off.value, cnt.value

    # ---------------------------------------------------------------- compute
    def _views(self, batch):
        y, loss, dx = C.c_void_p(), C.c_void_p(), C.c_void_p()
        check(lib().oxf_transformer_output(self._h, C.byref(y), C.byref(loss), C.byref(dx)))
        rows = batch * self.cfg.seq
        return (device_view(y.value, (rows, self.cfg.out), self),
                device_view(loss.value, (rows,), self),
                device_view(dx.value, (rows, self.cfg.hidden), self))

    def forward(self, x: torch.Tensor, causal: bool = False) -> torch.Tensor:
        batch = x.numel() // (self.cfg.seq * self.cfg.hidden)
        check(lib().oxf_transformer_forward(self._h, x.data_ptr(), batch, int(causal), None))
        return self._views(batch)[0]

    def train_forward(self, x: torch.Tensor) -> torch.Tensor:
        self._batch = x.numel() // (self.cfg.seq * self.cfg.hidden)
        check(lib().oxf_transformer_train_forward(self._h, x.data_ptr(), self._batch))
        return self._views(self._batch)[0]

    def set_target(self, target: torch.Tensor) -> torch.Tensor:
        check(lib().oxf_transformer_set_target(self._h, target.data_ptr()))
        return self._views(self._batch)[1]

    def scaled_loss_sum(self, scale: float) -> torch.Tensor:
        """scale * (sum of the row losses of the last set_target), as a fresh
        one-element device tensor: one library launch (oxf_slice_map_sum),
        no PyTorch kernel, on the current stream."""
        out = torch.empty(1, device=self.params.device)
        kernels.map_sum(self._views(self._batch)[1], _lib.UNARY_SCALE, float(scale), out)
        return out

    def set_output_gradient(self, dy: torch.Tensor) -> None:
        check(lib().oxf_transformer_set_output_gradient(self._h, dy.data_ptr()))

    def backward_stage(self, stage: int) -> None:
        check(lib().oxf_transformer_backward_stage(self._h, stage))

    def backward(self) -> torch.Tensor:
        for s in range(3):
            self.backward_stage(s)
        return self._views(self._batch)[2]

    def zero_grads(self) -> None:
        check(lib().oxf_transformer_zero_grads(self._h))

    def sgd(self, lr: float) -> None:
        check(lib().oxf_transformer_sgd(self._h, float(lr)))

    def set_heads(self, heads: int) -> None:
        """Multi-head attention (oxf_transformer_set_heads); 1 is the
        reference's single-head attention."""
        check(lib().oxf_transformer_set_heads(self._h, int(heads)))

    @property
    def heads(self) -> int:
        return int(lib().oxf_transformer_heads(self._h))

    def train_step_host(self, x: np.ndarray, target: np.ndarray, lr: float) -> float:
        """The e2e API: host arrays in, one SGD step, mean row loss out."""
        x = np.ascontiguousarray(x, np.float32)
        target = np.ascontiguousarray(target, np.float32)
        batch = x.size // (self.cfg.seq * self.cfg.hidden)
        loss = C.c_float()
        check(lib().oxf_transformer_train_step_host(self._h, x.ctypes.data, target.ctypes.data,
                                                    batch, float(lr), C.byref(loss)))
        return loss.value

    def set_timing(self, on: bool) -> None:
        check(lib().oxf_transformer_set_timing(self._h, int(on)))

    def read_timing(self) -> tuple[float, float, int]:
        """(GEMM device ms, GEMM flops, GEMM launches) since the last read."""
        ms, fl, n = C.c_double(), C.c_double(), C.c_int()
        check(lib().oxf_transformer_read_timing(self._h, C.byref(ms), C.byref(fl), C.byref(n)))
        return ms.value, fl.value, n.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().oxf_transformer_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class TransformerStack:
    """A stack of L Post-Norm transformer blocks, block i's output feeding
    block i+1 (every block but the last maps hidden to hidden). The reference
    executor takes exactly one block (model.rs:448-449, although its
    checkpoint metadata carries a block count); this is the multi-block
    executor built from single-block engines. Forward chains the blocks;
    backward sets the last block's loss gradient, then hands each block's
    input gradient to the block below as its output gradient
    (oxf_transformer_set_output_gradient). Gradients accumulate per block,
    and sgd applies each block's step. Every kernel is the library's; only
    the loop over blocks is here."""

    def __init__(self, cfgs, max_batch: int = 1, stream=None, heads: int = 1):
        cfgs = list(cfgs)
        if not cfgs:
            raise ValueError("a stack needs at least one block")
        for lo, hi in zip(cfgs, cfgs[1:]):
            if lo.out != hi.hidden or lo.seq != hi.seq:
                raise ValueError("block output width must equal the next block's hidden")
        self.blocks = [Transformer(c, max_batch, stream, heads=heads) for c in cfgs]

    def __len__(self) -> int:
        return len(self.blocks)

    def set_params(self, flats) -> None:
        for b, f in zip(self.blocks, flats):
            b.set_params(f)

    def get_params(self):
        return [b.get_params() for b in self.blocks]

    def forward(self, x: torch.Tensor, causal: bool = False) -> torch.Tensor:
        for b in self.blocks:
            x = b.forward(x, causal)
        return x

    def train_forward(self, x: torch.Tensor) -> torch.Tensor:
        for b in self.blocks:
            x = b.train_forward(x)
        return x

    def set_target(self, target: torch.Tensor) -> torch.Tensor:
        """Row losses of the last block's output against target."""
        return self.blocks[-1].set_target(target)

    def backward(self) -> torch.Tensor:
        """dL/dx of the stack's input; parameter gradients accumulate."""
        dx = self.blocks[-1].backward()
        for b in reversed(self.blocks[:-1]):
            b.set_output_gradient(dx)
            dx = b.backward()
        return dx

    def zero_grads(self) -> None:
        for b in self.blocks:
            b.zero_grads()

    def sgd(self, lr: float) -> None:
        for b in self.blocks:
            b.sgd(lr)

    def close(self) -> None:
        for b in self.blocks:
            b.close()


class Mlp:
    """Batched MlpExecutor (forward, backward with deferred SGD)."""

    def __init__(self, cfg: MlpConfig, max_rows: int, stream=None, _handle=None):
        self.cfg = cfg
        if stream is None:
            stream = torch.cuda.current_stream()
        h = _handle
        if h is None:
            h = C.c_void_p()
            spec = cfg.spec()
            check(lib().oxf_mlp_create(C.byref(spec), max_rows, C.c_void_p(stream.cuda_stream),
                                       C.byref(h)))
        self._h = h
        self.n = int(lib().oxf_mlp_param_count(h))
        self.params = device_view(lib().oxf_mlp_params(h), (self.n,), self)
        self.grads = device_view(lib().oxf_mlp_grads(h), (self.n,), self)

    def forward(self, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
        check(lib().oxf_mlp_forward(self._h, x.data_ptr(), y.data_ptr(), x.shape[0]))
        return y

    def backward(self, dy: torch.Tensor, dx: torch.Tensor | None) -> None:
        check(lib().oxf_mlp_backward(self._h, dy.data_ptr(),
                                     dx.data_ptr() if dx is not None else None, dy.shape[0]))

    def zero_grads(self) -> None:
        check(lib().oxf_mlp_zero_grads(self._h))

    def sgd(self, lr: float) -> None:
        check(lib().oxf_mlp_sgd(self._h, float(lr)))

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().oxf_mlp_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Runtime:
    """CudaRuntime (src/cuda/runtime.rs:24-212) through include/oxf_host.h:
    a device, its primary stream and an exact-size buffer pool. By default it
    borrows torch's current stream as its primary stream, so tensors made by
    torch and the runtime's work are ordered on one stream."""

    def __init__(self, device: int | None = None, stream=None):
        if device is None:
            device = torch.cuda.current_device()
        if stream is None:
            stream = torch.cuda.current_stream()
        h = C.c_void_p()
        check(lib().oxf_runtime_create(int(device), C.c_void_p(stream.cuda_stream), C.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    def sync(self) -> None:
        check(lib().oxf_runtime_sync(self._h))

    def reserve_buffers(self, length: int, count: int) -> None:
        check(lib().oxf_runtime_reserve_buffers(self._h, int(length), int(count)))

    def pooled_buffers(self) -> int:
        n = C.c_size_t()
        check(lib().oxf_runtime_pooled_buffers(self._h, C.byref(n)))
        return n.value

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().oxf_runtime_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _sp(stream):
    return None if stream is None else C.c_void_p(stream.cuda_stream)


def _dp(t):
    return None if t is None else t.data_ptr()


class Linear:
    """Linear (src/net/linear.rs:72-533) through include/oxf_host.h: weights
    [in, out] and an optional bias held in the runtime's pool, copied from
    host arrays. Methods take float32 CUDA tensors of rows x in / rows x out
    and run on the runtime's primary stream unless `stream` is given."""

    def __init__(self, rt: Runtime, weights, bias=None, act: int = _lib.ACT_IDENTITY):
        w = np.ascontiguousarray(weights, np.float32)
        b = None if bias is None else np.ascontiguousarray(bias, np.float32)
        self.in_, self.out = w.shape
        self.act = act
        spec = LayerSpec(self.in_, self.out, int(act), int(b is not None))
        h = C.c_void_p()
        check(lib().oxf_linear_create(rt.handle, C.byref(spec), w.ctypes.data,
                                      None if b is None else b.ctypes.data, C.byref(h)))
        self._h = h
        self._rt = rt
        wp, bp = C.c_void_p(), C.c_void_p()
        check(lib().oxf_linear_params(h, C.byref(wp), C.byref(bp)))
        self.weights = device_view(wp.value, (self.in_, self.out), self)
        self.bias = device_view(bp.value, (self.out,), self) if bp.value else None

    def forward(self, x, residual=None, y=None, pre_activation=None, stream=None):
        """Linear::forward: y = act(x·W + b + residual); pre_activation, if
        given, receives x·W + b + residual."""
        rows = x.shape[0]
        if y is None:
            y = torch.empty((rows, self.out), device=x.device)
        check(lib().oxf_linear_forward(self._h, _dp(x), rows, _dp(residual), _dp(y),
                                       _dp(pre_activation), _sp(stream)))
        return y

    def backward(self, pre_activation, output_gradient, residual_gradient=None, stream=None):
        """Linear::backward / backward_with_res: (G, bias gradient or None)."""
        rows = output_gradient.shape[0]
        g = torch.empty_like(output_gradient)
        bg = torch.empty(self.out, device=g.device) if self.bias is not None else None
        check(lib().oxf_linear_backward(self._h, _dp(pre_activation), _dp(output_gradient),
                                        _dp(residual_gradient), rows, _dp(g), _dp(bg),
                                        _sp(stream)))
        return g, bg

    def learn(self, x, gradient, bias_gradient, lr: float, stream=None) -> None:
        """Linear::learn: W -= lr·xᵀ·G, b -= lr·bias_gradient."""
        check(lib().oxf_linear_learn(self._h, _dp(x), _dp(gradient), _dp(bias_gradient),
                                     x.shape[0], float(lr), _sp(stream)))

    def input_gradient(self, gradient, dx=None, stream=None):
        """Linear::input_gradient: G·Wᵀ."""
        rows = gradient.shape[0]
        if dx is None:
            dx = torch.empty((rows, self.in_), device=gradient.device)
        check(lib().oxf_linear_input_gradient(self._h, _dp(gradient), rows, _dp(dx),
                                              _sp(stream)))
        return dx

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().oxf_linear_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
