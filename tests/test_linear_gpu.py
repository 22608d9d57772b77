"""Linear (src/net/linear.rs:72-533) and CudaRuntime through the host C ABI
(oxf_runtime_* / oxf_linear_* in include/oxf_host.h), against the oracle.

Tolerances: TF32 products 5e-3 of max|want| (the oracle rounds operands
RNA as the reference does, gemm.rs:286-347); elementwise steps (the
activation-gradient product, column sums, the bias update) 1e-5.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
RNA = O.GEMM_TF32_RNA
TF32_TOL = 5e-3
TOL = 1e-5
F32 = np.float32


@pytest.fixture(scope="module")
def M():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import _lib, kernels, models
    yield _lib, models
    assert kernels.device_error() == 0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, F32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy().copy()


def test_config1_through_linear_forward(M):
    """Config 1 through Linear::forward (no bias, Identity): X [256,128]
    U(-1,1) from seed 0, W [128,64] U(-1/sqrt(128), 1/sqrt(128)); equal to
    the oracle with RNA operand rounding up to f32 summation order."""
    L, models = M
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (256, 128)).astype(F32)
    b = 1 / np.sqrt(128)
    w = rng.uniform(-b, b, (128, 64)).astype(F32)
    rt = models.Runtime()
    lin = models.Linear(rt, w)
    y = host(lin.forward(dev(x)))
    want, _ = O.linear_forward(O.LinearParams(w), x, rounding=RNA)
    assert np.abs(y - want).max() <= 1e-5 * np.abs(want).max()
    lin.close()
    rt.close()


@pytest.mark.parametrize("act", [0, 1, 2, 3])
def test_forward_backward_learn_input_gradient(M, act):
    """Every Linear method on a biased layer with a residual, against the
    oracle's restatement of each step (linear.rs:185-230, 246-275,
    373-391, 431-434)."""
    L, models = M
    rows, n_in, n_out, lr = 300, 96, 160, 0.05
    rng = np.random.default_rng(10 + act)
    x = rng.standard_normal((rows, n_in)).astype(F32)
    w = rng.uniform(-0.2, 0.2, (n_in, n_out)).astype(F32)
    bias = (0.1 * rng.standard_normal(n_out)).astype(F32)
    res = rng.standard_normal((rows, n_out)).astype(F32)
    dy = rng.standard_normal((rows, n_out)).astype(F32)
    dres = rng.standard_normal((rows, n_out)).astype(F32)
    rt = models.Runtime()
    lin = models.Linear(rt, w, bias, act)
    xd = dev(x)
    pre = torch.empty((rows, n_out), device="cuda")
    y = lin.forward(xd, residual=dev(res), pre_activation=pre)
    y_ref, pre_ref = O.linear_forward(O.LinearParams(w, bias, act), x, res, rounding=RNA)
    assert rel_err(host(y), y_ref) < TF32_TOL
    assert rel_err(host(pre), pre_ref) < TF32_TOL

    # backward from the layer's own pre-activation: elementwise steps exact
    z = host(pre)
    g, bg = lin.backward(pre if act else None, dev(dy))
    g_ref = dy * O.act_derivative(act, z) if act else dy
    assert rel_err(host(g), g_ref) < TOL
    assert rel_err(host(bg), O.sum_cols(g_ref)) < TOL
    if act:  # backward_with_res: (dY + dR) ⊙ act'(Z)
        g2, bg2 = lin.backward(pre, dev(dy), dev(dres))
        g2_ref = (dy + dres) * O.act_derivative(act, z)
        assert rel_err(host(g2), g2_ref) < TOL
        assert rel_err(host(bg2), O.sum_cols(g2_ref)) < TOL

    gh = host(g)
    dx = host(lin.input_gradient(g))
    assert rel_err(dx, O.gemm(gh, w, b_trans=True, rounding=RNA)) < TF32_TOL
    lin.learn(xd, g, bg, lr)
    dw = w - host(lin.weights)
    assert rel_err(dw, lr * O.gemm(x, gh, a_trans=True, rounding=RNA)) < TF32_TOL
    assert rel_err(bias - host(lin.bias), lr * host(bg)) < 1e-4
    lin.close()
    rt.close()


def test_one_layer_step_matches_oracle_mlp_step(M):
    """forward -> backward -> input_gradient -> learn on one biased GELU
    layer equals the oracle's one-layer MlpExecutor step (mlp.rs:121-168:
    dX with the old weights, then the immediate SGD)."""
    L, models = M
    rows, n_in, n_out, lr = 256, 64, 128, 0.05
    rng = np.random.default_rng(3)
    x = rng.standard_normal((rows, n_in)).astype(F32)
    w = rng.uniform(-0.25, 0.25, (n_in, n_out)).astype(F32)
    bias = (0.1 * rng.standard_normal(n_out)).astype(F32)
    dy = rng.standard_normal((rows, n_out)).astype(F32)
    ref = O.MlpParams([O.LinearParams(w, bias, O.GELU)])
    _, dx_ref = O.mlp_train_step(ref, x, dy, lr, rounding=RNA)
    rt = models.Runtime()
    lin = models.Linear(rt, w, bias, L.ACT_GELU)
    xd = dev(x)
    pre = torch.empty((rows, n_out), device="cuda")
    lin.forward(xd, pre_activation=pre)
    g, bg = lin.backward(pre, dev(dy))
    dx = lin.input_gradient(g)
    lin.learn(xd, g, bg, lr)
    assert rel_err(host(dx), dx_ref) < TF32_TOL
    assert rel_err(w - host(lin.weights), w - ref.layers[0].w) < TF32_TOL
    assert rel_err(bias - host(lin.bias), bias - ref.layers[0].b) < TF32_TOL
    lin.close()
    rt.close()


def test_side_stream_and_pool(M):
    """A side stream waits for the primary stream first (the reference's
    stream.join(runtime.stream())): the same forward on it gives the same
    bits. reserve_buffers fills the exact-size pool; a Linear's buffers go
    back to it when the layer is destroyed."""
    L, models = M
    rng = np.random.default_rng(4)
    x = rng.standard_normal((128, 64)).astype(F32)
    w = rng.uniform(-0.3, 0.3, (64, 32)).astype(F32)
    rt = models.Runtime()
    rt.reserve_buffers(64 * 32, 3)
    assert rt.pooled_buffers() == 3
    lin = models.Linear(rt, w, act=L.ACT_SILU)
    assert rt.pooled_buffers() == 2  # the weights took a pooled buffer
    xd = dev(x)
    a = host(lin.forward(xd))
    side = torch.cuda.Stream()
    b = lin.forward(xd, stream=side)
    side.synchronize()
    np.testing.assert_array_equal(host(b), a)
    lin.close()
    assert rt.pooled_buffers() == 3
    rt.close()


def test_errors_are_statuses(M):
    L, models = M
    import ctypes as C
    from oxf._host_sigs import LayerSpec
    rt = models.Runtime()
    spec = LayerSpec(4, 3, 0, 1)
    w = np.zeros((4, 3), F32)
    h = C.c_void_p()
    # a biased layer without bias values
    assert L.lib().oxf_linear_create(rt.handle, C.byref(spec), w.ctypes.data, None,
                                     C.byref(h)) == L.INVALID_ARG
    assert L.lib().oxf_linear_forward(None, None, 0, None, None, None, None) == L.INVALID_ARG
    lin = models.Linear(rt, w, np.zeros(3, F32))
    # learn on a biased layer without a bias gradient (linear.rs:394)
    x = torch.zeros((2, 4), device="cuda")
    g = torch.zeros((2, 3), device="cuda")
    assert L.lib().oxf_linear_learn(lin._h, x.data_ptr(), g.data_ptr(), None, 2, 0.1,
                                    None) == L.INVALID_ARG
    assert b"bias gradient" in L.lib().oxf_last_error_string()
    # zero rows: nothing to do
    assert L.lib().oxf_linear_forward(lin._h, None, 0, None, None, None, None) == 0
    lin.close()
    rt.close()
