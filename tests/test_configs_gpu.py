"""Every benchmark configuration (configs 1-5) at its own size, on the GPU, against the
oracle (oracle/oxf_oracle.c, multithreaded) or float64.

GEMM-bearing outputs are compared with the oracle run in the reference's
operand rounding, TF32 round-to-nearest-away (src/cuda/device/gemm.rs:286-347,
GEMM_TF32_RNA), while the tensor cores truncate (round toward zero): the
difference is inside the TF32 bound. Tolerances, all as max|gpu - want| over
max|want| of the same output unless a scale is named:
  TF32 products and executor forward outputs   5e-3
  executor gradients and updates               1e-2 of their own tensor's scale
                                               (a backward pass chains up to
                                               a dozen dependent TF32 products)
  row / elementwise kernels                    1e-5 (backward kernels: of the
                                               scale of the terms they combine)

Layouts and distributions are the configurations' own (seeded host RNGs,
numpy default_rng).
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
FWD_TOL = 5e-3
GRAD_TOL = 1e-2
ROW_TOL = 1e-5
F32 = np.float32


@pytest.fixture(scope="module")
def G():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import _lib, kernels, models
    yield _lib, kernels, models
    assert kernels.device_error() == 0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, F32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy().copy()


def close(got, want, scale, tol=ROW_TOL):
    return float(np.abs(np.asarray(got, np.float64) - want).max()) <= tol * scale


# ---------------------------------------------------------------- config 1
def config1_operands():
    """X [256,128] U(-1,1) from seed 0, then W [128,64]
    U(-1/sqrt(128), 1/sqrt(128)) from the same generator."""
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (256, 128)).astype(F32)
    b = 1 / np.sqrt(128)
    w = rng.uniform(-b, b, (128, 64)).astype(F32)
    return x, w


def test_c1_linear_seed0(G):
    """Linear forward of config 1 (no bias, Identity) through
    matrix_multiply's argument order (module.rs:179-191): within 5e-3 of the
    exact product, and equal to the oracle with the reference's RNA operand
    rounding up to f32 summation order (the tiny-product kernel rounds RNA
    and sums in K order)."""
    _, K, _ = G
    x, w = config1_operands()
    y = torch.empty((256, 64), device="cuda")
    K.matrix_multiply(dev(x), dev(w), y)
    got = host(y)
    exact = x.astype(np.float64) @ w.astype(np.float64)
    assert rel_err(got, exact) < TF32_TOL
    want = O.gemm(x, w, rounding=RNA)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()


# ---------------------------------------------------------------- config 2
def test_c2_row_suite_at_config_size(G):
    """[4096, 1024]: x and upstream gradients N(0,1), gamma = 1 + 0.1 N(0,1),
    beta = 0.1 N(0,1), eps = 1e-5. Softmax, LayerNorm (plain and affine),
    RMSNorm (plain and with gamma) forward and backward, GELU forward and
    backward, and the row-broadcast add, each against the oracle."""
    _, K, _ = G
    R, C = 4096, 1024
    rng = np.random.default_rng(2000)
    x = rng.standard_normal((R, C)).astype(F32)
    dy = rng.standard_normal((R, C)).astype(F32)
    gamma = (1 + 0.1 * rng.standard_normal(C)).astype(F32)
    beta = (0.1 * rng.standard_normal(C)).astype(F32)
    out = torch.empty((R, C), device="cuda")

    p = O.softmax_rows(x)
    assert rel_err(host(K.softmax_rows(dev(x))), p) < ROW_TOL
    assert rel_err(host(K.layer_norm_rows(dev(x))), O.layer_norm_rows(x)) < ROW_TOL
    assert rel_err(host(K.layer_norm_rows(dev(x), 1e-5, dev(gamma), dev(beta))),
                   O.layer_norm_rows(x, 1e-5, gamma, beta)) < ROW_TOL
    assert rel_err(host(K.rms_norm_rows(dev(x))), O.rms_norm_rows(x)) < ROW_TOL
    assert rel_err(host(K.rms_norm_rows(dev(x), 1e-5, dev(gamma))),
                   O.rms_norm_rows(x, 1e-5, gamma)) < ROW_TOL

    got = host(K.softmax_backward(dev(p), dev(dy), out))
    assert close(got, O.softmax_backward(p, dy), np.abs(p * dy).max())
    inv_std = 1 / np.sqrt(x.var(axis=1, keepdims=True) + 1e-5)
    got = host(K.layer_norm_backward(dev(x), dev(dy), out))
    assert close(got, O.layer_norm_backward(x, dy), np.abs(inv_std * dy).max())
    inv_r = 1 / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-5)
    got = host(K.rms_norm_backward(dev(x), dev(dy), out))
    assert close(got, O.rms_norm_backward(x, dy), np.abs(inv_r * dy).max())

    assert rel_err(host(K.unary(dev(x), 2, O.GELU)), O.act_forward(O.GELU, x)) < ROW_TOL
    got = host(K.mul_act_derivative(dev(dy), dev(x), O.GELU))
    assert rel_err(got, dy * O.act_derivative(O.GELU, x)) < ROW_TOL
    got = host(K.binary_assign_by_rows(dev(x), dev(beta), 0))
    assert rel_err(got, O.binary_assign_by_rows(x, beta, 0)) < ROW_TOL


# ---------------------------------------------------------------- config 3
def test_c3_mlp_step_at_config_size(G):
    """One full MLP step of config 3: X [8192,1024] N(0,1), Linear 1024->4096
    + GELU -> Linear 4096->1024 with the residual range (0, 2), Kaiming-
    uniform weights (bound sqrt(6/fan_in)), biases 0.01 N(0,1), MSE against
    N(0,1) targets. Output, row losses, input gradient and the whole SGD
    update against the oracle's MlpExecutor restatement (mlp.rs:53-168)."""
    L, K, M = G
    rows, d, h, lr = 8192, 1024, 4096, 1e-3
    rng = np.random.default_rng(3000)
    x = rng.standard_normal((rows, d)).astype(F32)
    w1 = rng.uniform(-np.sqrt(6 / d), np.sqrt(6 / d), (d, h)).astype(F32)
    b1 = (0.01 * rng.standard_normal(h)).astype(F32)
    w2 = rng.uniform(-np.sqrt(6 / h), np.sqrt(6 / h), (h, d)).astype(F32)
    b2 = (0.01 * rng.standard_normal(d)).astype(F32)
    t = rng.standard_normal((rows, d)).astype(F32)
    flat = np.concatenate([w1.ravel(), b1, w2.ravel(), b2])

    ref = O.MlpParams([O.LinearParams(w1, b1, O.GELU), O.LinearParams(w2, b2)], (0, 2))
    y_ref = O.mlp_forward(ref, x, rounding=RNA)
    loss_ref = O.loss_rows(y_ref, t)
    dy_ref = O.mse_grad(y_ref, t)
    _, dx_ref = O.mlp_train_step(ref, x, dy_ref, lr, rounding=RNA)
    new_ref = np.concatenate([p.ravel() for p in ref.params()])

    cfg = M.MlpConfig([M.Layer(d, h, L.ACT_GELU, True), M.Layer(h, d, 0, True)], (0, 2))
    eng = M.Mlp(cfg, rows)
    eng.params.copy_(dev(flat))
    eng.zero_grads()
    xd, td = dev(x), dev(t)
    y = torch.empty((rows, d), device="cuda")
    eng.forward(xd, y)
    loss = torch.empty(rows, device="cuda")
    dy = torch.empty((rows, d), device="cuda")
    K.mse_loss_grad(y, td, loss, dy)
    dx = torch.empty((rows, d), device="cuda")
    eng.backward(dy, dx)
    eng.sgd(lr)
    assert rel_err(host(y), y_ref) < FWD_TOL
    assert rel_err(host(loss), loss_ref) < FWD_TOL
    assert rel_err(host(dx), dx_ref) < GRAD_TOL
    upd, upd_ref = flat - host(eng.params), flat - new_ref
    off = 0
    for n, name in ((d * h, "w1"), (h, "b1"), (h * d, "w2"), (d, "b2")):
        err = rel_err(upd[off:off + n], upd_ref[off:off + n])
        assert err < GRAD_TOL, (name, err)
        off += n
    eng.close()


# ---------------------------------------------------------------- square sweep
@pytest.mark.parametrize("n", [512, 1024, 2048, 4096, 8192])
def test_square_sweep_against_float64(G, n):
    """Config 3's square sweep, U(-1,1) operands: the whole product against
    float64 up to 2048; at 4096 and 8192, 32 sampled rows and 32 sampled
    columns (a row or column permutation, or errors that cancel across a
    row, would show; a row-sum checksum could not see them)."""
    _, K, _ = G
    rng = np.random.default_rng(3100 + n)
    A = rng.uniform(-1, 1, (n, n)).astype(F32)
    B = rng.uniform(-1, 1, (n, n)).astype(F32)
    out = torch.empty((n, n), device="cuda")
    K.gemm(dev(A), dev(B), out)
    got = host(out)
    if n <= 2048:
        assert rel_err(got, A.astype(np.float64) @ B.astype(np.float64)) < TF32_TOL
        return
    rows = rng.choice(n, 32, replace=False)
    cols = rng.choice(n, 32, replace=False)
    want_r = A[rows].astype(np.float64) @ B.astype(np.float64)
    want_c = A.astype(np.float64) @ B[:, cols].astype(np.float64)
    scale = max(np.abs(want_r).max(), np.abs(want_c).max())
    assert np.abs(got[rows] - want_r).max() / scale < TF32_TOL
    assert np.abs(got[:, cols] - want_c).max() / scale < TF32_TOL


# ---------------------------------------------------------------- config 4
def _oracle_transformer(models, cfg, flat):
    parts = iter(models.split_params(cfg, flat))
    q, k, v, o = cfg.layers()

    def lin(spec):
        w = next(parts)
        b = next(parts) if spec.bias else None
        return O.LinearParams(w, b, spec.act)

    lq, lk, lv = lin(q), lin(k), lin(v)
    pos = next(parts)
    ffn = O.MlpParams([lin(layer) for layer in cfg.ffn.layers], cfg.ffn.res_range)
    lo = lin(o)
    return O.TransformerParams(lq, lk, lv, pos, ffn, lo, cfg.norm, cfg.seq)


def test_c4_inference_sequences_at_config_size(G):
    """Config 4 at its per-sequence size: [2048, 1024], NormType::Rms, FFN
    1024 -> 4096 -> 1024 GELU, Xavier-uniform projections, position table
    N(0, 0.02), inputs N(0,1). Two sequences in one batched call, each
    against the oracle's InferenceBlock::forward (inference.rs:76-109)."""
    L, K, M = G
    seq, hidden, ffn = 2048, 1024, 4096
    cfg = M.transformer_config(seq, hidden, ffn, norm=L.NORM_RMS)
    flat = M.init_transformer_params(cfg, seed=4000)
    x = np.random.default_rng(4001).standard_normal((2, seq, hidden)).astype(F32)
    eng = M.Transformer(cfg, max_batch=2)
    eng.set_params(flat)
    y = host(eng.forward(dev(x.reshape(2 * seq, hidden))))
    ref = _oracle_transformer(M, cfg, flat)
    for b in range(2):
        want = O.transformer_forward(ref, x[b], rounding=RNA)
        assert rel_err(y[b * seq:(b + 1) * seq], want) < FWD_TOL, b
    eng.close()


# ---------------------------------------------------------------- config 5
def test_c5_forward_against_reference_rounding(G):
    """Config 5's forward at its full per-sequence size ([1024, 2048], FFN
    8192, LayerNorm) against the oracle in the reference's RNA operand
    rounding (the training-step test compares in the tensor cores' own
    rounding, to isolate summation order)."""
    L, K, M = G
    seq, hidden, ffn = 1024, 2048, 8192
    cfg = M.transformer_config(seq, hidden, ffn, norm=L.NORM_LAYER)
    flat = M.init_transformer_params(cfg, seed=0)
    x = np.random.default_rng(21).standard_normal((1, seq, hidden)).astype(F32)
    eng = M.Transformer(cfg, max_batch=1)
    eng.set_params(flat)
    y = host(eng.train_forward(dev(x.reshape(seq, hidden))))
    want = O.transformer_forward(_oracle_transformer(M, cfg, flat), x[0], rounding=RNA)
    assert rel_err(y, want) < FWD_TOL
    eng.close()
