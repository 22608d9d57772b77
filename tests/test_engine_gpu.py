"""GPU parity of the executors (transformer and MLP engines) against the
oracle's single-sequence reference semantics, through the host C ABI.

The GPU runs every product in TF32 (operands truncated to 10 mantissa bits);
the oracle runs the same formulas with TF32 truncation emulated
(GEMM_TF32_RZ), so what remains is summation order and the tensor core's
internal accumulation. Tolerances: forward outputs 5e-3 (the north_star
TF32 bound), gradients and updates 1e-2 of their own scale (errors of a
whole backward pass compound through ~12 dependent products).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
FWD_TOL = 5e-3
GRAD_TOL = 1e-2
RZ = O.GEMM_TF32_RZ


@pytest.fixture(scope="module")
def M():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import _lib, kernels, models
    yield models
    assert kernels.device_error() == 0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy().copy()


def oracle_model(models, cfg, flat):
    """oracle.TransformerParams from a flat cursor-order parameter array."""
    parts = models.split_params(cfg, flat)
    q, k, v, o = cfg.layers()
    it = iter(parts)

    def lin(spec):
        w = next(it)
        b = next(it) if spec.bias else None
        return O.LinearParams(w, b, spec.act)

    lq, lk, lv = lin(q), lin(k), lin(v)
    pos = next(it)
    ffn = O.MlpParams([lin(l) for l in cfg.ffn.layers], cfg.ffn.res_range)
    lo = lin(o)
    return O.TransformerParams(lq, lk, lv, pos, ffn, lo, cfg.norm, cfg.seq)


CASES = [
    # seq, hidden, ffn, norm, bias
    (32, 64, 128, 1, False),
    (32, 64, 128, 0, True),
    (64, 128, 256, 1, True),
]


@pytest.mark.parametrize("seq,hidden,ffn,norm,bias", CASES)
def test_training_step_single_sequence(M, seq, hidden, ffn, norm, bias):
    """One reference training step (TrainingTransformer::forward + backward
    with per-layer SGD, encoder.rs:114-186) on one sequence."""
    cfg = M.transformer_config(seq, hidden, ffn, norm=norm, bias=bias)
    flat = M.init_transformer_params(cfg, seed=11)
    rng = np.random.default_rng(5)
    x = rng.standard_normal((seq, hidden)).astype(np.float32)
    t = rng.standard_normal((seq, hidden)).astype(np.float32)
    lr = 0.05

    ref = oracle_model(M, cfg, flat)
    y_ref, loss_ref, dx_ref = O.transformer_train_step(ref, x, t, lr, rounding=RZ)

    eng = M.Transformer(cfg, max_batch=1)
    eng.set_params(flat)
    eng.zero_grads()
    y = host(eng.train_forward(dev(x)))
    tt = dev(t)
    loss = host(eng.set_target(tt))
    dx = host(eng.backward())
    eng.sgd(lr)
    new = eng.get_params()
    assert rel_err(y, y_ref) < FWD_TOL
    assert rel_err(loss, loss_ref) < FWD_TOL
    assert rel_err(dx, dx_ref) < GRAD_TOL
    # compare the parameter update lr*grad, tensor by tensor
    check_per_tensor(cfg, flat - new, flat - ref.flat())
    eng.close()


def check_per_tensor(cfg, got, want, tol=GRAD_TOL):
    """Per-tensor relative error of a flat cursor-order vector. A bias
    gradient is a column sum of G that can cancel to ~0 (the key bias's is
    exactly 0: softmax ignores a per-row constant), so it is measured
    against the scale of its Linear's weight gradient instead."""
    off, prev_scale = 0, None
    for sh in cfg.shapes():
        n = int(np.prod(sh))
        g, w = got[off:off + n], want[off:off + n]
        scale = float(np.abs(w).max())
        if len(sh) == 1 and prev_scale is not None:
            scale = max(scale, prev_scale)
        err = float(np.abs(np.asarray(g, np.float64) - w).max()) / max(scale, 1e-30)
        assert err < tol, (sh, err)
        prev_scale = float(np.abs(w).max()) if len(sh) == 2 else None
        off += n


def test_batched_gradients_are_sums_of_sequences(M):
    """B sequences in one call == the sum of B single-sequence gradients
    (the data-parallel step relies on this)."""
    seq, hidden, ffn, B = 32, 64, 128, 3
    cfg = M.transformer_config(seq, hidden, ffn, norm=1)
    flat = M.init_transformer_params(cfg, seed=3)
    rng = np.random.default_rng(9)
    x = rng.standard_normal((B, seq, hidden)).astype(np.float32)
    t = rng.standard_normal((B, seq, hidden)).astype(np.float32)
    g_ref = np.zeros(flat.size, np.float32)
    ys = []
    for b in range(B):
        ref = oracle_model(M, cfg, flat)
        y, _, _ = O.transformer_train_step(ref, x[b], t[b], 0.0, grads=g_ref, rounding=RZ)
        ys.append(y)
    eng = M.Transformer(cfg, max_batch=4)
    eng.set_params(flat)
    eng.zero_grads()
    y = host(eng.train_forward(dev(x.reshape(B * seq, hidden))))
    eng.set_target(dev(t.reshape(B * seq, hidden)))
    eng.backward()
    g = host(eng.grads)
    assert rel_err(y, np.concatenate(ys)) < FWD_TOL
    check_per_tensor(cfg, g, g_ref)
    # buckets tile the arena in cursor order: attention+position, ffn, output
    b2, b1, b0 = eng.bucket(2), eng.bucket(1), eng.bucket(0)
    assert b2[0] == 0 and b2[0] + b2[1] == b1[0] and b1[0] + b1[1] == b0[0]
    assert b0[0] + b0[1] == eng.n
    eng.close()


@pytest.mark.parametrize("causal", [False, True])
def test_inference_forward(M, causal):
    """InferenceTransformer::forward (encoder) and the decoder's masked
    forward (decoder.rs:50-52) with NormType::Rms."""
    seq, hidden, ffn, B = 64, 128, 512, 2
    cfg = M.transformer_config(seq, hidden, ffn, norm=0)
    flat = M.init_transformer_params(cfg, seed=21)
    x = np.random.default_rng(2).standard_normal((B, seq, hidden)).astype(np.float32)
    eng = M.Transformer(cfg, max_batch=B)
    eng.set_params(flat)
    y = host(eng.forward(dev(x.reshape(B * seq, hidden)), causal=causal))
    ref = oracle_model(M, cfg, flat)
    for b in range(B):
        want = O.transformer_forward(ref, x[b], causal=causal, rounding=RZ)
        assert rel_err(y[b * seq:(b + 1) * seq], want) < FWD_TOL
    eng.close()


MH_CASES = [
    # seq, hidden, ffn, norm, bias, heads
    (32, 64, 128, 1, False, 2),
    (64, 128, 256, 0, True, 4),
    (32, 128, 256, 1, False, 16),   # 8-wide heads
    (16, 48, 96, 1, True, 8),       # 6-wide heads: column slices TMA cannot describe
]


@pytest.mark.parametrize("seq,hidden,ffn,norm,bias,heads", MH_CASES)
def test_multi_head_training_step(M, seq, hidden, ffn, norm, bias, heads):
    """Multi-head attention (oxf_transformer_set_heads): B = 2 sequences
    through one training step against the oracle's per-head restatement
    (oxo_transformer_train_step_heads), gradients summed over sequences."""
    cfg = M.transformer_config(seq, hidden, ffn, norm=norm, bias=bias)
    flat = M.init_transformer_params(cfg, seed=17)
    rng = np.random.default_rng(6)
    B = 2
    x = rng.standard_normal((B, seq, hidden)).astype(np.float32)
    t = rng.standard_normal((B, seq, hidden)).astype(np.float32)
    g_ref = np.zeros(flat.size, np.float32)
    ys, dxs = [], []
    for b in range(B):
        ref = oracle_model(M, cfg, flat)
        y, _, dx = O.transformer_train_step(ref, x[b], t[b], 0.0, grads=g_ref, rounding=RZ,
                                            heads=heads)
        ys.append(y)
        dxs.append(dx)
    eng = M.Transformer(cfg, max_batch=B, heads=heads)
    assert eng.heads == heads
    eng.set_params(flat)
    eng.zero_grads()
    y = host(eng.train_forward(dev(x.reshape(B * seq, hidden))))
    eng.set_target(dev(t.reshape(B * seq, hidden)))
    dx = host(eng.backward())
    g = host(eng.grads)
    assert rel_err(y, np.concatenate(ys)) < FWD_TOL
    assert rel_err(dx, np.concatenate(dxs)) < GRAD_TOL
    check_per_tensor(cfg, g, g_ref)
    eng.close()


@pytest.mark.parametrize("seq,heads", [(64, 4), (256, 4), (256, 2)])
@pytest.mark.parametrize("causal", [False, True])
def test_multi_head_inference_forward(M, causal, seq, heads):
    """Multi-head inference forward (encoder and the decoder's causal mask)
    on two sequences against the oracle: per-head products at seq 64, the
    fused kernel (oxf_attention_heads_forward, 32- and 64-wide heads) at
    seq 256."""
    hidden, ffn, B = 128, 256, 2
    cfg = M.transformer_config(seq, hidden, ffn, norm=0)
    flat = M.init_transformer_params(cfg, seed=23)
    x = np.random.default_rng(3).standard_normal((B, seq, hidden)).astype(np.float32)
    eng = M.Transformer(cfg, max_batch=B)
    eng.set_params(flat)
    y1 = host(eng.forward(dev(x.reshape(B * seq, hidden)), causal=causal))
    eng.set_heads(heads)
    y = host(eng.forward(dev(x.reshape(B * seq, hidden)), causal=causal))
    ref = oracle_model(M, cfg, flat)
    for b in range(B):
        want = O.transformer_forward(ref, x[b], causal=causal, rounding=RZ, heads=heads)
        assert rel_err(y[b * seq:(b + 1) * seq], want) < FWD_TOL
    # back to one head: the single-head result again, bit for bit
    eng.set_heads(1)
    y1b = host(eng.forward(dev(x.reshape(B * seq, hidden)), causal=causal))
    np.testing.assert_array_equal(y1b, y1)
    eng.close()


def test_set_heads_rejects_non_divisors(M):
    from oxf import _lib
    cfg = M.transformer_config(16, 64, 128)
    eng = M.Transformer(cfg, max_batch=1)
    for bad in (0, -2, 3, 128):
        with pytest.raises(RuntimeError):
            eng.set_heads(bad)
    assert eng.heads == 1
    assert _lib.lib().oxf_transformer_set_heads(None, 2) == _lib.INVALID_ARG
    eng.close()


def test_backward_needs_the_training_forward(M):
    """The inference forward stores no pre-activations (FFN, output Linear)
    and no probabilities, so a backward after it is refused; after
    train_forward it runs, and both forwards give the same output."""
    rng = np.random.default_rng(31)
    cfg = M.transformer_config(32, 64, 128)
    eng = M.Transformer(cfg, max_batch=1)
    eng.set_params(rng.uniform(-0.1, 0.1, cfg.param_count()).astype(np.float32))
    x = dev(rng.standard_normal((32, 64)))
    y_inf = host(eng.forward(x))
    with pytest.raises(RuntimeError, match="train_forward"):
        eng.backward_stage(0)
    y_tr = host(eng.train_forward(x))
    assert rel_err(y_inf, y_tr) < FWD_TOL
    eng.set_target(dev(rng.standard_normal((32, 64))))
    eng.backward()
    eng.close()


def test_two_block_stack_matches_oracle_composition(M):
    """TransformerStack: two blocks, block 1's output feeding block 2, one
    training step on two sequences. The oracle runs block 2's reference step
    on block 1's output; block 1's step then gets block 2's input gradient
    as its output gradient (a target of y1 - dL/dy1 * width gives exactly
    that MSE gradient). Outputs, input gradients and every tensor's summed
    gradient against the oracle."""
    seq, hidden, ffn, B = 32, 64, 128, 2
    cfgs = [M.transformer_config(seq, hidden, ffn, norm=1),
            M.transformer_config(seq, hidden, ffn, norm=0, bias=True)]
    flats = [M.init_transformer_params(c, seed=40 + i) for i, c in enumerate(cfgs)]
    rng = np.random.default_rng(12)
    x = rng.standard_normal((B, seq, hidden)).astype(np.float32)
    t = rng.standard_normal((B, seq, hidden)).astype(np.float32)
    g_ref = [np.zeros(f.size, np.float32) for f in flats]
    ys, dxs = [], []
    for b in range(B):
        r1, r2 = (oracle_model(M, c, f) for c, f in zip(cfgs, flats))
        y1 = O.transformer_forward(r1, x[b], rounding=RZ)
        y2, _, dy1 = O.transformer_train_step(r2, y1, t[b], 0.0, grads=g_ref[1], rounding=RZ)
        _, _, dx = O.transformer_train_step(oracle_model(M, cfgs[0], flats[0]), x[b],
                                            y1 - dy1 * np.float32(hidden), 0.0, grads=g_ref[0],
                                            rounding=RZ)
        ys.append(y2)
        dxs.append(dx)
    st = M.TransformerStack(cfgs, max_batch=B)
    st.set_params(flats)
    st.zero_grads()
    y = host(st.train_forward(dev(x.reshape(B * seq, hidden))))
    st.set_target(dev(t.reshape(B * seq, hidden)))
    dx = host(st.backward())
    assert rel_err(y, np.concatenate(ys)) < FWD_TOL
    assert rel_err(dx, np.concatenate(dxs)) < GRAD_TOL
    for blk, cfg, gr in zip(st.blocks, cfgs, g_ref):
        check_per_tensor(cfg, host(blk.grads), gr)
    # inference through the stack equals the training forward's output
    np.testing.assert_allclose(host(st.forward(dev(x.reshape(B * seq, hidden)))), y,
                               rtol=0, atol=1e-5 * np.abs(y).max())
    with pytest.raises(ValueError):
        M.TransformerStack([M.transformer_config(seq, hidden, ffn, out=32), cfgs[1]])
    st.close()


def test_train_step_host_api(M):
    """The host-memory step (H2D, forward, loss, backward, SGD on the mean
    gradient, loss D2H) equals the device-level calls."""
    seq, hidden, ffn, B = 32, 64, 128, 2
    cfg = M.transformer_config(seq, hidden, ffn, norm=1)
    flat = M.init_transformer_params(cfg, seed=4)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((B * seq, hidden)).astype(np.float32)
    t = rng.standard_normal((B * seq, hidden)).astype(np.float32)
    a = M.Transformer(cfg, max_batch=B)
    a.set_params(flat)
    loss = a.train_step_host(x, t, 0.1)
    b = M.Transformer(cfg, max_batch=B)
    b.set_params(flat)
    b.zero_grads()
    b.train_forward(dev(x))
    rl = host(b.set_target(dev(t)))
    b.backward()
    b.sgd(0.1 / B)
    assert abs(loss - rl.mean()) < 1e-5 * max(1.0, abs(loss))
    assert rel_err(a.get_params() - flat, b.get_params() - flat) < 1e-4
    a.close()
    b.close()


@pytest.mark.parametrize("res", [None, (0, 2)])
def test_mlp_engine(M, res):
    """MlpExecutor forward + backward + SGD (mlp.rs:53-168) with biases,
    GELU and the residual range of config 3, scaled down."""
    from oxf import _lib
    rows, d, h = 96, 64, 256
    cfg = M.MlpConfig([M.Layer(d, h, _lib.ACT_GELU, True), M.Layer(h, d, 0, True)], res)
    rng = np.random.default_rng(8)
    w1 = rng.uniform(-np.sqrt(6 / d), np.sqrt(6 / d), (d, h)).astype(np.float32)
    b1 = (0.01 * rng.standard_normal(h)).astype(np.float32)
    w2 = rng.uniform(-np.sqrt(6 / h), np.sqrt(6 / h), (h, d)).astype(np.float32)
    b2 = (0.01 * rng.standard_normal(d)).astype(np.float32)
    x = rng.standard_normal((rows, d)).astype(np.float32)
    t = rng.standard_normal((rows, d)).astype(np.float32)
    flat = np.concatenate([w1.ravel(), b1, w2.ravel(), b2])
    lr = 0.05
    ref = O.MlpParams([O.LinearParams(w1, b1, O.GELU), O.LinearParams(w2, b2)], res)
    y_ref = O.mlp_forward(ref, x, rounding=RZ)
    dy_ref = O.mse_grad(y_ref, t)
    _, dx_ref = O.mlp_train_step(ref, x, dy_ref, lr, rounding=RZ)

    eng = M.Mlp(cfg, rows)
    eng.params.copy_(dev(flat))
    eng.zero_grads()
    xd = dev(x)
    y = torch.empty((rows, d), device="cuda")
    eng.forward(xd, y)
    assert rel_err(host(y), y_ref) < FWD_TOL
    dy = dev(dy_ref)
    dx = torch.empty((rows, d), device="cuda")
    eng.backward(dy, dx)
    eng.sgd(lr)
    assert rel_err(host(dx), dx_ref) < GRAD_TOL
    new_ref = np.concatenate([p.ravel() for p in ref.params()])
    assert rel_err(flat - host(eng.params), flat - new_ref) < GRAD_TOL
    eng.close()


def test_pipelined_host_steps_match_device_steps(M):
    """DataParallelTrainer.run_host (inputs of step i+1 copied on a side
    stream while step i computes, losses read one step late) gives the same
    losses and parameters as device-resident steps taken one at a time."""
    from oxf.dp import DataParallelTrainer
    seq, hidden, ffn, B, steps = 32, 64, 128, 2, 4
    cfg = M.transformer_config(seq, hidden, ffn, norm=1)
    flat = M.init_transformer_params(cfg, seed=6)
    rng = np.random.default_rng(3)
    data = [(rng.standard_normal((B * seq, hidden)).astype(np.float32),
             rng.standard_normal((B * seq, hidden)).astype(np.float32)) for _ in range(steps)]
    a = M.Transformer(cfg, max_batch=B)
    a.set_params(flat)
    ta = DataParallelTrainer(a, B, 0.05, seq)
    pinned = [(torch.from_numpy(x).pin_memory(), torch.from_numpy(t).pin_memory())
              for x, t in data]
    got = ta.run_host(pinned)
    b = M.Transformer(cfg, max_batch=B)
    b.set_params(flat)
    tb = DataParallelTrainer(b, B, 0.05, seq)
    want = [float(tb.step(dev(x), dev(t)).item()) for x, t in data]
    assert len(got) == steps
    # column sums and split-K tiles add atomically, so runs agree to rounding
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-7)
    assert rel_err(a.get_params() - flat, b.get_params() - flat) < 1e-4
    a.close()
    b.close()


def test_checkpoint_engine_round_trip(M, tmp_path):
    """dump_transformer / load_transformer and dump_mlp / load_mlp on the
    engines' device arenas: the loaded engines hold the same parameters and
    compute the same outputs."""
    from oxf import _lib
    from oxf import checkpoint as ck
    seq, hidden, ffn, B = 32, 64, 128, 2
    cfg = M.transformer_config(seq, hidden, ffn, norm=0, bias=True)
    flat = M.init_transformer_params(cfg, seed=9)
    a = M.Transformer(cfg, max_batch=B)
    a.set_params(flat)
    ck.dump_transformer(a, tmp_path / "model")
    b = ck.load_transformer(tmp_path / "model.toml", max_batch=B)
    assert b.cfg == cfg
    np.testing.assert_array_equal(b.get_params(), flat)
    x = dev(np.random.default_rng(4).standard_normal((B * seq, hidden)))
    ya = host(a.forward(x))
    yb = host(b.forward(x))
    np.testing.assert_array_equal(ya, yb)
    a.close()
    b.close()

    mcfg = M.MlpConfig([M.Layer(64, 256, _lib.ACT_GELU, True), M.Layer(256, 64, 0, True)], (0, 2))
    m = M.Mlp(mcfg, 96)
    mflat = np.random.default_rng(5).standard_normal(m.n).astype(np.float32)
    m.params.copy_(dev(mflat))
    ck.dump_mlp_engine(m, tmp_path / "mlp")
    m2 = ck.load_mlp_engine(tmp_path / "mlp", 96)
    assert m2.cfg == mcfg
    np.testing.assert_array_equal(host(m2.params), mflat)
    m.close()
    m2.close()


def test_full_size_c5_sequence_matches_oracle(M):
    """Config 5 at its full per-sequence size ([1024, 2048], FFN 8192,
    LayerNorm): one sequence's training step (output, loss, input gradient
    and the per-tensor SGD update) against the oracle's multithreaded C
    restatement, inside a batch of 2 so the batched paths are exercised.
    The second sequence's contribution is taken out by running it alone."""
    seq, hidden, ffn = 1024, 2048, 8192
    cfg = M.transformer_config(seq, hidden, ffn, norm=1)
    flat = M.init_transformer_params(cfg, seed=0)
    rng = np.random.default_rng(21)
    x = rng.standard_normal((2, seq, hidden)).astype(np.float32)
    t = rng.standard_normal((2, seq, hidden)).astype(np.float32)
    lr = 1e-3

    ref = oracle_model(M, cfg, flat)
    y_ref, loss_ref, dx_ref = O.transformer_train_step(ref, x[0], t[0], lr, rounding=RZ)

    eng = M.Transformer(cfg, max_batch=2)
    eng.set_params(flat)
    eng.zero_grads()
    y = host(eng.train_forward(dev(x.reshape(2 * seq, hidden))))
    loss = host(eng.set_target(dev(t.reshape(2 * seq, hidden))))
    dx = host(eng.backward())
    g2 = host(eng.grads).copy()
    assert rel_err(y[:seq], y_ref) < FWD_TOL
    assert rel_err(loss[:seq], loss_ref) < FWD_TOL
    assert rel_err(dx[:seq], dx_ref) < GRAD_TOL
    eng.zero_grads()
    eng.train_forward(dev(x[1]))
    eng.set_target(dev(t[1]))
    eng.backward()
    g1 = host(eng.grads)
    check_per_tensor(cfg, lr * (g2 - g1), flat - ref.flat())
    eng.close()


def test_trainer_checkpoint_round_trip_on_the_engine(tmp_path):
    """DataParallelTrainer.save_checkpoint / load_checkpoint on the engine's
    device arena (one rank): the parameters after a step survive a write,
    an overwrite of the arena and a read; a checkpoint of another shape is
    refused and leaves the arena as it was."""
    import torch
    from oxf import _lib, models
    from oxf.dp import DataParallelTrainer
    cfg = models.transformer_config(64, 128, 256, norm=_lib.NORM_LAYER)
    m = models.Transformer(cfg, max_batch=2)
    m.set_params(models.init_transformer_params(cfg, seed=0))
    tr = DataParallelTrainer(m, 2, 0.05, 64)
    g = torch.Generator(device="cuda").manual_seed(4)
    x = torch.randn(2 * 64, 128, device="cuda", generator=g)
    t = torch.randn(2 * 64, 128, device="cuda", generator=g)
    tr.step(x, t)
    torch.cuda.synchronize()
    saved = m.get_params()
    path = str(tmp_path / "engine_ckpt")
    tr.save_checkpoint(path, cfg)
    m.params.zero_()
    tr.load_checkpoint(path, cfg)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(m.get_params(), saved)
    other = models.transformer_config(64, 128, 512, norm=_lib.NORM_LAYER)
    with pytest.raises(ValueError):
        tr.load_checkpoint(path, other)
    np.testing.assert_array_equal(m.get_params(), saved)
    tr.close()
    m.close()
