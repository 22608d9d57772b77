"""CPU tests of the oracle itself: hand-derived known answers, the numpy
golden fixtures (independent restatement), finite-difference checks of
every backward formula, and invariants over random shapes (softmax rows are
distributions, normalised rows have the stated moments, the GEMM is
bilinear). These pin the checker before any GPU test trusts it.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

GOLDEN = np.load(Path(__file__).resolve().parent / "golden" / "golden.npz")


# ---------------------------------------------------------------- known answers
def test_softmax_constant_row_is_uniform():
    x = np.full((3, 37), 2.5, np.float32)
    np.testing.assert_allclose(O.softmax_rows(x), 1.0 / 37, rtol=1e-6)


def test_layer_norm_of_arithmetic_row():
    # row [a, a+1, ..., a+n-1]: mean a+(n-1)/2, var (n^2-1)/12
    n, a = 8, 3.0
    x = (a + np.arange(n, dtype=np.float32))[None, :]
    var = (n * n - 1) / 12.0
    want = (np.arange(n) - (n - 1) / 2.0) / np.sqrt(var + 1e-5)
    np.testing.assert_allclose(O.layer_norm_rows(x)[0], want, rtol=1e-5, atol=1e-6)


def test_rms_norm_of_unit_row():
    x = np.where(np.arange(10) % 2 == 0, 1.0, -1.0).astype(np.float32)[None, :]
    np.testing.assert_allclose(O.rms_norm_rows(x)[0], x[0] / np.sqrt(1.0 + 1e-5), rtol=1e-6)


def test_gelu_at_zero_and_limits():
    z = np.array([0.0, 10.0, -10.0], np.float32)
    y = O.act_forward(O.GELU, z)
    assert y[0] == 0.0 and abs(y[1] - 10.0) < 1e-5 and abs(y[2]) < 1e-5
    assert abs(O.act_derivative(O.GELU, np.array([0.0], np.float32))[0] - 0.5) < 1e-7


def test_identity_linear():
    x = np.random.default_rng(0).standard_normal((5, 4)).astype(np.float32)
    lin = O.LinearParams(np.eye(4, dtype=np.float32))
    y, _ = O.linear_forward(lin, x)
    np.testing.assert_array_equal(y, x)


def test_causal_mask_upper_triangle():
    m = O.causal_mask(np.zeros((4, 4), np.float32))
    assert np.isneginf(m[np.triu_indices(4, 1)]).all() and (m[np.tril_indices(4)] == 0).all()


def test_tf32_rounding_bit_patterns():
    # 1 + 2^-11 is a tie between 1 and 1 + 2^-10: RNA rounds away, RZ truncates.
    x = np.float32(1.0 + 2.0 ** -11)
    assert O.tf32_rna(float(x)) == 1.0 + 2.0 ** -10
    assert O.tf32_rz(float(x)) == 1.0
    assert O.tf32_rna(-float(x)) == -(1.0 + 2.0 ** -10)
    assert O.tf32_rna(1.0 + 2.0 ** -12) == 1.0


# ---------------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("name,fn", [
    ("softmax", lambda x: O.softmax_rows(x)),
    ("layer_norm", lambda x: O.layer_norm_rows(x)),
    ("rms_norm", lambda x: O.rms_norm_rows(x)),
    ("gelu", lambda x: O.act_forward(O.GELU, x)),
    ("gelu_d", lambda x: O.act_derivative(O.GELU, x)),
    ("sum_rows", lambda x: O.sum_rows(x)),
    ("sum_cols", lambda x: O.sum_cols(x)),
])
def test_oracle_matches_golden_forward(name, fn):
    assert rel_err(fn(GOLDEN["rows_x"]), GOLDEN[name]) < 2e-6


def test_oracle_matches_golden_backward():
    x, dy = GOLDEN["rows_x"], GOLDEN["rows_dy"]
    p = O.softmax_rows(x)
    assert rel_err(O.softmax_backward(p, dy), GOLDEN["softmax_bwd"]) < 2e-6
    assert rel_err(O.layer_norm_backward(x, dy), GOLDEN["layer_norm_bwd"]) < 2e-6
    assert rel_err(O.rms_norm_backward(x, dy), GOLDEN["rms_norm_bwd"]) < 2e-6
    assert rel_err(O.loss_rows(x, GOLDEN["loss_t"]), GOLDEN["loss_rows"]) < 2e-6


@pytest.mark.parametrize("rounding,tol", [(O.GEMM_F32, 1e-6), (O.GEMM_TF32_RNA, 2e-3),
                                          (O.GEMM_TF32_RZ, 4e-3)])
def test_oracle_gemm_golden(rounding, tol):
    c = O.gemm(GOLDEN["gemm_a"], GOLDEN["gemm_b"], rounding=rounding)
    assert rel_err(c, GOLDEN["gemm_c"]) < tol


def test_oracle_gemm_transposed_modes():
    A, B = GOLDEN["gemm_a"], GOLDEN["gemm_b"]
    want = GOLDEN["gemm_c"]
    assert rel_err(O.gemm(A.T.copy(), B, a_trans=True), want) < 1e-6
    assert rel_err(O.gemm(A, B.T.copy(), b_trans=True), want) < 1e-6
    assert rel_err(O.gemm(A.T.copy(), B.T.copy(), a_trans=True, b_trans=True), want) < 1e-6


def _tiny_transformer(norm):
    g = GOLDEN
    k = f"tf_{norm}_"
    lin = lambda n, act=O.IDENTITY: O.LinearParams(g[k + n], None, act)
    ffn = O.MlpParams([lin("w1", O.GELU), lin("w2")])
    nt = O.NORM_LAYER if norm == "layer" else O.NORM_RMS
    return O.TransformerParams(lin("wq"), lin("wk"), lin("wv"), g[k + "pos"], ffn, lin("wo"), nt,
                               g[k + "x"].shape[0])


@pytest.mark.parametrize("norm", ["layer", "rms"])
def test_oracle_transformer_step_golden(norm):
    """Full training step (forward, backward, immediate SGD) against the
    numpy restatement of encoder.rs:114-186."""
    t = _tiny_transformer(norm)
    k = f"tf_{norm}_"
    y, loss, dx = O.transformer_train_step(t, GOLDEN[k + "x"], GOLDEN[k + "t"], 0.05)
    assert rel_err(y, GOLDEN[k + "y"]) < 1e-5
    assert rel_err(dx, GOLDEN[k + "dx"]) < 1e-4
    for name, arr in [("wq", t.q.w), ("wk", t.k.w), ("wv", t.v.w), ("pos", t.position),
                      ("w1", t.ffn.layers[0].w), ("w2", t.ffn.layers[1].w), ("wo", t.o.w)]:
        assert rel_err(arr, GOLDEN[k + name + "_new"]) < 1e-5, name


# ---------------------------------------------------------------- finite differences
def _fd_check(f, x, dy, analytic, h=1e-3, n_probe=12, rng=None):
    """Central differences of sum(f(x) * dy) w.r.t. probed entries of x."""
    rng = rng or np.random.default_rng(7)
    x = x.astype(np.float64)
    idx = [tuple(rng.integers(0, s) for s in x.shape) for _ in range(n_probe)]
    for i in idx:
        xp, xm = x.copy(), x.copy()
        xp[i] += h
        xm[i] -= h
        num = ((f(xp.astype(np.float32)).astype(np.float64) - f(xm.astype(np.float32))) * dy).sum() / (2 * h)
        assert abs(num - analytic[i]) < 2e-2 * max(1.0, abs(num)), (i, num, analytic[i])


def test_fd_layer_norm_backward(rng):
    x = rng.standard_normal((3, 16)).astype(np.float32)
    dy = rng.standard_normal((3, 16)).astype(np.float32)
    _fd_check(O.layer_norm_rows, x, dy, O.layer_norm_backward(x, dy))


def test_fd_rms_norm_backward(rng):
    x = rng.standard_normal((3, 16)).astype(np.float32)
    dy = rng.standard_normal((3, 16)).astype(np.float32)
    _fd_check(O.rms_norm_rows, x, dy, O.rms_norm_backward(x, dy))


def test_fd_softmax_backward(rng):
    x = rng.standard_normal((3, 16)).astype(np.float32)
    dy = rng.standard_normal((3, 16)).astype(np.float32)
    _fd_check(O.softmax_rows, x, dy, O.softmax_backward(O.softmax_rows(x), dy))


def test_fd_gelu_derivative(rng):
    x = rng.standard_normal((4, 8)).astype(np.float32)
    dy = rng.standard_normal((4, 8)).astype(np.float32)
    _fd_check(lambda v: O.act_forward(O.GELU, v), x, dy, O.act_derivative(O.GELU, x) * dy)


def test_fd_transformer_input_gradient():
    """dL/dx of the oracle's training step against central differences of
    the summed row loss (lr = 0 leaves the weights untouched)."""
    t = _tiny_transformer("layer")
    x, tg = GOLDEN["tf_layer_x"], GOLDEN["tf_layer_t"]
    _, _, dx = O.transformer_train_step(t.copy(), x, tg, 0.0)

    def loss(xx):
        y = O.transformer_forward(t, xx)
        return O.loss_rows(y, tg).astype(np.float64).sum()

    rng = np.random.default_rng(3)
    for _ in range(6):
        i = (rng.integers(0, x.shape[0]), rng.integers(0, x.shape[1]))
        xp, xm = x.astype(np.float64).copy(), x.astype(np.float64).copy()
        xp[i] += 1e-2
        xm[i] -= 1e-2
        num = (loss(xp.astype(np.float32)) - loss(xm.astype(np.float32))) / 2e-2
        assert abs(num - dx[i]) < 5e-3 + 5e-2 * abs(num), (i, num, dx[i])


def test_grads_accumulate_equals_immediate_update():
    """Deferred update from accumulated gradients == the reference's
    immediate per-layer SGD for one sequence (the DP step relies on it)."""
    t1 = _tiny_transformer("rms")
    t2 = t1.copy()
    x, tg = GOLDEN["tf_rms_x"], GOLDEN["tf_rms_t"]
    O.transformer_train_step(t1, x, tg, 0.05)
    g = np.zeros(t2.flat().size, np.float32)
    O.transformer_train_step(t2, x, tg, 0.0, grads=g)
    assert rel_err(t2.flat() - 0.05 * g, t1.flat()) < 1e-6


def _ref_hash(x):
    """common.rs:3-9 in numpy uint32 arithmetic (wrapping)."""
    x = np.asarray(x, np.uint32)
    with np.errstate(over="ignore"):
        x = x + (x << np.uint32(13))
        x = x - (x >> np.uint32(17))
        x = x * (x << np.uint32(5))
    return x


def test_fills_known_answers():
    """slice_set_seq (elementwise.rs:24-35) and slice_set_random
    (elementwise.rs:37-43) against independent numpy restatements."""
    np.testing.assert_array_equal(O.fill_seq(5), [0, 1, 2, 3, 4])
    np.testing.assert_array_equal(O.fill_seq(5, ascending=False), [5, 4, 3, 2, 1])
    n, seed = 4099, 0xFFFFFF00  # seed + index wraps past 2^32
    idx = np.arange(n, dtype=np.uint64)
    h = _ref_hash(((np.uint64(seed) + idx) & np.uint64(0xFFFFFFFF)).astype(np.uint32))
    want = h.astype(np.float32) / np.float32(4294967296.0)
    np.testing.assert_array_equal(O.fill_random(n, seed), want)
    assert O.fill_random(1, 0)[0] == 0.0  # hash(0) == 0


def test_map_sum_and_matrix_slice_known_answers(rng):
    x = rng.standard_normal(10000).astype(np.float32)
    assert abs(O.map_sum(x, 4) - 0.5 * np.sum(x.astype(np.float64) ** 2)) < 1e-5 * np.sum(x ** 2)
    assert abs(O.map_sum(x, 0, 2.0) - 2 * np.sum(x.astype(np.float64))) < 1e-3
    m = np.arange(6 * 8, dtype=np.float32).reshape(6, 8)
    got = O.matrix_slice(m, 3, 4, 2, 4)
    want = np.concatenate([m[r:r + 3, c:c + 4].ravel() for r in (0, 3) for c in (0, 4)])
    np.testing.assert_array_equal(got, want)


def test_exchange_sgd_known_answers():
    """The data-parallel update: rank-order f32 sum, one rounding, every
    rank written, nothing outside [offset, offset+count) touched."""
    n = 11
    p = np.arange(n, dtype=np.float32)
    g = [np.full(n, v, np.float32) for v in (1.0, 2.0, 3.0)]
    out = O.exchange_sgd([p, p, p], g, 2, 7, 0.5)
    for q in range(3):
        want = p.copy()
        want[2:9] -= np.float32(3.0)  # 0.5 * (1 + 2 + 3)
        np.testing.assert_array_equal(out[q], want)
    np.testing.assert_array_equal(p, np.arange(n, dtype=np.float32))  # inputs untouched
    # left-to-right order: (1e8 + 1) rounds to 1e8 in f32, then - 1e8 = 0
    g = [np.float32([1e8]), np.float32([1.0]), np.float32([-1e8])]
    out = O.exchange_sgd([np.float32([5.0])] * 3, g, 0, 1, 1.0)
    assert out[0][0] == 5.0 and out[2][0] == 5.0
    # one rounding: p - s*lr with s*lr not representable
    p1, g1 = np.float32([1.0]), np.float32([1.0 + 2.0 ** -23])
    lr = np.float32(1.0 - 2.0 ** -24)
    want = np.float32(np.float64(p1[0]) - np.float64(g1[0]) * np.float64(lr))
    assert O.exchange_sgd([p1], [g1], 0, 1, float(lr))[0][0] == want


def test_dot_known_answers(rng):
    """Vector::dot (vector.rs:109-115): 1·1 + 2·2 + ... and a float64 check."""
    x = np.arange(1, 101, dtype=np.float32)
    assert O.dot(x, x) == float(np.sum(np.arange(1, 101) ** 2))  # 338350, exact in f32
    a = rng.standard_normal(100001).astype(np.float32)
    b = rng.standard_normal(100001).astype(np.float32)
    want = float(np.dot(a.astype(np.float64), b.astype(np.float64)))
    assert abs(O.dot(a, b) - want) <= 1e-5 * float(np.sum(np.abs(a * b)))
    assert O.dot(a[:0], b[:0]) == 0.0


# ---------------------------------------------------------------- invariants (property tests)
from hypothesis import given, settings, strategies as st  # noqa: E402

INVARIANT = settings(max_examples=30, deadline=None)
shapes = st.tuples(st.integers(1, 9), st.integers(1, 300))


def _rows(shape, seed, scale=3.0):
    return (scale * np.random.default_rng(seed).standard_normal(shape)).astype(np.float32)


@INVARIANT
@given(shape=shapes, seed=st.integers(0, 2**31 - 1), scale=st.floats(0.1, 4.0))
def test_softmax_rows_are_distributions(shape, seed, scale):
    """Every row of softmax(scale·x) is a probability distribution whose
    order follows x's (max-subtracted exp, row.rs:55-113)."""
    x = _rows(shape, seed)
    p = O.softmax_rows(x, scale=scale).astype(np.float64)
    assert (p >= 0).all() and (p <= 1).all()
    np.testing.assert_allclose(p.sum(axis=1), 1.0, rtol=0, atol=1e-5)
    i = np.argmax(x, axis=1)
    assert (p[np.arange(x.shape[0]), i] >= p.max(axis=1) * (1 - 1e-6)).all()


@INVARIANT
@given(shape=shapes, seed=st.integers(0, 2**31 - 1), period=st.integers(1, 12))
def test_causal_softmax_rows_see_only_the_past(shape, seed, period):
    """With causal period s, row r attends to columns 0..r mod s only."""
    x = _rows(shape, seed)
    p = O.softmax_rows(x, causal_period=period).astype(np.float64)
    for r in range(x.shape[0]):
        last = r % period
        assert not p[r, last + 1:].any()
        assert abs(p[r, :last + 1].sum() - 1.0) < 1e-5


@INVARIANT
@given(rows=st.integers(1, 6), cols=st.integers(2, 300), seed=st.integers(0, 2**31 - 1),
       shift=st.floats(-50, 50), scale=st.floats(0.5, 8.0))
def test_layer_norm_rows_are_standardised_and_shift_invariant(rows, cols, seed, shift, scale):
    """LayerNorm output has zero mean and variance var/(var+eps) per row
    (biased variance, row.rs:115-177), and adding a constant to a row does
    not change it."""
    x = _rows((rows, cols), seed, scale)
    y = O.layer_norm_rows(x).astype(np.float64)
    var = x.astype(np.float64).var(axis=1)
    np.testing.assert_allclose(y.mean(axis=1), 0.0, atol=2e-5)
    np.testing.assert_allclose(y.var(axis=1), var / (var + 1e-5), rtol=2e-4)
    y2 = O.layer_norm_rows((x + np.float32(shift)).astype(np.float32)).astype(np.float64)
    np.testing.assert_allclose(y2, y, atol=2e-3 * (1 + abs(shift) / scale))


@INVARIANT
@given(rows=st.integers(1, 6), cols=st.integers(1, 300), seed=st.integers(0, 2**31 - 1))
def test_rms_norm_rows_have_unit_mean_square(rows, cols, seed):
    """RMSNorm output has mean square ms/(ms+eps) per row (row.rs:349-396)."""
    x = _rows((rows, cols), seed)
    y = O.rms_norm_rows(x).astype(np.float64)
    ms = (x.astype(np.float64) ** 2).mean(axis=1)
    np.testing.assert_allclose((y ** 2).mean(axis=1), ms / (ms + 1e-5), rtol=1e-4)


@INVARIANT
@given(m=st.integers(1, 24), n=st.integers(1, 24), k=st.integers(1, 40),
       seed=st.integers(0, 2**31 - 1), a=st.floats(-3, 3), b=st.floats(-3, 3))
def test_gemm_is_bilinear(m, n, k, seed, a, b):
    """The f32 oracle GEMM is linear in each operand to f32 rounding, and
    agrees with the float64 product (gemm.rs:202-373 semantics)."""
    rng = np.random.default_rng(seed)
    A1, A2 = (rng.standard_normal((m, k)).astype(np.float32) for _ in range(2))
    B = rng.standard_normal((k, n)).astype(np.float32)
    lhs = O.gemm((np.float32(a) * A1 + np.float32(b) * A2).astype(np.float32), B)
    rhs = a * O.gemm(A1, B).astype(np.float64) + b * O.gemm(A2, B).astype(np.float64)
    scale = (abs(a) + abs(b) + 1) * (np.abs(A1).max() + np.abs(A2).max()) * np.abs(B).max() * k
    assert np.abs(lhs - rhs).max() <= 1e-5 * scale
    exact = A1.astype(np.float64) @ B.astype(np.float64)
    assert np.abs(O.gemm(A1, B) - exact).max() <= 1e-5 * max(1.0, np.abs(exact).max()) * k ** 0.5


@INVARIANT
@given(world=st.integers(1, 8), n=st.integers(1, 200), data=st.data(),
       lr=st.floats(1e-4, 2.0), seed=st.integers(0, 2**31 - 1))
def test_exchange_sgd_any_world_and_range(world, n, data, lr, seed):
    """For any world size and ragged range, every rank ends with the same
    parameters: p - lr * (g_0 + ... + g_{W-1}) inside [offset, offset+count)
    (rank-order f32 sum, then one rounding: within one ulp of the float64
    evaluation of that expression), unchanged outside; inputs untouched."""
    offset = data.draw(st.integers(0, n))
    count = data.draw(st.integers(0, n - offset))
    rng = np.random.default_rng(seed)
    p = rng.standard_normal(n).astype(np.float32)
    gs = [rng.standard_normal(n).astype(np.float32) for _ in range(world)]
    p_in, g_in = p.copy(), [g.copy() for g in gs]
    out = O.exchange_sgd([p] * world, gs, offset, count, lr)
    np.testing.assert_array_equal(p, p_in)
    for g, g0 in zip(gs, g_in):
        np.testing.assert_array_equal(g, g0)
    s = gs[0].copy()
    for g in gs[1:]:
        s = (s + g).astype(np.float32)
    want = p.copy()
    sl = slice(offset, offset + count)
    want[sl] = (p[sl].astype(np.float64) - s[sl].astype(np.float64) * np.float64(np.float32(lr))
                ).astype(np.float32)
    for q in range(world):
        np.testing.assert_array_equal(out[q], out[0])
    one_ulp = np.spacing(np.maximum(np.abs(out[0]), np.abs(want)))  # sign-safe near zero
    assert (np.abs(out[0] - want) <= one_ulp).all()
    np.testing.assert_array_equal(out[0][:offset], p[:offset])
    np.testing.assert_array_equal(out[0][offset + count:], p[offset + count:])


# ---------------------------------------------------------------- multi-head attention
def _mha_f64(q, k, v, h, causal):
    """Multi-head attention in float64: head j takes columns j·D/h.. of Q, K
    and j·Hv/h.. of V, scores scaled by 1/sqrt(D/h); outputs concatenated."""
    q, k, v = (np.asarray(a, np.float64) for a in (q, k, v))
    S, D = q.shape
    Hv = v.shape[1]
    dq, dv = D // h, Hv // h
    att, P = np.zeros((S, Hv)), np.zeros((h, S, S))
    for j in range(h):
        s = q[:, j * dq:(j + 1) * dq] @ k[:, j * dq:(j + 1) * dq].T / np.sqrt(dq)
        if causal:
            s[np.triu_indices(S, 1)] = -np.inf
        e = np.exp(s - s.max(1, keepdims=True))
        P[j] = e / e.sum(1, keepdims=True)
        att[:, j * dv:(j + 1) * dv] = P[j] @ v[:, j * dv:(j + 1) * dv]
    return att, P


def _mha_backward_f64(q, k, v, P, dr, h):
    q, k, v, dr = (np.asarray(a, np.float64) for a in (q, k, v, dr))
    S, D = q.shape
    Hv = v.shape[1]
    hq, hv = D // h, Hv // h
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    for j in range(h):
        cq, cv = slice(j * hq, (j + 1) * hq), slice(j * hv, (j + 1) * hv)
        p = P[j]
        dp = dr[:, cv] @ v[:, cv].T
        dv[:, cv] = p.T @ dr[:, cv]
        ds = p * (dp - (p * dp).sum(1, keepdims=True)) / np.sqrt(hq)
        dq[:, cq] = ds @ k[:, cq]
        dk[:, cq] = ds.T @ q[:, cq]
    return dq, dk, dv


@pytest.mark.parametrize("heads", [1, 2, 4])
@pytest.mark.parametrize("causal", [False, True])
def test_attention_heads_against_float64(heads, causal):
    """The oracle's multi-head attention core (forward and backward) against
    an independent float64 restatement; heads = 1 is the reference's
    single-head attention (attention.rs:359-401, 297-308)."""
    rng = np.random.default_rng(40 + heads)
    S, D, Hv = 24, 32, 48
    q = rng.standard_normal((S, D)).astype(np.float32)
    k = rng.standard_normal((S, D)).astype(np.float32)
    v = rng.standard_normal((S, Hv)).astype(np.float32)
    dr = rng.standard_normal((S, Hv)).astype(np.float32)
    att, p = O.attention_heads(q, k, v, heads, causal)
    att_ref, p_ref = _mha_f64(q, k, v, heads, causal)
    assert rel_err(att, att_ref) < 1e-5
    assert rel_err(p, p_ref) < 1e-5
    got = O.attention_heads_backward(q, k, v, p, dr, heads)
    want = _mha_backward_f64(q, k, v, p_ref, dr, heads)
    for g, w in zip(got, want):
        assert rel_err(g, w) < 1e-5


def test_transformer_heads_one_is_the_single_head_block():
    """The multi-head entry points with one head reproduce the single-head
    block bit for bit (forward and one training step), and more heads
    change the result."""
    seq, hidden, ffn = 16, 32, 64
    rng = np.random.default_rng(8)
    def lin(i, o, act=O.IDENTITY):
        return O.LinearParams((rng.standard_normal((i, o)) * 0.2).astype(np.float32), None, act)
    t = O.TransformerParams(lin(hidden, hidden), lin(hidden, hidden), lin(hidden, hidden),
                            (0.1 * rng.standard_normal((seq, hidden))).astype(np.float32),
                            O.MlpParams([lin(hidden, ffn, O.GELU), lin(ffn, hidden)]),
                            lin(hidden, hidden), O.NORM_LAYER, seq)
    x = rng.standard_normal((seq, hidden)).astype(np.float32)
    tg = rng.standard_normal((seq, hidden)).astype(np.float32)
    s, keep = t.struct()
    y1 = np.empty((seq, hidden), np.float32)
    O.lib().oxo_transformer_forward_heads(O.C.byref(s), O._p(x), O._p(y1), 0, O.GEMM_F32, 1)
    np.testing.assert_array_equal(y1, O.transformer_forward(t, x))
    g1 = np.zeros(t.flat().size, np.float32)
    g2 = np.zeros_like(g1)
    r1 = O.transformer_train_step(t.copy(), x, tg, 0.0, grads=g1)
    s2, keep2 = t.struct()
    y2, l2, dx2 = (np.empty((seq, hidden), np.float32), np.empty(seq, np.float32),
                   np.empty_like(x))
    O.lib().oxo_transformer_train_step_heads(O.C.byref(s2), O._p(x), O._p(tg), O._p(y2),
                                             O._p(l2), O._p(dx2), 0.0, O._p(g2), O.GEMM_F32, 1)
    np.testing.assert_array_equal(r1[2], dx2)
    np.testing.assert_array_equal(g1, g2)
    y4 = O.transformer_forward(t, x, heads=4)
    assert rel_err(y4, y1) > 1e-4
