"""GPU parity of the row, elementwise and reduction kernels against the CPU
oracle, through the C ABI. Tolerance (north_star): norm / softmax /
elementwise <= 1e-5, measured as max|gpu - oracle| / max|oracle| per output.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-5

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import kernels
    return kernels


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# widths: warp-per-row tiers, block-per-row tiers, the 16384 cap, ragged
# widths (looped path) and a width past the register cap
WIDTHS = [1, 3, 4, 36, 128, 1000, 1024, 2048, 2052, 4096, 8192, 12288, 16384, 20000]
ROWS = [1, 7, 33]


def cases(rng, widths=WIDTHS, rows=ROWS):
    for c in widths:
        for r in rows:
            if r * c > 2_000_000:
                continue
            yield r, c


def test_softmax_rows(K, rng):
    for r, c in cases(rng):
        x = rng.standard_normal((r, c)).astype(np.float32) * 3
        for scale, period in [(1.0, 0), (0.125, 0), (1.0, r)]:
            want = O.softmax_rows(x, scale, period)
            got = host(K.softmax_rows(dev(x), scale, period))
            assert rel_err(got, want) < TOL, (r, c, scale, period)


def test_softmax_causal_period_batched(K, rng):
    # 3 sequences of 16 rows each: row index is taken modulo the period
    x = rng.standard_normal((48, 16)).astype(np.float32)
    got = host(K.softmax_rows(dev(x), 0.5, 16))
    assert rel_err(got, O.softmax_rows(x, 0.5, 16)) < TOL
    assert np.all(got[np.arange(48) % 16 == 0, 1:] == 0.0)


def test_layer_norm_rows(K, rng):
    for r, c in cases(rng):
        x = (rng.standard_normal((r, c)) * 2 + 0.5).astype(np.float32)
        assert rel_err(host(K.layer_norm_rows(dev(x))), O.layer_norm_rows(x)) < TOL, (r, c)


def test_layer_norm_affine(K, rng):
    for c in [36, 1024, 2048, 20000]:
        x = rng.standard_normal((5, c)).astype(np.float32)
        g = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
        b = (0.1 * rng.standard_normal(c)).astype(np.float32)
        got = host(K.layer_norm_rows(dev(x), 1e-5, dev(g), dev(b)))
        assert rel_err(got, O.layer_norm_rows(x, 1e-5, g, b)) < TOL


def test_rms_norm_rows(K, rng):
    for r, c in cases(rng):
        x = rng.standard_normal((r, c)).astype(np.float32)
        assert rel_err(host(K.rms_norm_rows(dev(x))), O.rms_norm_rows(x)) < TOL, (r, c)
    x = rng.standard_normal((4, 1024)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    assert rel_err(host(K.rms_norm_rows(dev(x), 1e-5, dev(g))), O.rms_norm_rows(x, 1e-5, g)) < TOL



@pytest.mark.parametrize("c", [64, 200, 512, 1000, 2048])
def test_norm_params_staged_per_block(K, rng, c):
    """Warp-per-row widths (up to 2048), where a block of eight rows stages
    gamma and beta in shared memory once: 37 rows leave the last block with
    five live rows. gamma only, beta only and both, LayerNorm and RMSNorm,
    out of place and in place; the device error word stays clear."""
    from oxf import _lib
    r = 37
    x = (rng.standard_normal((r, c)) * 2 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    b = (0.1 * rng.standard_normal(c)).astype(np.float32)
    for gg, bb in [(g, b), (g, None), (None, b)]:
        want = O.layer_norm_rows(x, 1e-5, gg, bb)
        out = torch.empty((r, c), device="cuda")
        K.norm_rows(dev(x), out, _lib.NORM_LAYER, 1e-5, None if gg is None else dev(gg),
                    None if bb is None else dev(bb))
        assert rel_err(host(out), want) < TOL, (c, gg is None, bb is None)
        got = host(K.layer_norm_rows(dev(x), 1e-5, None if gg is None else dev(gg),
                                     None if bb is None else dev(bb)))
        assert rel_err(got, want) < TOL
    out = torch.empty((r, c), device="cuda")
    K.norm_rows(dev(x), out, _lib.NORM_RMS, 1e-5, dev(g))
    assert rel_err(host(out), O.rms_norm_rows(x, 1e-5, g)) < TOL
    assert rel_err(host(K.rms_norm_rows(dev(x), 1e-5, dev(g))), O.rms_norm_rows(x, 1e-5, g)) < TOL
    assert K.device_error() == 0


def test_activation_forward_several_pieces_per_thread(K, rng):
    """In-place activation forward over 700001 float4s, more than the grid
    covers in one pass, so threads load their next piece before storing the
    current one and the last pass is ragged; identity takes the generic loop."""
    n = 4 * 700001
    a = (3 * rng.standard_normal(n)).astype(np.float32)
    for act in (O.GELU, O.RELU, O.SILU):
        assert rel_err(host(K.unary(dev(a), 2, act)), O.act_forward(act, a)) < TOL, act
    np.testing.assert_array_equal(host(K.unary(dev(a), 2, 0)), a)

def close(got, want, scale, tol=TOL):
    """max|got - want| <= tol * scale, where scale is the magnitude of the
    largest term the formula combines (not of its possibly cancelling
    result)."""
    return float(np.abs(np.asarray(got, np.float64) - want).max()) <= tol * scale


def test_backward_kernels(K, rng):
    for r, c in cases(rng):
        x = rng.standard_normal((r, c)).astype(np.float32)
        dy = rng.standard_normal((r, c)).astype(np.float32)
        p = O.softmax_rows(x)
        out = torch.empty((r, c), device="cuda")
        got = host(K.softmax_backward(dev(p), dev(dy), out, 0.5))
        assert close(got, O.softmax_backward(p, dy, 0.5), np.abs(p * dy).max() + 1e-30), (r, c)
        # LN: dx = inv_std/N (N dy - sum dy - xhat sum(dy xhat)): terms ~ inv_std |dy|
        inv_std = 1 / np.sqrt(x.var(axis=1, keepdims=True) + 1e-5)
        got = host(K.layer_norm_backward(dev(x), dev(dy), out))
        assert close(got, O.layer_norm_backward(x, dy), np.abs(inv_std * dy).max(), 2 * TOL), (r, c)
        # RMS: dx = dy/r - x sum(x dy)/(N r^3): terms ~ |dy|/r
        inv_r = 1 / np.sqrt((x * x).mean(axis=1, keepdims=True) + 1e-5)
        got = host(K.rms_norm_backward(dev(x), dev(dy), out))
        assert close(got, O.rms_norm_backward(x, dy), np.abs(inv_r * dy).max()), (r, c)


def test_row_and_column_sums(K, rng):
    for r, c in cases(rng, rows=[1, 7, 257]):
        x = rng.standard_normal((r, c)).astype(np.float32)
        out = torch.empty(r, device="cuda")
        assert rel_err(host(K.sum_rows(dev(x), out)), O.sum_rows(x)) < TOL, (r, c)
        outc = torch.empty(c, device="cuda")
        assert rel_err(host(K.sum_cols(dev(x), outc)), O.sum_cols(x)) < 1e-5, (r, c)
        K.sum_cols(dev(x), outc, accumulate=True)
        assert rel_err(host(outc), 2 * O.sum_cols(x)) < 1e-5


@pytest.mark.parametrize("rows", [1, 6, 16, 128])
def test_column_sums_of_wide_short_matrices(K, rng, rows):
    """The position gradient's shape: a few sequences' rows of S*H = 2^21
    columns (config 5), summed and accumulated into an existing gradient."""
    cols = 1 << 21 if rows <= 16 else 1 << 18
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    want = x.astype(np.float64).sum(axis=0)
    outc = torch.empty(cols, device="cuda")
    got = host(K.sum_cols(dev(x), outc))
    assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(x).sum(axis=0).max())
    assert rel_err(got, O.sum_cols(x)) < 1e-5
    K.sum_cols(dev(x), outc, accumulate=True)
    assert np.abs(host(outc) - 2 * want).max() <= 2e-5 * max(1.0, np.abs(x).sum(axis=0).max())


def test_loss_rows_and_mse_grad(K, rng):
    for r, c in cases(rng, widths=[1, 36, 1024, 2048, 20000]):
        y = rng.standard_normal((r, c)).astype(np.float32)
        t = rng.standard_normal((r, c)).astype(np.float32)
        out = torch.empty(r, device="cuda")
        assert rel_err(host(K.loss_rows(dev(y), dev(t), out)), O.loss_rows(y, t)) < TOL
        g = torch.empty((r, c), device="cuda")
        assert rel_err(host(K.mse_grad(dev(y), dev(t), g)), O.mse_grad(y, t)) < TOL


@pytest.mark.parametrize("n", [0, 1, 3, 4, 1001, 4096, 1 << 20])
def test_elementwise(K, rng, n):
    a = rng.standard_normal(n).astype(np.float32)
    b = (rng.standard_normal(n) + 3).astype(np.float32)
    out = torch.empty(n, device="cuda")
    if n == 0:
        K.binary(dev(a), dev(b), out, 0)  # empty slices are a no-op
        return
    for op in range(4):
        assert rel_err(host(K.binary(dev(a), dev(b), out, op)), O.binary(a, b, op)) < TOL
        t = dev(a)
        K.binary_assign(t, dev(b), op)
        assert rel_err(host(t), O.binary(a, b, op)) < TOL
    for act in (O.GELU, O.RELU, O.SILU):
        assert rel_err(host(K.unary(dev(a), 2, act)), O.act_forward(act, a)) < TOL
        assert rel_err(host(K.unary(dev(a), 3, act)), O.act_derivative(act, a)) < TOL
    assert rel_err(host(K.unary(dev(a), 0, 0.25)), a * np.float32(0.25)) < TOL
    assert rel_err(host(K.unary(dev(a), 1, 2.0)), a + np.float32(2.0)) < TOL
    assert rel_err(host(K.unary(dev(a), 4)), 0.5 * a * a) < TOL
    w = dev(a)
    K.sgd_update(w, dev(b), 0.01)
    assert rel_err(host(w), a - b * np.float32(0.01)) < TOL


@pytest.mark.parametrize("c", [1, 3, 4, 1024, 1030])
def test_binary_assign_by_rows(K, rng, c):
    m = rng.standard_normal((9, c)).astype(np.float32)
    v = (rng.standard_normal(c) + 2).astype(np.float32)
    for op in range(4):
        got = host(K.binary_assign_by_rows(dev(m), dev(v), op))
        assert rel_err(got, O.binary_assign_by_rows(m, v, op)) < TOL


def test_causal_mask_and_transpose(K, rng):
    for r, c in [(1, 1), (5, 9), (33, 33), (100, 64), (1024, 1024)]:
        m = rng.standard_normal((r, c)).astype(np.float32)
        got = host(K.causal_mask(dev(m)))
        np.testing.assert_array_equal(got, O.causal_mask(m))
        out = torch.empty((c, r), device="cuda")
        np.testing.assert_array_equal(host(K.transpose(dev(m), out)), m.T)


def test_slice_reductions(K, rng):
    for n in [0, 1, 1000, 1 << 20]:
        x = rng.standard_normal(n).astype(np.float32)
        out = torch.empty(1, device="cuda")
        s = host(K.slice_sum(dev(x), out))[0]
        assert abs(s - x.astype(np.float64).sum()) < 1e-4 * max(1.0, np.abs(x).sum())
        mx = host(K.slice_max(dev(x), out))[0]
        assert mx == (x.max() if n else np.float32(-3.4028235e38))


def test_shape_validation_matches_reference_asserts(K):
    from oxf._lib import OxfError, check, lib
    t = torch.zeros(10, device="cuda")
    # len % cols != 0 (norm.rs:12 needs whole rows)
    with pytest.raises(OxfError):
        check(lib().oxf_matrix_softmax_rows(K.ms(t), 3, 1.0, 0, None))
    # row vector length must equal cols (rows.rs:18)
    with pytest.raises(OxfError):
        K.binary_assign_by_rows(torch.zeros(3, 4, device="cuda"), torch.zeros(5, device="cuda"), 0)


def test_mse_loss_grad_fused(K, rng):
    for r, c in [(1, 1), (7, 36), (33, 1024), (5, 2048), (3, 20000)]:
        y = rng.standard_normal((r, c)).astype(np.float32)
        t = rng.standard_normal((r, c)).astype(np.float32)
        loss = torch.empty(r, device="cuda")
        dy = torch.empty((r, c), device="cuda")
        K.mse_loss_grad(dev(y), dev(t), loss, dy)
        assert rel_err(host(loss), O.loss_rows(y, t)) < TOL
        assert rel_err(host(dy), O.mse_grad(y, t)) < TOL


@pytest.mark.parametrize("n", [0, 1, 1000, (1 << 25) + 3])
def test_fills_match_reference_bitwise(K, n):
    """slice_set / slice_set_seq / slice_set_random: identical values to the
    oracle's restatement of elementwise.rs:15-43 (seq rounds large indices
    to f32 the same way)."""
    x = torch.empty(n, device="cuda")
    K.fill(x, 2.5)
    assert (host(x) == 2.5).all()
    for asc in (True, False):
        K.fill_seq(x, asc)
        np.testing.assert_array_equal(host(x), O.fill_seq(n, asc))
    for seed in (0, 12345, 0xFFFFFFF0):
        K.fill_random(x, seed)
        np.testing.assert_array_equal(host(x), O.fill_random(n, seed))


def test_map_sum(K, rng):
    x = rng.standard_normal(123457).astype(np.float32)
    out = torch.empty(1, device="cuda")
    for op, p in ((4, 0.0), (0, 0.5), (1, 1.0), (2, 1.0), (3, 1.0)):
        K.map_sum(dev(x), op, p, out)
        want = O.map_sum(x, op, p)
        scale = O.map_sum(np.abs(x), 0, 1.0) if op in (0, 1) else abs(want)
        assert abs(host(out)[0] - want) <= 1e-5 * max(scale, 1.0), (op, host(out)[0], want)
    with pytest.raises(Exception):
        K.map_sum(dev(x), 9, 0.0, out)


def test_dot(K, rng):
    """oxf_slice_dot against the oracle's Vector::dot (vector.rs:109-115),
    including the empty vector and the length check."""
    x = rng.standard_normal(123457).astype(np.float32)
    y = rng.standard_normal(123457).astype(np.float32)
    out = torch.empty(1, device="cuda")
    K.dot(dev(x), dev(y), out)
    want = O.dot(x, y)
    assert abs(host(out)[0] - want) <= 1e-5 * float(np.sum(np.abs(x * y)))
    K.dot(dev(x[:0].copy()), dev(y[:0].copy()), out)
    assert host(out)[0] == 0.0
    with pytest.raises(Exception, match="length"):
        K.dot(dev(x), dev(y[:10].copy()), out)


def test_matrix_slice(K, rng):
    m = rng.standard_normal((96, 160)).astype(np.float32)
    for tr, tc, tpr, nt in ((32, 40, 4, 12), (96, 160, 1, 1), (1, 1, 160, 160 * 96), (8, 16, 5, 3)):
        out = torch.empty(nt * tr * tc, device="cuda")
        K.matrix_slice(dev(m), out, tr, tc, tpr)
        np.testing.assert_array_equal(host(out), O.matrix_slice(m, tr, tc, tpr, nt))
    with pytest.raises(Exception, match="past the input"):
        K.matrix_slice(dev(m), torch.empty(13 * 32 * 40, device="cuda"), 32, 40, 4)
    with pytest.raises(Exception, match="exceeds input_cols"):
        K.matrix_slice(dev(m), torch.empty(32 * 40, device="cuda"), 32, 40, 5)


def test_bounded_wait_expires_and_context_survives(K):
    """Failure detection without a GPU fault: a wait that nothing completes
    expires after its bound (20 ms here; 4 s in the pipelines), sets the
    device error word and returns; the next kernels run normally."""
    import ctypes
    from oxf import _lib
    expired = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().oxf_wait_timeout_selftest(20000, ctypes.c_void_p(expired.data_ptr()),
                                                   K._stream(None)))
    torch.cuda.synchronize()
    assert int(expired.item()) == 1
    assert K.device_error() == 0x1FF
    assert K.device_error() == 0  # reading clears the word
    a = torch.randn(256, 128, device="cuda")
    b = torch.randn(128, 64, device="cuda")
    y = torch.empty(256, 64, device="cuda")
    K.matrix_multiply(a, b, y)
    ref = a.double() @ b.double()
    assert ((y.double() - ref).abs().max() / ref.abs().max()).item() < 5e-3
    assert K.device_error() == 0
