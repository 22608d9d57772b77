"""GPU parity of the tcgen05 TF32 GEMM (and its fused epilogue) against the
oracle's float64 product, through the C ABI.

Tolerances (north_star): plain TF32 <= 5e-3, 3xTF32 <= 1e-4, both as
max|gpu - exact| / max|exact| over the output. The reference rounds operands
to TF32 with round-to-nearest-away (gemm.rs:286-347); the tcgen05 path drops
the low 13 mantissa bits instead, which the 5e-3 bound covers.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

pytestmark = pytest.mark.gpu
TF32_TOL = 5e-3
TF32X3_TOL = 1e-4

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import kernels
    yield kernels
    code = kernels.device_error()
    assert code == 0, f"a bounded in-kernel wait timed out (code {code:#x})"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def operands(rng, M, N, Kd, at, bt, batch=None, dist="uniform"):
    gen = (lambda s: rng.uniform(-1, 1, s)) if dist == "uniform" else rng.standard_normal
    a_shape = (Kd, M) if at else (M, Kd)
    b_shape = (N, Kd) if bt else (Kd, N)
    if batch:
        a_shape, b_shape = (batch,) + a_shape, (batch,) + b_shape
    return gen(a_shape).astype(np.float32), gen(b_shape).astype(np.float32)


def config1_operands():
    """Config 1: X [256,128] U(-1,1) from seed 0, then W [128,64]
    U(-1/sqrt(128), 1/sqrt(128)) from the same generator."""
    g = np.random.default_rng(0)
    x = g.uniform(-1, 1, (256, 128)).astype(np.float32)
    w = g.uniform(-1 / np.sqrt(128), 1 / np.sqrt(128), (128, 64)).astype(np.float32)
    return x, w


def exact(A, B, at, bt):
    """float64 product of the f32 operands (numpy BLAS; the oracle's
    oxo_gemm_f64 computes the same thing, far slower)."""
    a = A.astype(np.float64)
    b = B.astype(np.float64)
    return (a.T if at else a) @ (b.T if bt else b)


SHAPES = [
    (128, 128, 32),     # one tile, one k-block
    (256, 64, 128),     # config 1 (Linear [256,128]x[128,64])
    (300, 200, 72),     # ragged M, N, K tails
    (128, 256, 1024),   # one BN=256 tile, deep K
    (1024, 1024, 1024),
    (516, 772, 260),
]


@pytest.mark.parametrize("at,bt", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,Kd", SHAPES)
def test_gemm_modes_tf32(K, rng, M, N, Kd, at, bt):
    A, B = operands(rng, M, N, Kd, at, bt)
    out = torch.empty((M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, a_trans=bool(at), b_trans=bool(bt))
    assert rel_err(host(out), exact(A, B, at, bt)) < TF32_TOL


@pytest.mark.parametrize("at,bt", [(0, 0), (1, 0), (0, 1)])
@pytest.mark.parametrize("M,N,Kd,variant", [
    (256, 64, 128, 0), (300, 200, 72, 0), (512, 384, 1024, 0),
    (300, 520, 96, 2),      # CTA pair, ragged
    (2048, 2560, 256, 0),   # enough 256 x 256 tiles for the CTA pair automatically
])
def test_gemm_tf32x3(K, rng, M, N, Kd, variant, at, bt):
    A, B = operands(rng, M, N, Kd, at, bt, dist="normal")
    out = torch.empty((M, N), device="cuda")
    ws = torch.empty(K.gemm_workspace_bytes(M, N, Kd, bool(at), bool(bt)) // 4 + 64,
                     device="cuda")
    K.gemm(dev(A), dev(B), out, a_trans=bool(at), b_trans=bool(bt), precision=1, workspace=ws,
           variant=variant)
    assert rel_err(host(out), exact(A, B, at, bt)) < TF32X3_TOL


def test_matrix_multiply_reference_signature(K, rng):
    """matrix_multiply(lhs, rhs, out, len, rows, cols) of module.rs:179-191
    on config 1's shapes and distributions (seed 0, as the config states)."""
    x, w = config1_operands()
    out = torch.empty((256, 64), device="cuda")
    K.matrix_multiply(dev(x), dev(w), out)
    assert rel_err(host(out), exact(x, w, 0, 0)) < TF32_TOL
    # and against the oracle's emulation of the reference's RNA operand rounding
    assert rel_err(host(out), O.gemm(x, w, rounding=O.GEMM_TF32_RNA)) < TF32_TOL


def test_unaligned_leading_dims_use_fallback(K, rng):
    # K = 33 gives a row pitch of 132 bytes, which TMA cannot describe
    for M, N, Kd in [(129, 257, 33), (7, 5, 3), (64, 64, 0)]:
        A, B = operands(rng, M, N, Kd, 0, 0)
        out = torch.empty((M, N), device="cuda")
        K.gemm(dev(A), dev(B), out)
        want = exact(A, B, 0, 0) if Kd else np.zeros((M, N))
        assert np.abs(host(out) - want).max() <= TF32_TOL * max(1.0, np.abs(want).max())


@pytest.mark.parametrize("at,bt", [(0, 1), (0, 0), (1, 0)])
def test_batched_gemm(K, rng, at, bt):
    # per-sequence attention products: [batch, S, S] = Q_b · K_bᵀ etc.
    batch, M, N, Kd = 3, 160, 96, 64
    A, B = operands(rng, M, N, Kd, at, bt, batch=batch)
    out = torch.empty((batch, M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, a_trans=bool(at), b_trans=bool(bt))
    got = host(out)
    for b in range(batch):
        assert rel_err(got[b], exact(A[b], B[b], at, bt)) < TF32_TOL, b


def test_batched_shared_operand(K, rng):
    batch, M, N, Kd = 4, 128, 192, 96
    A = rng.uniform(-1, 1, (batch, M, Kd)).astype(np.float32)
    B = rng.uniform(-1, 1, (Kd, N)).astype(np.float32)
    out = torch.empty((batch, M, N), device="cuda")
    K.gemm(dev(A), dev(B), out)
    got = host(out)
    for b in range(batch):
        assert rel_err(got[b], exact(A[b], B, 0, 0)) < TF32_TOL


def test_fused_linear_epilogue(K, rng):
    """Y = gelu(X·W + b + R) with the pre-activation stored (Linear::affine_on
    + activate_on, linear.rs:185-230)."""
    M, N, Kd = 384, 320, 256
    X, W = operands(rng, M, N, Kd, 0, 0)
    b = (0.1 * rng.standard_normal(N)).astype(np.float32)
    R = rng.standard_normal((M, N)).astype(np.float32)
    out = torch.empty((M, N), device="cuda")
    pre = torch.empty((M, N), device="cuda")
    K.gemm(dev(X), dev(W), out, bias=dev(b), residual=dev(R), pre_out=pre, act=1)
    z = exact(X, W, 0, 0) + b + R
    assert rel_err(host(pre), z) < TF32_TOL
    assert rel_err(host(out), O.act_forward(O.GELU, z.astype(np.float32))) < TF32_TOL


def test_grad_activation_epilogue(K, rng):
    """dZ = (G·Wᵀ) ⊙ gelu'(Z) fused (linear.rs:254-264 then 431-434)."""
    M, N, Kd = 256, 192, 128
    G = rng.standard_normal((M, Kd)).astype(np.float32)
    W = rng.uniform(-0.2, 0.2, (N, Kd)).astype(np.float32)  # stored [in=N, out=Kd]
    Z = rng.standard_normal((M, N)).astype(np.float32)
    out = torch.empty((M, N), device="cuda")
    K.gemm(dev(G), dev(W), out, b_trans=True, aux=dev(Z), grad_act=1)
    want = exact(G, W, 0, 1) * O.act_derivative(O.GELU, Z)
    assert rel_err(host(out), want) < TF32_TOL


def test_alpha_beta(K, rng):
    M, N, Kd = 200, 136, 64
    A, B = operands(rng, M, N, Kd, 0, 0)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    out = dev(C0)
    K.gemm(dev(A), dev(B), out, alpha=0.125, beta=-2.0)
    assert rel_err(host(out), 0.125 * exact(A, B, 0, 0) - 2.0 * C0) < TF32_TOL


@pytest.mark.parametrize("split", [0, 1, 3, 16])
def test_accumulate_split_k(K, rng, split):
    """W-gradient shape Xᵀ·G with a long K, accumulated atomically into an
    existing gradient buffer (split_k = 0 lets the library choose)."""
    M, N, Kd = 256, 384, 4096
    X = rng.standard_normal((Kd, M)).astype(np.float32)
    G = rng.standard_normal((Kd, N)).astype(np.float32)
    G0 = rng.standard_normal((M, N)).astype(np.float32)
    out = dev(G0)
    K.gemm(dev(X), dev(G), out, a_trans=True, accumulate=True, split_k=split, alpha=0.5)
    assert rel_err(host(out), G0 + 0.5 * exact(X, G, 1, 0)) < TF32_TOL


def test_refalgo_matches_reference_rounding(K, rng):
    """The measurement-only restatement of the reference kernel rounds
    operands RNA like gemm.rs; compare with the oracle's RNA emulation."""
    M, N, Kd = 256, 192, 128
    A, B = operands(rng, M, N, Kd, 0, 0)
    out = torch.empty((M, N), device="cuda")
    K.matrix_multiply_refalgo(dev(A), dev(B), out)
    assert rel_err(host(out), O.gemm(A, B, rounding=O.GEMM_TF32_RNA)) < 1e-5
    with pytest.raises(Exception):
        K.matrix_multiply_refalgo(dev(A[:, :100]), dev(B[:100]), out[:, :].view(M, N))


def test_large_square(K, rng):
    """Size-independent check at a sweep size: C·1 == A·(B·1) row sums."""
    n = 4096
    A = torch.empty((n, n), device="cuda").uniform_(-1, 1)
    B = torch.empty((n, n), device="cuda").uniform_(-1, 1)
    out = torch.empty((n, n), device="cuda")
    K.gemm(A, B, out)
    ones = torch.ones((n, 1), device="cuda", dtype=torch.float64)
    lhs = out.double() @ ones
    rhs = A.double() @ (B.double() @ ones)
    assert ((lhs - rhs).abs().max() / rhs.abs().max()).item() < TF32_TOL


def test_batch_reduce(K, rng):
    """C = R + Σ_b A_b·B_bᵀ in one GEMM (the input gradient of the three
    projections, attention.rs:127-131)."""
    batch, M, N, Kd = 3, 256, 192, 128
    A = rng.uniform(-1, 1, (batch, M, Kd)).astype(np.float32)
    B = rng.uniform(-1, 1, (batch, N, Kd)).astype(np.float32)
    R = rng.standard_normal((M, N)).astype(np.float32)
    out = torch.empty((M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, b_trans=True, residual=dev(R), reduce_batch=True)
    want = R + sum(exact(A[b], B[b], 0, 1) for b in range(batch))
    assert rel_err(host(out), want) < TF32_TOL


@pytest.mark.parametrize("variant", [1, 2, 3])
@pytest.mark.parametrize("at,bt", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,Kd", [(256, 256, 64), (300, 520, 72), (1024, 768, 256)])
def test_cta_pair_and_single_variants(K, rng, M, N, Kd, at, bt, variant):
    """variant 1: one CTA per 128-row tile; variant 2: a CTA pair per
    256 x 256 tile (tcgen05.mma.cta_group::2, half of B in each CTA);
    variant 3: a CTA pair per 256 x 512 tile (two MMAs per K step, the
    accumulator in all 512 TMEM columns; N = 256 leaves half the tile empty,
    N = 520 and 768 a ragged second tile)."""
    A, B = operands(rng, M, N, Kd, at, bt)
    out = torch.empty((M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, a_trans=bool(at), b_trans=bool(bt), variant=variant)
    assert rel_err(host(out), exact(A, B, at, bt)) < TF32_TOL


@pytest.mark.parametrize("variant", [2, 3])
def test_cta_pair_features(K, rng, variant):
    """Batched operands, fused epilogue, split-K accumulation and
    batch-reduce on the CTA-pair kernel (256- and 512-wide tiles)."""
    batch, M, N, Kd = 3, 256, 384, 128
    A, B = operands(rng, M, N, Kd, 0, 0, batch=batch)
    out = torch.empty((batch, M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, variant=variant)
    got = host(out)
    for b in range(batch):
        assert rel_err(got[b], exact(A[b], B[b], 0, 0)) < TF32_TOL
    X, W = operands(rng, 512, 256, 256, 0, 0)
    bias = (0.1 * rng.standard_normal(256)).astype(np.float32)
    R = rng.standard_normal((512, 256)).astype(np.float32)
    y = torch.empty((512, 256), device="cuda")
    pre = torch.empty((512, 256), device="cuda")
    K.gemm(dev(X), dev(W), y, bias=dev(bias), residual=dev(R), pre_out=pre, act=1, variant=variant)
    z = exact(X, W, 0, 0) + bias + R
    assert rel_err(host(pre), z) < TF32_TOL
    assert rel_err(host(y), O.act_forward(O.GELU, z.astype(np.float32))) < TF32_TOL
    Xt = rng.standard_normal((2048, 256)).astype(np.float32)
    G = rng.standard_normal((2048, 512)).astype(np.float32)
    G0 = rng.standard_normal((256, 512)).astype(np.float32)
    acc = dev(G0)
    K.gemm(dev(Xt), dev(G), acc, a_trans=True, accumulate=True, split_k=4, variant=variant)
    assert rel_err(host(acc), G0 + exact(Xt, G, 1, 0)) < TF32_TOL
    Ab = rng.uniform(-1, 1, (3, 256, 128)).astype(np.float32)
    Bb = rng.uniform(-1, 1, (3, 256, 128)).astype(np.float32)
    Rb = rng.standard_normal((256, 256)).astype(np.float32)
    red = torch.empty((256, 256), device="cuda")
    K.gemm(dev(Ab), dev(Bb), red, b_trans=True, residual=dev(Rb), reduce_batch=True, variant=variant)
    want = Rb + sum(exact(Ab[b], Bb[b], 0, 1) for b in range(3))
    assert rel_err(host(red), want) < TF32_TOL


@pytest.mark.parametrize("variant", [1, 2, 3])
@pytest.mark.parametrize("M,N,Kd", [(300, 200, 72), (512, 384, 128), (520, 1100, 96)])
def test_epilogue_tiles_batched_and_shared(K, rng, M, N, Kd, variant):
    """The TMA-staged epilogue on batched outputs: a residual shared by the
    batch (stride 0, a 2-D tensor map), per-item aux and pre-activation
    outputs (3-D maps), beta * C read back through TMA, ragged M and N
    (partial 32x32 tiles clipped by the map), and the bias tail."""
    batch = 2
    A, B = operands(rng, M, N, Kd, 0, 0, batch=batch)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float32)
    R = rng.standard_normal((M, N)).astype(np.float32)
    C0 = rng.standard_normal((batch, M, N)).astype(np.float32)
    out = dev(C0)
    pre = torch.empty((batch, M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, alpha=0.5, beta=0.25, bias=dev(bias), residual=dev(R),
           pre_out=pre, act=1, variant=variant)
    for b in range(batch):
        z = 0.5 * exact(A[b], B[b], 0, 0) + 0.25 * C0[b] + bias + R
        assert rel_err(host(pre)[b], z) < TF32_TOL
        assert rel_err(host(out)[b], O.act_forward(O.GELU, z.astype(np.float32))) < TF32_TOL
    X = rng.standard_normal((batch, M, N)).astype(np.float32)
    g = torch.empty((batch, M, N), device="cuda")
    K.gemm(dev(A), dev(B), g, aux=dev(X), grad_act=1, variant=variant)
    for b in range(batch):
        want = exact(A[b], B[b], 0, 0) * O.act_derivative(O.GELU, X[b]).astype(np.float64)
        assert rel_err(host(g)[b], want) < TF32_TOL


def test_epilogue_unaligned_output_falls_back(K, rng):
    """Aligned operands but an output leading dimension that TMA cannot
    describe (201 floats): the tcgen05 kernel keeps per-thread stores."""
    M, N, Kd = 256, 200, 128
    A, B = operands(rng, M, N, Kd, 0, 0)
    big = torch.zeros((M, 201), device="cuda")
    view = big[:, :N]
    R = rng.standard_normal((M, N)).astype(np.float32)
    K.gemm(dev(A), dev(B), view, residual=dev(R))
    assert rel_err(host(big)[:, :N], exact(A, B, 0, 0) + R) < TF32_TOL
    assert not host(big)[:, N:].any()


def test_accumulate_rejects_split_with_bias(K, rng):
    """Split-K adds each partial product into C, so a bias or residual would
    be added once per split: refused when asked for, avoided when automatic."""
    M, N, Kd = 256, 256, 4096
    A, B = operands(rng, M, N, Kd, 1, 0)
    bias = rng.standard_normal(N).astype(np.float32)
    acc = torch.zeros((M, N), device="cuda")
    with pytest.raises(Exception, match="split_k"):
        K.gemm(dev(A), dev(B), acc, a_trans=True, bias=dev(bias), accumulate=True, split_k=4)
    K.gemm(dev(A), dev(B), acc, a_trans=True, bias=dev(bias), accumulate=True)
    assert rel_err(host(acc), exact(A, B, 1, 0) + bias) < TF32_TOL


@pytest.mark.parametrize("M,N,Kd", [(256, 64, 128), (300, 200, 72), (1024, 512, 2048)])
def test_matrix_multiply_fp32_is_f32_exact(K, rng, M, N, Kd):
    """matrix_multiply_fp32 (gemm.rs:16-113): f32 products, no TF32
    rounding, so it agrees with the float64 product to f32 summation error
    (far tighter than TF32's 5e-3) and matches the oracle's f32 GEMM."""
    A, B = operands(rng, M, N, Kd, 0, 0)
    out = torch.empty((M, N), device="cuda")
    K.matrix_multiply_fp32(dev(A), dev(B), out)
    got = host(out)
    assert rel_err(got, exact(A, B, 0, 0)) < 1e-5
    assert rel_err(got, O.gemm(A, B)) < 1e-5


@pytest.mark.parametrize("at,bt", [(0, 0), (1, 0), (0, 1)])
def test_wide_tiles_many_per_pair(K, at, bt):
    """Long K and enough 256 x 512 tiles that every CTA pair runs several:
    the automatic choice takes the wide tile here, and each pair reuses its
    single TMEM accumulator from tile to tile. Also the same product with
    the 256 x 256 tile forced, which must agree to rounding. The check is a
    float64 product on the GPU."""
    g = torch.Generator(device="cuda").manual_seed(11)
    M, N, Kd = 4096, 4096 + 64, 2048
    A = torch.randn((Kd, M) if at else (M, Kd), device="cuda", generator=g)
    B = torch.randn((N, Kd) if bt else (Kd, N), device="cuda", generator=g)
    want = (A.double().T if at else A.double()) @ (B.double().T if bt else B.double())
    scale = want.abs().max().item()
    for variant in (0, 2, 3):
        out = torch.empty((M, N), device="cuda")
        K.gemm(A, B, out, a_trans=bool(at), b_trans=bool(bt), variant=variant)
        err = (out.double() - want).abs().max().item() / scale
        assert err < TF32_TOL, (variant, err)


@pytest.mark.parametrize("M,Kd,variant", [(2048, 512, 3), (16384, 4096, 0)])
@pytest.mark.parametrize("epi", ["residual", "pre_act", "grad_act", "beta", "accumulate"])
def test_wide_tiles_heavy_epilogues(K, epi, M, Kd, variant):
    """Every epilogue that reads an input tile, writes a pre-activation or
    adds into C, on the 256 x 512 pair tile (forced at short K, chosen
    automatically at long K, where 16384 rows give 128 wide tiles for the
    74 CTA pairs): its warps stage through two tiles each. Ragged N (1000)
    leaves the last tile half empty. Checked against a float64 product on
    the GPU, and against the 256 x 256 tile (variant 2)."""
    from oxf import _lib
    g = torch.Generator(device="cuda").manual_seed(13)
    N = 1000
    A = torch.randn((M, Kd), device="cuda", generator=g)
    B = torch.randn((Kd, N), device="cuda", generator=g)
    R = torch.randn((M, N), device="cuda", generator=g)
    X = torch.randn((M, N), device="cuda", generator=g)
    C0 = torch.randn((M, N), device="cuda", generator=g)
    prod = A.double() @ B.double()
    scale = prod.abs().max().item()
    outs = {}
    for v in (variant, 2):
        out = C0.clone()
        pre = torch.empty((M, N), device="cuda")
        if epi == "residual":
            K.gemm(A, B, out, residual=R, variant=v)
            want = prod + R.double()
        elif epi == "pre_act":
            K.gemm(A, B, out, pre_out=pre, act=_lib.ACT_GELU, variant=v)
            want = torch.from_numpy(O.act_forward(O.GELU, prod.float().cpu().numpy())).cuda()
            err = (pre.double() - prod).abs().max().item() / scale
            assert err < TF32_TOL, (v, "pre", err)
        elif epi == "grad_act":
            K.gemm(A, B, out, aux=X, grad_act=_lib.ACT_GELU, variant=v)
            d = torch.from_numpy(O.act_derivative(O.GELU, X.cpu().numpy())).cuda()
            want = prod * d.double()
        elif epi == "beta":
            K.gemm(A, B, out, beta=0.5, variant=v)
            want = prod + 0.5 * C0.double()
        else:
            K.gemm(A, B, out, accumulate=True, variant=v)
            want = prod + C0.double()
        err = (out.double() - want.double()).abs().max().item() / scale
        assert err < TF32_TOL, (v, err)
        outs[v] = out
    assert (outs[variant] - outs[2]).abs().max().item() <= 2 * TF32_TOL * scale
    assert K.device_error() == 0


@pytest.mark.parametrize("at,bt", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("M,N,Kd,batch", [(256, 64, 128, 1), (36, 52, 200, 1), (20, 28, 4, 1),
                                          (68, 36, 256, 3)])
def test_small_products_latency_kernel(K, rng, M, N, Kd, batch, at, bt):
    """Products of at most 2^22 multiply-adds with K <= 256 run on the
    one-round-trip CUDA-core kernel: TF32-rounded (RNA) operands, f32
    accumulation, any operand layout, ragged tiles (sizes not multiples of
    16, leading dimensions multiples of 4), batches."""
    A, B = operands(rng, M, N, Kd, at, bt, batch=batch if batch > 1 else None)
    out = torch.empty((batch, M, N) if batch > 1 else (M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, a_trans=bool(at), b_trans=bool(bt))
    got = host(out)
    if batch > 1:
        for b in range(batch):
            assert rel_err(got[b], exact(A[b], B[b], at, bt)) < TF32_TOL
    else:
        assert rel_err(got, exact(A, B, at, bt)) < TF32_TOL


def test_small_products_match_reference_rounding_and_epilogue(K, rng):
    """Config 1 (256x128 · 128x64) against the oracle with the reference's
    TF32 RNA operand rounding: equal up to f32 summation order. Then the
    fused epilogue (alpha, beta·C, bias, residual, pre-activation, GELU),
    the activation gradient, and accumulation on the same kernel."""
    x, w = config1_operands()
    y = torch.empty((256, 64), device="cuda")
    K.matrix_multiply(dev(x), dev(w), y)
    want = O.gemm(x, w, rounding=O.GEMM_TF32_RNA)
    assert np.abs(host(y) - want).max() <= 1e-5 * np.abs(want).max()
    M, N, Kd = 96, 80, 64
    A, B = operands(rng, M, N, Kd, 0, 0)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float32)
    R = rng.standard_normal((M, N)).astype(np.float32)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    out, pre = dev(C0), torch.empty((M, N), device="cuda")
    K.gemm(dev(A), dev(B), out, alpha=0.5, beta=0.25, bias=dev(bias), residual=dev(R),
           pre_out=pre, act=1)
    z = 0.5 * exact(A, B, 0, 0) + 0.25 * C0 + bias + R
    assert rel_err(host(pre), z) < TF32_TOL
    assert rel_err(host(out), O.act_forward(O.GELU, z.astype(np.float32))) < TF32_TOL
    X = rng.standard_normal((M, N)).astype(np.float32)
    g = torch.empty((M, N), device="cuda")
    K.gemm(dev(A), dev(B), g, aux=dev(X), grad_act=1)
    want = exact(A, B, 0, 0) * O.act_derivative(O.GELU, X).astype(np.float64)
    assert rel_err(host(g), want) < TF32_TOL
    acc = dev(C0)
    K.gemm(dev(A), dev(B), acc, accumulate=True)
    assert rel_err(host(acc), C0 + exact(A, B, 0, 0)) < TF32_TOL


@pytest.mark.parametrize("M,N,Kd", [(4096, 2048, 512), (2048, 4096, 4096)])
def test_schedules_agree_and_capture(K, monkeypatch, M, N, Kd):
    """Multi-wave products (more tiles than CTA pairs) on the dynamic tile
    schedule (units claimed from a per-stream counter, handed through the
    shared-memory tile queue) and on the static one (OXF_GEMM_SCHEDULE=static)
    give bit-identical outputs: each tile's arithmetic is the same whichever
    CTA computes it. The second shape takes the 256 x 512 tile. A CUDA-graph
    capture of the same product (static schedule under capture) replays to
    the same bits, and the same product launched on two streams at once
    (one counter slot each) is right on both."""
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, Kd, device="cuda", generator=g)
    B = torch.randn(Kd, N, device="cuda", generator=g)
    dyn = torch.empty(M, N, device="cuda")
    K.gemm(A, B, dyn)
    monkeypatch.setenv("OXF_GEMM_SCHEDULE", "static")
    sta = torch.empty(M, N, device="cuda")
    K.gemm(A, B, sta)
    monkeypatch.delenv("OXF_GEMM_SCHEDULE")
    torch.cuda.synchronize()
    assert torch.equal(dyn, sta)
    cap = torch.zeros(M, N, device="cuda")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side), torch.cuda.graph(graph, stream=side):
        K.gemm(A, B, cap, stream=side)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(cap, dyn)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    o1, o2 = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
    s1.wait_stream(torch.cuda.current_stream())
    s2.wait_stream(torch.cuda.current_stream())
    for _ in range(3):
        K.gemm(A, B, o1, stream=s1)
        K.gemm(A, B, o2, stream=s2)
    torch.cuda.synchronize()
    assert torch.equal(o1, dyn) and torch.equal(o2, dyn)
    assert K.device_error() == 0


@pytest.mark.parametrize("at,bt", [(0, 0), (1, 0), (0, 1)])
@pytest.mark.parametrize("M,N,Kd", [(1024, 1024, 1024), (512, 768, 2048), (300, 520, 4096)])
def test_small_plain_products_split_k(K, M, N, Kd, at, bt):
    """Plain products (alpha only) whose 256 x 256 tiles fill under 3/4 of the
    CTA pairs split K: the output is zeroed first and the splits add into it.
    The output starts as garbage here, which must not leak; alpha scales
    every split. A beta != 0 product of the same shape takes the unsplit
    path and must also be right."""
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn((Kd, M) if at else (M, Kd), device="cuda", generator=g)
    B = torch.randn((N, Kd) if bt else (Kd, N), device="cuda", generator=g)
    want = (A.double().T if at else A.double()) @ (B.double().T if bt else B.double())
    scale = want.abs().max().item()
    out = torch.full((M, N), float("nan"), device="cuda")
    K.gemm(A, B, out, a_trans=bool(at), b_trans=bool(bt), alpha=0.5)
    assert ((out.double() - 0.5 * want).abs().max().item() / (0.5 * scale)) < TF32_TOL
    C0 = torch.randn(M, N, device="cuda", generator=g)
    out2 = C0.clone()
    K.gemm(A, B, out2, a_trans=bool(at), b_trans=bool(bt), beta=1.0)
    assert ((out2.double() - want - C0.double()).abs().max().item() / scale) < TF32_TOL
