"""The allocation-free 3xTF32 GEMM entry point (oxf_gemm_tf32x3_noalloc).

It exists for callers that cannot call cudaMalloc: plugin hosts that own the
device memory budget through their own allocator, and latency-critical paths
that must not pay for cudaMalloc's implicit synchronisation. Its scratch is
a 16 MiB static device array instead of a caller workspace. This checks,
through the C ABI, that calls in a row give the same results as the
workspace entry point (oxf_gemm) within the 3xTF32 tolerance, on one-CTA and
CTA-pair tiles, batched and NT operands, and a shape needing exactly 16 MiB;
that a shape needing more is refused with an error; that misaligned operands
(no splits) are not limited; and that invalid descriptors get oxf_gemm's
errors.

Named test_zz_* so pytest collects it last.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TF32X3_TOL = 1e-4


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import _lib
    return _lib


def _dims(t):
    return (t.shape[0], t.shape[1], t.shape[2]) if t.dim() == 3 else (1, t.shape[0], t.shape[1])


def _desc(L, A, B, Cm, at, bt):
    """A descriptor for 2-D or batched 3-D operands (a 2-D operand is shared
    by the batch: stride 0); leading dimensions from the tensors' strides."""
    ba, ar, ac = _dims(A)
    bb, _, _ = _dims(B)
    bo, M, N = _dims(Cm)
    K = ar if at else ac
    d = L.GemmDesc()
    L.lib().oxf_gemm_desc_init(C.byref(d), M, N, K, int(at), int(bt), A.data_ptr(), B.data_ptr(),
                               Cm.data_ptr())
    d.batch = max(ba, bb, bo)
    d.lda, d.stride_a = A.stride(-2), (A.stride(0) if A.dim() == 3 else 0)
    d.ldb, d.stride_b = B.stride(-2), (B.stride(0) if B.dim() == 3 else 0)
    d.ldc, d.stride_c = Cm.stride(-2), (Cm.stride(0) if Cm.dim() == 3 else 0)
    return d


def _out(A, B, at, bt):
    ba, ar, ac = _dims(A)
    bb, br, bc = _dims(B)
    M = ac if at else ar
    N = br if bt else bc
    batch = max(ba, bb)
    return torch.empty((batch, M, N) if batch > 1 else (M, N), device="cuda")


def _with_workspace(L, A, B, at, bt):
    """The existing entry point: oxf_gemm, TF32X3, caller workspace."""
    out = _out(A, B, at, bt)
    d = _desc(L, A, B, out, at, bt)
    d.precision = L.PREC_TF32X3
    need = L.lib().oxf_gemm_workspace_size(C.byref(d))
    ws = torch.empty(need // 4 + 64, device="cuda")
    d.workspace, d.workspace_bytes = ws.data_ptr(), need
    L.check(L.lib().oxf_gemm(C.byref(d), None))
    torch.cuda.synchronize()
    return out


def _no_alloc(L, A, B, at, bt):
    out = _out(A, B, at, bt)
    d = _desc(L, A, B, out, at, bt)
    L.check(L.lib().oxf_gemm_tf32x3_noalloc(C.byref(d), None))
    torch.cuda.synchronize()
    return out


def _exact(A, B, at, bt):
    a = A.double().transpose(-1, -2) if at else A.double()
    b = B.double().transpose(-1, -2) if bt else B.double()
    return torch.matmul(a, b)


def _check_against_both(L, A, B, at, bt, label):
    got = _no_alloc(L, A, B, at, bt).cpu().numpy()
    want = _with_workspace(L, A, B, at, bt).cpu().numpy()
    err = np.abs(got - want).max() / np.abs(want).max()
    assert err <= TF32X3_TOL, (label, err)
    exact = _exact(A, B, at, bt)
    err_exact = np.abs(got - exact.cpu().numpy()).max() / exact.abs().max().item()
    assert err_exact <= TF32X3_TOL, (label, err_exact)


def test_no_alloc_matches_workspace_entry_point_twice(L):
    g = torch.Generator(device="cuda").manual_seed(7)
    # one-CTA tiles (NN, TN) and a CTA-pair shape (2048 x 2560 x 256: 80 pair
    # tiles, 9.4 MB of splits); each call follows another on the same scratch
    cases = [((384, 512, 256), False, False), ((256, 192, 320), True, False),
             ((2048, 2560, 256), False, False)]
    for (M, N, K), at, bt in cases:
        A = torch.randn((K, M) if at else (M, K), device="cuda", generator=g)
        B = torch.randn((N, K) if bt else (K, N), device="cuda", generator=g)
        _check_against_both(L, A, B, at, bt, (M, N, K, at, bt))


def test_no_alloc_batched_shared_operand_and_nt(L):
    """A per-batch A ([3, M, K]) against one B shared by the batch (stride 0),
    B given as [N, K] (NT): the batch scales A's splits, not B's."""
    g = torch.Generator(device="cuda").manual_seed(8)
    A = torch.randn((3, 256, 512), device="cuda", generator=g)
    B = torch.randn((384, 512), device="cuda", generator=g)
    _check_against_both(L, A, B, False, True, "batched NT")


def test_no_alloc_limit_is_exact(L):
    """2*(M*K + K*N)*4 bytes of splits (regions rounded to 256 B): M=256,
    K=64, N=32512 needs exactly 16 MiB and runs; N=32516 needs 16 MiB + 2 KiB
    and is refused."""
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn((256, 64), device="cuda", generator=g)
    B = torch.randn((64, 32512), device="cuda", generator=g)
    d = _desc(L, A, B, _out(A, B, False, False), False, False)
    d.precision = L.PREC_TF32X3
    assert L.lib().oxf_gemm_workspace_size(C.byref(d)) == 16 << 20
    _check_against_both(L, A, B, False, False, "exactly 16 MiB")
    B2 = torch.zeros((64, 32516), device="cuda")
    out = _out(A, B2, False, False)
    d = _desc(L, A, B2, out, False, False)
    st = L.lib().oxf_gemm_tf32x3_noalloc(C.byref(d), None)
    assert st == L.UNSUPPORTED_SHAPE
    assert b"16 MiB" in L.lib().oxf_last_error_string()


def test_no_alloc_simt_fallback_has_no_limit(L):
    """A leading dimension that is not a multiple of 4 floats cannot be read
    by TMA: the product runs on the CUDA cores without operand splits, so a
    shape whose nominal split size (50 MB) exceeds the scratch is accepted."""
    g = torch.Generator(device="cuda").manual_seed(10)
    A = torch.randn((512, 4098), device="cuda", generator=g)
    B = torch.randn((4098, 1024), device="cuda", generator=g)
    _check_against_both(L, A, B, False, False, "SIMT fallback")


def test_no_alloc_validates_like_oxf_gemm(L):
    A = torch.zeros((64, 64), device="cuda")
    out = torch.empty((64, 64), device="cuda")
    d = _desc(L, A, A, out, False, False)
    d.M = -1
    assert L.lib().oxf_gemm_tf32x3_noalloc(C.byref(d), None) == L.INVALID_ARG
    assert L.lib().oxf_gemm_tf32x3_noalloc(None, None) == L.INVALID_ARG
    d = _desc(L, A, A, out, False, False)
    d.M = 0  # an empty output is a no-op, as for oxf_gemm
    assert L.lib().oxf_gemm_tf32x3_noalloc(C.byref(d), None) == 0


def test_no_alloc_rejects_shapes_beyond_its_scratch(L):
    # 2 * (M*K + K*N) * 4 bytes of splits: 2048^2 operands need 64 MiB > 16 MiB
    A = torch.zeros((2048, 2048), device="cuda")
    B = torch.zeros((2048, 2048), device="cuda")
    out = torch.empty((2048, 2048), device="cuda")
    d = _desc(L, A, B, out, False, False)
    st = L.lib().oxf_gemm_tf32x3_noalloc(C.byref(d), None)
    assert st == L.UNSUPPORTED_SHAPE
    assert b"16 MiB" in L.lib().oxf_last_error_string()
