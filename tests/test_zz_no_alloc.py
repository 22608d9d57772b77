"""The allocation-free 3xTF32 GEMM entry point (oxf_gemm_tf32x3_noalloc).

It exists for callers that cannot call cudaMalloc: plugin hosts that own the
device memory budget through their own allocator, and latency-critical paths
that must not pay for cudaMalloc's implicit synchronisation. Its scratch is
a 16 MiB static device array instead of a caller workspace. This checks,
through the C ABI, that two calls in a row give the same results as the
workspace entry point (oxf_gemm) within the 3xTF32 tolerance, and that a
shape needing more than 16 MiB is refused with an error.

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


def _desc(L, A, B, Cm, at, bt):
    M = A.shape[1] if at else A.shape[0]
    K = A.shape[0] if at else A.shape[1]
    N = B.shape[0] if bt else B.shape[1]
    d = L.GemmDesc()
    L.lib().oxf_gemm_desc_init(C.byref(d), M, N, K, int(at), int(bt), A.data_ptr(), B.data_ptr(),
                               Cm.data_ptr())
    return d


def _with_workspace(L, A, B, at, bt):
    """The existing entry point: oxf_gemm, TF32X3, caller workspace."""
    M = A.shape[1] if at else A.shape[0]
    N = B.shape[0] if bt else B.shape[1]
    out = torch.empty((M, N), device="cuda")
    d = _desc(L, A, B, out, at, bt)
    d.precision = L.PREC_TF32X3
    need = L.lib().oxf_gemm_workspace_size(C.byref(d))
    ws = torch.empty(need // 4 + 64, device="cuda")
    d.workspace, d.workspace_bytes = ws.data_ptr(), need
    L.check(L.lib().oxf_gemm(C.byref(d), None))
    torch.cuda.synchronize()
    return out


def _no_alloc(L, A, B, at, bt):
    M = A.shape[1] if at else A.shape[0]
    N = B.shape[0] if bt else B.shape[1]
    out = torch.empty((M, N), device="cuda")
    d = _desc(L, A, B, out, at, bt)
    L.check(L.lib().oxf_gemm_tf32x3_noalloc(C.byref(d), None))
    torch.cuda.synchronize()
    return out


def test_no_alloc_matches_workspace_entry_point_twice(L):
    g = torch.Generator(device="cuda").manual_seed(7)
    cases = [((384, 512, 256), False, False), ((256, 192, 320), True, False)]
    for (M, N, K), at, bt in cases:  # two calls in a row, different shapes and data
        A = torch.randn((K, M) if at else (M, K), device="cuda", generator=g)
        B = torch.randn((N, K) if bt else (K, N), device="cuda", generator=g)
        got = _no_alloc(L, A, B, at, bt).cpu().numpy()
        want = _with_workspace(L, A, B, at, bt).cpu().numpy()
        err = np.abs(got - want).max() / np.abs(want).max()
        assert err <= TF32X3_TOL, (M, N, K, err)
        exact = ((A.double().T if at else A.double()) @ (B.double().T if bt else B.double()))
        err_exact = np.abs(got - exact.cpu().numpy()).max() / exact.abs().max().item()
        assert err_exact <= TF32X3_TOL, (M, N, K, err_exact)


def test_no_alloc_rejects_shapes_beyond_its_scratch(L):
    # 2 * (M*K + K*N) * 4 bytes of splits: 2048^2 operands need 64 MiB > 16 MiB
    A = torch.zeros((2048, 2048), device="cuda")
    B = torch.zeros((2048, 2048), device="cuda")
    out = torch.empty((2048, 2048), device="cuda")
    d = _desc(L, A, B, out, False, False)
    st = L.lib().oxf_gemm_tf32x3_noalloc(C.byref(d), None)
    assert st == L.UNSUPPORTED_SHAPE
    assert b"16 MiB" in L.lib().oxf_last_error_string()
