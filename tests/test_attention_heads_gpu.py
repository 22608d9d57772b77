"""The fused multi-head attention kernel (oxf_attention_heads_forward)
against the oracle's per-head restatement (oxo_attention_forward_heads):
out = residual + softmax(Q_j K_jᵀ / sqrt(w)) V_j in each head's columns.

The kernel multiplies in TF32 (operands truncated to 10 mantissa bits, as
the GEMMs do) and accumulates the softmax online in f32; the oracle
truncates its products' operands the same way (GEMM_TF32_RZ). Tolerance
5e-3 of the output scale, the TF32 bound.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 5e-3


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import kernels
    yield kernels
    assert kernels.device_error() == 0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy().copy()


CASES = [
    # batch, seq, d, heads (head width d / heads)
    (2, 256, 128, 2),   # 64-wide heads, two query tiles
    (3, 384, 128, 4),   # 32-wide heads, three query tiles
    (1, 128, 64, 1),    # one head, one tile
    (2, 512, 1024, 16),  # config 4's width with 16 heads
]


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("batch,seq,d,heads", CASES)
def test_fused_heads_match_oracle(K, batch, seq, d, heads, causal):
    rng = np.random.default_rng(seq + heads + int(causal))
    q = rng.standard_normal((batch, seq, d)).astype(np.float32)
    k = rng.standard_normal((batch, seq, d)).astype(np.float32)
    v = rng.standard_normal((batch, seq, d)).astype(np.float32)
    res = rng.standard_normal((batch, seq, d)).astype(np.float32)
    out = torch.full((batch, seq, d), float("nan"), device="cuda")
    K.attention_heads_forward(dev(q), dev(k), dev(v), out, heads, residual=dev(res),
                              causal=causal)
    got = host(out)
    for b in range(batch):
        att, _ = O.attention_heads(q[b], k[b], v[b], heads, causal, rounding=O.GEMM_TF32_RZ)
        assert rel_err(got[b], att + res[b]) < TOL, b


def test_fused_heads_without_residual_and_large_logits(K):
    """No residual; logits of order 100 (the online maximum must rescale
    the running output as it grows)."""
    rng = np.random.default_rng(7)
    batch, seq, d, heads = 2, 384, 128, 2
    q = (10 * rng.standard_normal((batch, seq, d))).astype(np.float32)
    k = (10 * rng.standard_normal((batch, seq, d))).astype(np.float32)
    v = rng.standard_normal((batch, seq, d)).astype(np.float32)
    out = torch.empty((batch, seq, d), device="cuda")
    K.attention_heads_forward(dev(q), dev(k), dev(v), out, heads)
    got = host(out)
    assert np.isfinite(got).all()
    for b in range(batch):
        att, _ = O.attention_heads(q[b], k[b], v[b], heads, False, rounding=O.GEMM_TF32_RZ)
        assert rel_err(got[b], att) < TOL


def test_fused_heads_refuses_unsupported_shapes(K):
    from oxf import _lib
    z = lambda *s: torch.zeros(s, device="cuda")
    # seq not a multiple of 128, head width 48, unequal query / value widths
    for (seq, dq, dv, heads) in [(200, 128, 128, 2), (128, 96, 96, 2), (128, 128, 64, 2)]:
        with pytest.raises(_lib.OxfError) as e:
            K.attention_heads_forward(z(1, seq, dq), z(1, seq, dq), z(1, seq, dv), z(1, seq, dv),
                                      heads)
        assert e.value.status == _lib.UNSUPPORTED_SHAPE
    with pytest.raises(_lib.OxfError) as e:  # heads must divide the widths
        K.attention_heads_forward(z(1, 128, 128), z(1, 128, 128), z(1, 128, 128),
                                  z(1, 128, 128), 3)
    assert e.value.status == _lib.INVALID_ARG
