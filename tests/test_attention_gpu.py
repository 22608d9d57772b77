"""Scaled dot-product attention (oxf_attention_forward), in both its forms
(three launches, and the softmax fused into the two products), against the
oracle's unfused restatement
of Attention::forward (src/net/transformer/attention.rs:243-253, 347-401):
scores = Q·Kᵀ, softmax over rows with the scale 1/sqrt(query.cols) and the
decoder's causal mask (row.rs:5-14, 55-113), then P·V plus the residual.
The oracle rounds GEMM operands to TF32 with round-to-nearest-away as the
reference does (gemm.rs:286-347). Tolerance: 5e-3 of max|want| (two chained
TF32 products).
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle as O
from conftest import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
RNA = O.GEMM_TF32_RNA
TOL = 5e-3
F32 = np.float32


@pytest.fixture(scope="module")
def K():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from oxf import kernels
    yield kernels
    assert kernels.device_error() == 0


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a, F32)).cuda()


def oracle_attention(q, k, v, residual, scale, causal):
    out = []
    for b in range(q.shape[0]):
        s = O.gemm(q[b], k[b], b_trans=True, rounding=RNA)
        p = O.softmax_rows(s, scale, q.shape[1] if causal else 0)
        o = O.gemm(p, v[b], rounding=RNA)
        out.append(o + residual[b] if residual is not None else o)
    return np.stack(out)


def run(K, q, k, v, residual, scale, causal):
    batch, seq, _ = q.shape
    out = torch.empty((batch, seq, v.shape[-1]), device="cuda")
    scores = torch.empty((batch, seq, seq), device="cuda")
    stats = torch.empty(K.attention_stats_floats(batch, seq), device="cuda")
    K.attention_forward(dev(q), dev(k), dev(v), out, scores, stats, scale,
                        residual=dev(residual) if residual is not None else None, causal=causal)
    torch.cuda.synchronize()
    return out.cpu().numpy(), scores


CASES = [
    # batch, seq, d_qk, d_v, causal, residual
    (2, 64, 64, 64, False, True),
    (3, 300, 96, 160, False, True),    # ragged keys: 300 = 256 + 44 (partial chunks, blocks)
    (2, 300, 96, 160, True, False),    # decoder mask
    (1, 1024, 128, 256, True, True),
    (2, 2048, 1024, 1024, False, True),  # config 4's per-sequence shape
    (2, 38, 20, 12, False, True),      # rows not 16-byte aligned: the unfused sequence
]


@pytest.fixture(params=["fused", "three-launch"])
def form(request, monkeypatch):
    """Both forms of oxf_attention_forward (OXF_ATTENTION is read at every
    call)."""
    if request.param == "fused":
        monkeypatch.setenv("OXF_ATTENTION", "fused")
    else:
        monkeypatch.delenv("OXF_ATTENTION", raising=False)
    return request.param


@pytest.mark.parametrize("batch,seq,dqk,dv,causal,res", CASES)
def test_attention_matches_oracle(K, form, batch, seq, dqk, dv, causal, res):
    rng = np.random.default_rng(seq * 7 + dqk + int(causal))
    q = rng.standard_normal((batch, seq, dqk)).astype(F32)
    k = rng.standard_normal((batch, seq, dqk)).astype(F32)
    v = rng.standard_normal((batch, seq, dv)).astype(F32)
    r = rng.standard_normal((batch, seq, dv)).astype(F32) if res else None
    scale = 1.0 / np.sqrt(dqk)
    got, _ = run(K, q, k, v, r, scale, causal)
    want = oracle_attention(q, k, v, r, scale, causal)
    assert np.isfinite(got).all()
    assert rel_err(got, want) < TOL


def test_unfused_fallback_leaves_probabilities(K):
    """With rows that TMA cannot read (seq % 4 != 0) the three-launch form
    runs, and the scores workspace then holds the probabilities."""
    rng = np.random.default_rng(5)
    q = rng.standard_normal((1, 38, 20)).astype(F32)
    k = rng.standard_normal((1, 38, 20)).astype(F32)
    v = rng.standard_normal((1, 38, 12)).astype(F32)
    _, scores = run(K, q, k, v, None, 0.25, True)
    p = scores.cpu().numpy()[0]
    s = O.gemm(q[0], k[0], b_trans=True, rounding=RNA)
    assert rel_err(p, O.softmax_rows(s, 0.25, 38)) < TOL
    assert np.all(p[np.triu_indices(38, 1)] == 0.0)


def test_very_negative_logits_and_ragged_keys(K, form):
    """Every logit about -864 (constant rows): the softmax is uniform, and the
    zero-filled keys past a ragged last block must contribute 0, not
    exp(0 - max) = inf against V's zero-filled rows."""
    seq, d = 300, 96
    q = np.full((1, seq, d), 3.0, F32)
    k = np.full((1, seq, d), 3.0, F32)
    v = np.random.default_rng(3).standard_normal((1, seq, 64)).astype(F32)
    got, _ = run(K, q, k, v, None, -1.0, False)
    want = np.broadcast_to(v[0].astype(np.float64).mean(axis=0), (seq, 64))
    assert np.isfinite(got).all()
    assert np.abs(got[0] - want).max() <= TOL * np.abs(want).max()


def test_empty_and_invalid(K):
    from oxf import _lib
    L = _lib.lib()
    assert L.oxf_attention_forward(None, None, None, None, None, None, None, 0, 16, 8, 8, 1.0, 0,
                                   None) == 0
    assert L.oxf_attention_forward(None, None, None, None, None, None, None, 1, 16, 8, 8, 1.0, 0,
                                   None) == _lib.INVALID_ARG
    assert L.oxf_attention_forward(None, None, None, None, None, None, None, -1, 16, 8, 8, 1.0, 0,
                                   None) == _lib.INVALID_ARG
