"""The kernel choice of oxf_gemm, through oxf_gemm_plan, without a GPU.

The plan is a pure function of the descriptor and the SM count (148 on
B200), so these tests pin, on CPU, the tile and K-split rule that the GPU
parity tests and the ncu measurements were taken with: each
configuration's products, the small-product paths, and the fallbacks. The
operand pointers only need the alignment TMA asks for; nothing is read.
"""
from __future__ import annotations

import ctypes as C

import pytest

SMS = 148
ALIGNED = 1 << 20  # a 16-byte aligned fake address: the plan never dereferences it


@pytest.fixture(scope="module")
def L():
    from oxf import _lib
    _lib.lib()
    return _lib


def plan(L, M, N, K, a_trans=False, b_trans=False, batch=1, reduce=False, accumulate=False,
         bias=False, residual=False, pre_out=False, aux=False, act=None, precision=None,
         variant=0, lda=None, sms=SMS):
    d = L.GemmDesc()
    L.lib().oxf_gemm_desc_init(C.byref(d), M, N, K, int(a_trans), int(b_trans), ALIGNED,
                               ALIGNED, ALIGNED)
    d.batch = batch
    if batch > 1:
        d.stride_b = K * N
        if not reduce:
            d.stride_c = M * N
        if reduce:
            d.stride_a = M * K
    if lda is not None:
        d.lda = lda
    d.reduce_batch = int(reduce)
    d.accumulate = int(accumulate)
    if bias:
        d.bias = ALIGNED
    if residual:
        d.residual, d.ldr = ALIGNED, N
    if pre_out:
        d.pre_out, d.ldp = ALIGNED, N
    if aux:
        d.aux, d.ldx = ALIGNED, N
        d.grad_act = L.ACT_GELU
    if act is not None:
        d.act = act
    if precision is not None:
        d.precision = precision
    d.variant = variant
    out = L.GemmPlanInfo()
    L.check(L.lib().oxf_gemm_plan(C.byref(d), sms, C.byref(out)))
    return out


def kernel(p):
    return (p.path, p.tile_m, p.tile_n, p.stages, p.staging)


PAIR, ONE = 4, 3


def test_config5_training_products(L):
    """One 128-sequence step (131072 tokens, hidden 2048, FFN 8192): the
    long-K products take 256 x 512 pair tiles, FFN1 and dZ1 (short K with a
    heavy epilogue) and P.V keep the 256-wide tile's two accumulators."""
    T, S, H, F = 131072, 1024, 2048, 8192
    g = L.ACT_GELU
    assert kernel(plan(L, T, H, F, residual=True)) == (PAIR, 256, 512, 3, 2)       # FFN2
    assert kernel(plan(L, T, F, H, pre_out=True, act=g)) == (PAIR, 256, 256, 6, 1)  # FFN1
    assert kernel(plan(L, T, F, H, b_trans=True, aux=True)) == (PAIR, 256, 256, 6, 1)  # dZ1
    assert kernel(plan(L, T, H, H)) == (PAIR, 256, 512, 3, 2)                        # y (K<4096)
    assert kernel(plan(L, S, H, S, batch=128, residual=True)) == (PAIR, 256, 256, 6, 1)  # P.V
    dw1 = plan(L, H, F, T, a_trans=True, accumulate=True)
    assert kernel(dw1) == (PAIR, 256, 512, 3, 2) and dw1.splits == 15 and dw1.units == 1920


def test_config4_inference_products(L):
    """64 sequences x 2048 tokens, hidden 1024, FFN 4096: as in the config-4
    launch list, P.V + residual and FFN1 (GELU, K = 1024) stay on the 256-wide
    tile, everything else takes the 256 x 512 tile with two staging tiles."""
    T, S, H, F = 131072, 2048, 1024, 4096
    wide2 = (PAIR, 256, 512, 3, 2)
    assert kernel(plan(L, T, H, H)) == wide2                                   # Q|K|V, y
    assert kernel(plan(L, S, S, H, b_trans=True, batch=64)) == wide2           # scores
    assert kernel(plan(L, S, H, S, batch=64, residual=True)) == (PAIR, 256, 256, 6, 1)
    assert kernel(plan(L, T, F, H, act=L.ACT_GELU)) == (PAIR, 256, 256, 6, 1)  # FFN1
    assert kernel(plan(L, T, H, F, residual=True)) == wide2                    # FFN2


def test_one_rank_share_at_eight_gpus(L):
    """16 sequences of config 5 (one rank's share at N = 8)."""
    t = 16384
    dwo = plan(L, 2048, 2048, t, a_trans=True, accumulate=True)
    assert (dwo.tile_n, dwo.splits, dwo.units) == (512, 9, 288)
    dw2 = plan(L, 8192, 2048, t, a_trans=True, accumulate=True)
    assert (dw2.tile_n, dw2.splits, dw2.units) == (512, 4, 512)
    assert kernel(plan(L, t, 8192, 2048, pre_out=True, act=L.ACT_GELU)) == (PAIR, 256, 256, 6, 1)


def test_k_split_products_compare_estimated_times(L):
    """Weight gradients take wide tiles with few splits where the 256 tile
    would need several times more (config 3; one rank's share at N = 8)."""
    c3_dw2 = plan(L, 4096, 1024, 8192, a_trans=True, accumulate=True)
    assert kernel(c3_dw2) == (PAIR, 256, 512, 3, 2) and c3_dw2.splits == 2
    assert c3_dw2.units == 64
    dwqkv16 = plan(L, 2048, 2048, 16384, a_trans=True, accumulate=True, batch=3)
    assert (dwqkv16.tile_n, dwqkv16.splits, dwqkv16.units) == (512, 3, 288)
    # an accumulation with a bias is never split (the bias would be added per split)
    assert plan(L, 2048, 2048, 16384, a_trans=True, accumulate=True, bias=True).splits == 1


def test_config3_residual_products_fill_a_partial_wave(L):
    """64 wide tiles on 74 pairs (0.86 of a wave) against 128 narrow ones in
    1.73 waves: the wide tile."""
    ffn2 = plan(L, 8192, 1024, 4096, residual=True, bias=True)
    assert kernel(ffn2) == (PAIR, 256, 512, 3, 2) and ffn2.units == 64
    ffn1 = plan(L, 8192, 4096, 1024, pre_out=True, act=L.ACT_GELU, bias=True)
    assert kernel(ffn1) == (PAIR, 256, 256, 6, 1)


def test_square_sweep(L):
    p8 = plan(L, 8192, 8192, 8192)
    assert kernel(p8) == (PAIR, 256, 512, 4, 1) and p8.group_m == 1  # 16 tile columns
    assert kernel(plan(L, 2048, 2048, 2048))[:3] == (PAIR, 256, 256)
    p1 = plan(L, 1024, 1024, 1024)  # too few tiles: K split into a zeroed C
    assert p1.path == PAIR and p1.zero_c == 1 and p1.splits == 4
    p5 = plan(L, 512, 512, 512)  # half a wave of one-CTA 128 x 64 tiles
    assert kernel(p5)[:3] == (ONE, 128, 64) and p5.splits == 2 and p5.zero_c == 1


def test_small_and_fallback_paths(L):
    # config 1: 256 x 64 x 128 runs on the tiny CUDA-core kernel
    assert plan(L, 256, 64, 128).path == L.GEMM_PATH_TINY
    # a leading dimension TMA cannot use: the SIMT kernel
    assert plan(L, 512, 512, 512, lda=514).path == L.GEMM_PATH_SIMT
    assert plan(L, 512, 512, 512, precision=L.PREC_F32).path == L.GEMM_PATH_SIMT
    # empty output: nothing runs
    assert plan(L, 0, 512, 512).path == L.GEMM_PATH_NONE
    # 3xTF32 on the pair with 3 stages of hi+lo tiles
    x3 = plan(L, 8192, 8192, 8192, precision=L.PREC_TF32X3)
    assert kernel(x3) == (PAIR, 256, 256, 3, 1)
    # variants force the tile
    assert kernel(plan(L, 8192, 8192, 8192, variant=1))[:2] == (ONE, 128)
    assert kernel(plan(L, 8192, 8192, 8192, variant=2))[:3] == (PAIR, 256, 256)


def test_measurement_overrides(L, monkeypatch):
    """OXF_GEMM_TILE and OXF_GEMM_GROUP_M, read at every call, change the
    plan as they change the launch (tile width, raster group)."""
    monkeypatch.setenv("OXF_GEMM_TILE", "256")
    assert plan(L, 8192, 8192, 8192).tile_n == 256
    monkeypatch.setenv("OXF_GEMM_TILE", "512")
    assert plan(L, 131072, 8192, 2048, pre_out=True, act=L.ACT_GELU).tile_n == 512
    monkeypatch.delenv("OXF_GEMM_TILE")
    assert plan(L, 131072, 8192, 2048, pre_out=True, act=L.ACT_GELU).group_m == 16
    monkeypatch.setenv("OXF_GEMM_GROUP_M", "4")
    assert plan(L, 131072, 8192, 2048, pre_out=True, act=L.ACT_GELU).group_m == 4


def test_plan_scales_with_sm_count(L):
    """The wave arithmetic follows the SM count it is given: config 3's dW2
    takes 2 K splits on 74 CTA pairs, and 8 on 37 (four waves of 64)."""
    a = plan(L, 4096, 1024, 8192, a_trans=True, accumulate=True, sms=148)
    b = plan(L, 4096, 1024, 8192, a_trans=True, accumulate=True, sms=74)
    assert (a.tile_n, a.splits, a.units) == (512, 2, 64)
    assert (b.tile_n, b.splits, b.units) == (512, 8, 256)


def test_plan_rejects_what_oxf_gemm_rejects(L):
    d = L.GemmDesc()
    L.lib().oxf_gemm_desc_init(C.byref(d), -1, 4, 4, 0, 0, ALIGNED, ALIGNED, ALIGNED)
    out = L.GemmPlanInfo()
    assert L.lib().oxf_gemm_plan(C.byref(d), SMS, C.byref(out)) == L.INVALID_ARG
    assert L.lib().oxf_gemm_plan(None, SMS, C.byref(out)) == L.INVALID_ARG
    L.lib().oxf_gemm_desc_init(C.byref(d), 4, 4, 4, 0, 0, ALIGNED, ALIGNED, ALIGNED)
    assert L.lib().oxf_gemm_plan(C.byref(d), SMS, None) == L.INVALID_ARG


@pytest.mark.gpu
def test_plan_for_the_current_device(L):
    """sm_count 0 plans for the current GPU: on a B200 (148 SMs) it is the
    148-SM plan the tests above pin."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    shapes = [dict(M=131072, N=2048, K=8192, residual=True),
              dict(M=4096, N=1024, K=8192, a_trans=True, accumulate=True),
              dict(M=1024, N=1024, K=1024)]
    for kw in shapes:
        here = plan(L, sms=0, **kw)
        want = plan(L, sms=sms, **kw)
        assert (here.path, here.tile_m, here.tile_n, here.stages, here.staging, here.splits,
                here.units) == (want.path, want.tile_m, want.tile_n, want.stages,
                                want.staging, want.splits, want.units), kw
