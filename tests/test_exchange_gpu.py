"""Fused gradient exchange + SGD (oxf_exchange_sgd, oxf/exchange.py) on the GPU.

One GPU: world 1 equals oxf_sgd_update bit for bit on ragged ranges and the
CPU oracle; a barrier wait that nothing completes expires into the device
error word without touching memory, and the context stays usable; the
data-parallel trainer's peer path equals its NCCL path at world 1.
Two GPUs (skipped with fewer): every rank ends with bit-identical
parameters equal to the oracle's, over ragged ranges; the trainer's peer
path matches its NCCL path and keeps the ranks in lockstep.
"""
from __future__ import annotations

import ctypes as C
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
sys.path.insert(0, str(ROOT / "oracle"))

import oracle as O  # noqa: E402

RANGES = [(0, 1), (1, 10), (5, 3), (2, 4), (3, 1), (7, 1000), (4096, 65536 + 3)]


def _ulp_diff(a: np.ndarray, b: np.ndarray) -> int:
    ia = a.view(np.int32).astype(np.int64)
    ib = b.view(np.int32).astype(np.int64)
    return int(np.abs(ia - ib).max()) if a.size else 0


def _desc(world, rank, params, grads, pads, timeout_us=0, blocks=0, epoch=1):
    from oxf import _lib
    d = _lib.ExchangeDesc()
    d.rank, d.world = rank, world
    for q in range(world):
        d.params[q] = params[q].data_ptr()
        d.grads[q] = grads[q].data_ptr()
        d.signals[q] = pads[q].data_ptr()
    d.epoch, d.blocks, d.timeout_us = epoch, blocks, timeout_us
    return d


def _pad():
    from oxf import _lib
    return torch.zeros(_lib.EXCHANGE_SIGNAL_BYTES // 4, dtype=torch.int32, device="cuda")


def _device_error() -> int:
    from oxf import _lib
    code = C.c_uint32(0)
    _lib.check(_lib.lib().oxf_device_error(C.byref(code)))
    return code.value


def test_world1_equals_sgd_update_and_oracle():
    from oxf import _lib
    lib = _lib.lib()
    n = 70001
    rng = np.random.default_rng(5)
    p0 = rng.standard_normal(n).astype(np.float32)
    g0 = rng.standard_normal(n).astype(np.float32)
    pad = _pad()
    lr = 0.0123
    for epoch, (off, cnt) in enumerate(RANGES, start=1):
        params = torch.from_numpy(p0).cuda()
        grads = torch.from_numpy(g0).cuda()
        d = _desc(1, 0, [params], [grads], [pad], epoch=epoch)
        _lib.check(lib.oxf_exchange_sgd(C.byref(d), off, cnt, lr, None))
        ref = torch.from_numpy(p0).cuda()
        sl = slice(off, off + cnt)
        _lib.check(lib.oxf_sgd_update(_lib.Slice(ref[sl].data_ptr(), cnt),
                                      _lib.CSlice(grads[sl].data_ptr(), cnt), lr, None))
        got = params.cpu().numpy()
        np.testing.assert_array_equal(got, ref.cpu().numpy())
        want = O.exchange_sgd([p0], [g0], off, cnt, lr)[0]
        assert _ulp_diff(got, want) <= 1, (off, cnt)
        np.testing.assert_array_equal(got[:off], p0[:off])
        np.testing.assert_array_equal(got[off + cnt:], p0[off + cnt:])
    assert _device_error() == 0


def test_argument_checks():
    from oxf import _lib
    lib = _lib.lib()
    p = torch.zeros(16, device="cuda")
    g = torch.zeros(16, device="cuda")
    pad = _pad()
    for kw in ({"epoch": 0}, {"blocks": -1}, {"blocks": _lib.EXCHANGE_MAX_BLOCKS + 1}):
        d = _desc(1, 0, [p], [g], [pad], **kw)
        assert lib.oxf_exchange_sgd(C.byref(d), 0, 16, 0.1, None) == _lib.INVALID_ARG
    d = _desc(1, 0, [p], [g], [pad])
    d.world = 9
    assert lib.oxf_exchange_sgd(C.byref(d), 0, 16, 0.1, None) == _lib.INVALID_ARG
    d = _desc(1, 0, [p], [g], [pad])
    d.rank = 1
    assert lib.oxf_exchange_sgd(C.byref(d), 0, 16, 0.1, None) == _lib.INVALID_ARG
    d = _desc(1, 0, [p], [g], [pad])
    d.params[0] = p.data_ptr() + 4  # not 16-byte aligned
    assert lib.oxf_exchange_sgd(C.byref(d), 0, 8, 0.1, None) == _lib.INVALID_ARG
    assert b"aligned" in lib.oxf_last_error_string()


def test_missing_peer_expires_into_error_word():
    """World 2 with only rank 0 launched: the peer's start signal never
    arrives, the bounded wait (20 ms) expires, the kernel records 0x201 and
    returns without touching either rank's parameters; the context stays
    usable. Rank 1's arenas and pad are plain local buffers here (no second
    GPU and no peer mapping): nothing ever sets the awaited flag."""
    from oxf import _lib
    lib = _lib.lib()
    assert _device_error() == 0
    n = 4099
    p = [torch.randn(n, device="cuda") for _ in range(2)]
    g = [torch.randn(n, device="cuda") for _ in range(2)]
    before = [t.clone() for t in p]
    pads = [_pad(), _pad()]
    d = _desc(2, 0, p, g, pads, timeout_us=20000, blocks=4)
    _lib.check(lib.oxf_exchange_sgd(C.byref(d), 0, n, 0.1, None))
    assert _device_error() == _lib.DEVERR_EXCHANGE_START
    for a, b in zip(p, before):
        assert torch.equal(a, b)
    # rank 0 announced itself in the would-be peer's pad
    assert int(pads[1].view(-1)[:_lib.EXCHANGE_MAX_RANKS * 4].max()) == 1
    # the context is usable afterwards
    q = torch.ones(8, device="cuda")
    d1 = _desc(1, 0, [q], [torch.ones(8, device="cuda")], [_pad()])
    _lib.check(lib.oxf_exchange_sgd(C.byref(d1), 0, 8, 0.5, None))
    assert torch.equal(q.cpu(), torch.full((8,), 0.5))
    assert _device_error() == 0


def _small_cfg():
    from oxf import _lib, models
    return models.transformer_config(64, 128, 256, norm=_lib.NORM_LAYER)


def test_trainer_peer_equals_nccl_at_world1():
    from oxf import models
    from oxf.dp import DataParallelTrainer
    cfg = _small_cfg()
    B, S, H = 4, 64, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    xs = [torch.randn(B * S, H, device="cuda", generator=g) for _ in range(3)]
    ts = [torch.randn(B * S, H, device="cuda", generator=g) for _ in range(3)]
    out = {}
    for mode in ("nccl", "peer"):
        m = models.Transformer(cfg, max_batch=B)
        m.set_params(models.init_transformer_params(cfg, seed=0))
        tr = DataParallelTrainer(m, B, 0.05, S, exchange=mode)
        losses = [float(tr.step(x, t)) for x, t in zip(xs, ts)]
        torch.cuda.synchronize()
        out[mode] = (m.get_params(), losses)
        tr.close()
        m.close()
    np.testing.assert_array_equal(out["peer"][0], out["nccl"][0])
    assert out["peer"][1] == out["nccl"][1]
    assert _device_error() == 0


# ------------------------------------------------------------------ 2 GPUs
def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from oxf import _lib, models
    from oxf.dp import DataParallelTrainer
    from oxf.exchange import PeerExchange
    res = {"rank": rank}
    # raw exchange over ragged ranges
    n = 1_000_003
    p0 = np.random.default_rng(7).standard_normal(n).astype(np.float32)
    gr = np.random.default_rng(100 + rank).standard_normal(n).astype(np.float32)
    params = torch.from_numpy(p0).cuda()
    grads = torch.from_numpy(gr).cuda()
    x = PeerExchange(params, grads)
    for off, cnt in RANGES + [(0, n), (123457, 400001)]:
        x.step(off, cnt, 0.01)
    torch.cuda.synchronize()
    code = C.c_uint32(0)
    _lib.check(_lib.lib().oxf_device_error(C.byref(code)))
    res["code"] = code.value
    res["params"] = params.cpu().numpy()
    x.close()
    # the trainer, peer vs NCCL, from the same parameters
    cfg = _small_cfg()
    B, S, H = 4, 64, 128
    for mode in ("peer", "nccl"):
        m = models.Transformer(cfg, max_batch=B // world)
        m.set_params(models.init_transformer_params(cfg, seed=0))
        tr = DataParallelTrainer(m, B, 0.05, S, exchange=mode)
        g = torch.Generator(device="cuda").manual_seed(11 + rank)
        losses = []
        for _ in range(3):
            xx = torch.randn(B // world * S, H, device="cuda", generator=g)
            tt = torch.randn(B // world * S, H, device="cuda", generator=g)
            losses.append(float(tr.step(xx, tt)))
        torch.cuda.synchronize()
        res[f"{mode}_params"] = m.get_params()
        res[f"{mode}_losses"] = losses
        tr.close()
        m.close()
    np.save(Path(out_dir) / f"rank{rank}.npy", res, allow_pickle=True)
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank did not finish")
        assert p.exitcode == 0
    r = [np.load(tmp_path / f"rank{q}.npy", allow_pickle=True).item() for q in range(2)]
    assert r[0]["code"] == 0 and r[1]["code"] == 0
    np.testing.assert_array_equal(r[0]["params"], r[1]["params"])
    n = r[0]["params"].size
    p = [np.random.default_rng(7).standard_normal(n).astype(np.float32)] * 2
    g = [np.random.default_rng(100 + q).standard_normal(n).astype(np.float32) for q in range(2)]
    for off, cnt in RANGES + [(0, n), (123457, 400001)]:
        p = O.exchange_sgd(p, g, off, cnt, 0.01)
    assert _ulp_diff(r[0]["params"], p[0]) <= 1
    # trainer: ranks in lockstep, peer == NCCL within the summation-order tolerance
    np.testing.assert_array_equal(r[0]["peer_params"], r[1]["peer_params"])
    np.testing.assert_array_equal(r[0]["nccl_params"], r[1]["nccl_params"])
    a, b = r[0]["peer_params"], r[0]["nccl_params"]
    assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()
    assert np.allclose(r[0]["peer_losses"], r[0]["nccl_losses"], rtol=1e-5)
