"""Data-parallel driver (oxf/dp.py) on CPU with world-size-2 gloo ranks.

The engine is replaced by a host stand-in built on the oracle (test-only),
so this checks the driver's own logic: batch sharding, the three bucketed
all-reduces in cursor order, the global-mean SGD update, equality of the
N-rank step with the 1-rank step on the same global batch, and that a rank
which dies, raises or stalls leaves the others with an error within the
process-group timeout instead of a hang.
"""
from __future__ import annotations

import os
import socket
import sys
import time
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
torch = pytest.importorskip("torch")
SEQ, H, F = 8, 12, 20
PG_TIMEOUT_S = 8  # process-group timeout: the bound on a collective that a peer misses


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class OracleModel:
    """Host stand-in with the engine interface DataParallelTrainer uses."""

    def __init__(self, flat: np.ndarray):
        sys.path.insert(0, str(ROOT / "oracle"))
        sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
        import oracle as O
        self.O = O
        self.flat = flat.astype(np.float32).copy()
        self.params = torch.from_numpy(self.flat)
        self.grads = torch.zeros_like(self.params)
        # cursor order: wq, wk, wv, pos, w1, w2, wo
        sizes = [H * H, H * H, H * H, SEQ * H, H * F, F * H, H * H]
        self.offsets = np.cumsum([0] + sizes)

    def _model(self):
        O, f, o = self.O, self.flat, self.offsets
        w = [f[o[i]:o[i + 1]] for i in range(7)]
        lin = lambda a, shape, act=O.IDENTITY: O.LinearParams(a.reshape(shape), None, act)
        return O.TransformerParams(lin(w[0], (H, H)), lin(w[1], (H, H)), lin(w[2], (H, H)),
                                   w[3].reshape(SEQ, H),
                                   O.MlpParams([lin(w[4], (H, F), O.GELU), lin(w[5], (F, H))]),
                                   lin(w[6], (H, H)), O.NORM_LAYER, SEQ)

    def zero_grads(self):
        self.grads.zero_()

    def train_forward(self, x):
        self._x = x.numpy().reshape(-1, SEQ, H)

    def set_target(self, t):
        t = t.numpy().reshape(-1, SEQ, H)
        g = np.zeros_like(self.flat)
        losses = []
        for b in range(self._x.shape[0]):
            _, loss, _ = self.O.transformer_train_step(self._model(), self._x[b], t[b], 0.0,
                                                       grads=g)
            losses.append(loss)
        self.grads += torch.from_numpy(g)
        self._row_loss = torch.from_numpy(np.concatenate(losses))
        return self._row_loss

    def scaled_loss_sum(self, scale):
        return (self._row_loss.sum() * scale).reshape(1)

    def backward_stage(self, s):
        # gradients were produced in set_target; a test may make stage 1 fail
        # after stage 0's bucket all-reduce has been issued
        if s == 1 and getattr(self, "fail_in_backward", False):
            raise RuntimeError("injected failure in backward stage 1")

    def bucket(self, s):
        o = self.offsets
        return {0: (int(o[6]), int(o[7] - o[6])), 1: (int(o[4]), int(o[6] - o[4])),
                2: (0, int(o[4]))}[s]

    def sgd(self, lr):
        self.params -= lr * self.grads  # self.flat shares memory with params


def _data(global_batch, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((global_batch * SEQ, H)).astype(np.float32)
    t = rng.standard_normal((global_batch * SEQ, H)).astype(np.float32)
    return x, t


def _flat0():
    rng = np.random.default_rng(0)
    sizes = [(H, H), (H, H), (H, H), (SEQ, H), (H, F), (F, H), (H, H)]
    parts = [rng.uniform(-0.3, 0.3, s) for s in sizes]
    parts[3] = 0.02 * rng.standard_normal((SEQ, H))
    return np.concatenate([p.ravel() for p in parts]).astype(np.float32)


def _worker(rank, world, port, global_batch, steps, out_dir, fail_rank, fail_mode="exit"):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=PG_TIMEOUT_S))
    sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
    from oxf.dp import DataParallelTrainer
    model = OracleModel(_flat0() if rank == 0 else np.zeros_like(_flat0()))
    tr = DataParallelTrainer(model, global_batch, lr=0.1, seq=SEQ)
    tr.broadcast_params(model.params)
    result = {"rank": rank}
    t0 = time.monotonic()
    try:
        for step in range(steps):
            if rank == fail_rank and step == 1:
                if fail_mode == "exit":
                    os._exit(3)  # this rank dies between steps
                if fail_mode == "raise":
                    model.fail_in_backward = True  # raises inside the step
                if fail_mode == "stall":
                    time.sleep(PG_TIMEOUT_S + 4)  # misses the next collective
            t0 = time.monotonic()
            x, t = _data(global_batch, seed=step)
            lo, hi = tr.local
            sl = slice(lo * SEQ, hi * SEQ)
            loss = tr.step(torch.from_numpy(x[sl]), torch.from_numpy(t[sl]))
            result[f"loss{step}"] = float(loss)
        result["params"] = model.params.numpy().copy()
    except Exception as ex:  # the surviving rank must see an error, not hang
        result["error"] = type(ex).__name__
        result["error_after_s"] = time.monotonic() - t0
    np.save(Path(out_dir) / f"rank{rank}.npy", result, allow_pickle=True)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def _run(world, global_batch, steps, tmp_path, fail_rank=-1, fail_mode="exit"):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, global_batch, steps, str(tmp_path),
                                               fail_rank, fail_mode)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
    out = {}
    for r in range(world):
        f = tmp_path / f"rank{r}.npy"
        if f.exists():
            out[r] = np.load(f, allow_pickle=True).item()
    return out


def test_shard_arithmetic():
    sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
    from oxf.dp import shard
    assert [shard(128, r, 8) for r in range(8)][3] == (48, 64)
    assert shard(6, 1, 2) == (3, 6)
    with pytest.raises(ValueError):
        shard(7, 0, 2)


def test_two_ranks_match_one_rank(tmp_path):
    (tmp_path / "one").mkdir()
    (tmp_path / "two").mkdir()
    one = _run(1, 4, 2, tmp_path / "one")
    two = _run(2, 4, 2, tmp_path / "two")
    p1, p20, p21 = one[0]["params"], two[0]["params"], two[1]["params"]
    np.testing.assert_array_equal(p20, p21)          # ranks stay in lockstep
    assert np.abs(p20 - p1).max() <= 1e-5 * np.abs(p1).max()
    assert abs(two[0]["loss1"] - one[0]["loss1"]) < 1e-5
    assert not np.array_equal(p1, _flat0())          # the steps did update


def test_dead_rank_is_an_error_not_a_hang(tmp_path):
    out = _run(2, 4, 3, tmp_path, fail_rank=1)
    assert 1 not in out                               # rank 1 exited without a result
    assert out[0].get("error"), out[0].keys()        # rank 0 got an error from its collective


def test_raising_rank_is_an_error_not_a_hang(tmp_path):
    """Rank 1 raises inside step 1, after issuing the first bucket's
    all-reduce but not the second. Rank 1 reports its own exception; rank 0's
    next collective ends with an error within the process-group timeout."""
    out = _run(2, 4, 3, tmp_path, fail_rank=1, fail_mode="raise")
    assert out[1].get("error") == "RuntimeError", out[1].keys()
    assert out[0].get("error"), out[0].keys()
    assert out[0]["error_after_s"] < PG_TIMEOUT_S + 10, out[0]["error_after_s"]


def test_stalled_rank_is_an_error_not_a_hang(tmp_path):
    """Rank 1 stalls between steps for longer than the process-group
    timeout. Rank 0's next collective ends with an error within that bound
    instead of waiting for it, and both processes finish."""
    out = _run(2, 4, 3, tmp_path, fail_rank=1, fail_mode="stall")
    assert out[0].get("error"), out[0].keys()
    assert out[0]["error_after_s"] < PG_TIMEOUT_S + 10, out[0]["error_after_s"]
    assert "params" not in out[0]


def test_peer_exchange_needs_cuda_arenas():
    sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
    from oxf.dp import DataParallelTrainer
    model = OracleModel(_flat0())
    with pytest.raises(ValueError):
        DataParallelTrainer(model, 4, lr=0.1, seq=SEQ, exchange="peer")
    with pytest.raises(ValueError):
        DataParallelTrainer(model, 4, lr=0.1, seq=SEQ, exchange="allgather")


def _ckpt_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    sys.path.insert(0, str(ROOT / "oxide-forge_b200"))
    from oxf import _lib, models
    from oxf.dp import DataParallelTrainer
    cfg = models.transformer_config(SEQ, H, F, norm=_lib.NORM_LAYER)
    model = OracleModel(_flat0() if rank == 0 else np.zeros_like(_flat0()))
    tr = DataParallelTrainer(model, 4, lr=0.1, seq=SEQ)
    tr.broadcast_params(model.params)
    x, t = _data(4, seed=0)
    lo, hi = tr.local
    tr.step(torch.from_numpy(x[lo * SEQ:hi * SEQ]), torch.from_numpy(t[lo * SEQ:hi * SEQ]))
    saved = model.params.numpy().copy()
    path = str(Path(out_dir) / "dp_ckpt")
    tr.save_checkpoint(path, cfg)
    model.params.zero_()
    tr.load_checkpoint(path, cfg)
    result = {"rank": rank, "saved": saved, "loaded": model.params.numpy().copy()}
    wrong = models.transformer_config(SEQ, H, F + 4, norm=_lib.NORM_LAYER)
    try:
        tr.load_checkpoint(path, wrong)
        result["wrong"] = "accepted"
    except Exception as ex:
        result["wrong"] = type(ex).__name__
    try:
        tr.load_checkpoint(str(Path(out_dir) / "missing"), cfg)
        result["missing"] = "accepted"
    except Exception as ex:
        result["missing"] = type(ex).__name__
    np.save(Path(out_dir) / f"ckpt{rank}.npy", result, allow_pickle=True)
    dist.destroy_process_group()


def test_dp_checkpoint_save_by_rank0_load_by_broadcast(tmp_path):
    """Checkpoint v1 from a data-parallel run: rank 0 writes the (identical)
    parameters; loading reads them on rank 0, checks them against the model's
    configuration and broadcasts them; a mismatching configuration or a
    missing file is an error on every rank."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_ckpt_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            raise AssertionError("a rank hung")
        assert p.exitcode == 0
    r = [np.load(tmp_path / f"ckpt{q}.npy", allow_pickle=True).item() for q in range(2)]
    np.testing.assert_array_equal(r[0]["saved"], r[1]["saved"])
    for q in range(2):
        np.testing.assert_array_equal(r[q]["loaded"], r[0]["saved"])
        assert r[q]["wrong"] != "accepted" and r[q]["missing"] != "accepted"
    assert (tmp_path / "dp_ckpt.toml").exists() and (tmp_path / "dp_ckpt.bin").exists()
