"""Data-parallel training of the transformer across the GPUs of one node.

The reference is single-GPU (src/cuda/runtime.rs:34-45) and applies SGD
per sequence inside backward (src/net/linear.rs:350-391). Here a step takes
a global batch of independent sequences, shards it across ranks (one
process per GPU, torch.distributed over NCCL), computes per-rank gradient
sums with the engine, all-reduces them in three buckets (output Linear,
feed-forward, attention + position; cursor order, contiguous) while the
next backward stage runs, and applies one SGD update with the gradient
averaged over the global batch:  W -= lr * (1/B) * sum_b grad_b.
For one sequence this is exactly the reference's update (every weight is
used for dX before it is updated, so deferring the update changes nothing).

With exchange="peer" the bucket all-reduces and the final update are
replaced by the fused peer-memory exchange (oxf/exchange.py): after each
backward stage one kernel per rank pulls its shard of the bucket's
gradients from every GPU over NVLink, updates that shard and pushes it to
every GPU's parameters. The update of each bucket then happens as soon as
its gradients are complete (no later stage reads that bucket's weights;
the next forward pass waits for all of them).

The model object only needs the engine interface used below, so the same
driver runs over `gloo` on CPU in tests with a host stand-in model.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def world() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def shard(global_batch: int, rank: int, world_size: int) -> tuple[int, int]:
    """[start, stop) of the sequences rank `rank` owns: contiguous, equal
    shares (global_batch must divide evenly so every rank runs the same
    collective schedule)."""
    if global_batch % world_size:
        raise ValueError(f"global batch {global_batch} does not divide over {world_size} ranks")
    per = global_batch // world_size
    return rank * per, (rank + 1) * per


class DataParallelTrainer:
    """SGD on the mean gradient of a sharded global batch.

    model: an engine with train_forward(x), set_target(t) -> row losses,
    scaled_loss_sum(scale) -> one-element tensor, backward_stage(s),
    bucket(s) -> (offset, count), grads (flat tensor), zero_grads(), sgd(lr).
    """

    STAGES = (0, 1, 2)

    EXCHANGES = ("nccl", "peer")

    def __init__(self, model, global_batch: int, lr: float, seq: int, group=None,
                 overlap: bool = True, exchange: str = "nccl", overlap_blocks: int = 32):
        if exchange not in self.EXCHANGES:
            raise ValueError(f"exchange must be one of {self.EXCHANGES}")
        if exchange == "peer" and not (torch.cuda.is_available()
                                       and getattr(model.params, "is_cuda", False)):
            raise ValueError("exchange='peer' needs a CUDA engine (peer memory over NVLink)")
        self.model = model
        self.exchange = exchange
        self.overlap_blocks = overlap_blocks
        self._peer = None
        self._xstream = None
        self.rank, self.world = world()
        self.global_batch = global_batch
        self.local = shard(global_batch, self.rank, self.world)
        self.local_batch = self.local[1] - self.local[0]
        self.lr = lr
        self.seq = seq
        self.group = group
        self.overlap = overlap

    def broadcast_params(self, params: torch.Tensor) -> None:
        """Every rank starts from rank 0's parameters."""
        if self.world > 1:
            dist.broadcast(params, 0, group=self.group)

    def step(self, x: torch.Tensor, target: torch.Tensor, _before_target=None) -> torch.Tensor:
        """One step on this rank's shard (x, target already on the device,
        [local_batch*seq, width]). Returns the global mean row loss as a
        one-element tensor on the model's device (not synchronised).
        _before_target (internal) runs between the forward pass and the use
        of `target`, e.g. to make the compute stream wait for its copy."""
        if self.exchange == "peer":
            return self._step_peer(x, target, _before_target)
        m = self.model
        m.zero_grads()
        m.train_forward(x)
        if _before_target is not None:
            _before_target()
        m.set_target(target)
        works = []
        for s in self.STAGES:
            m.backward_stage(s)
            if self.world > 1:
                off, cnt = m.bucket(s)
                bucket = m.grads[off:off + cnt]
                if self.overlap:
                    works.append(dist.all_reduce(bucket, group=self.group, async_op=True))
                else:
                    dist.all_reduce(bucket, group=self.group)
        # this rank's share of the global mean row loss, then summed over ranks
        loss = m.scaled_loss_sum(1.0 / (self.global_batch * self.seq))
        if self.world > 1:
            works.append(dist.all_reduce(loss, group=self.group, async_op=self.overlap))
            for w in works:
                if w is not None:
                    w.wait()
        m.sgd(self.lr / self.global_batch)
        return loss

    def _step_peer(self, x, target, _before_target):
        """step() with the fused exchange: every bucket's kernel runs on one
        side stream (so a rank's exchanges never overlap one another), each
        after its backward stage; the compute stream waits for the last."""
        from .exchange import PeerExchange

        m = self.model
        compute = torch.cuda.current_stream()
        if self._peer is None:
            self._peer = PeerExchange(m.params, m.grads, group=self.group)
            self._xstream = torch.cuda.Stream(device=compute.device)
        xs = self._xstream
        lr = self.lr / self.global_batch
        m.zero_grads()
        m.train_forward(x)
        if _before_target is not None:
            _before_target()
        m.set_target(target)
        last = self.STAGES[-1]
        for s in self.STAGES:
            m.backward_stage(s)
            if not self.overlap:
                continue
            off, cnt = m.bucket(s)
            xs.wait_stream(compute)
            # Buckets that overlap later backward stages use few CTAs; the
            # last one has the GPU to itself.
            self._peer.step(off, cnt, lr, blocks=0 if s == last else self.overlap_blocks,
                            stream=xs)
        if not self.overlap:
            # One exchange over the whole arena once backward is done: no
            # exchange CTA shares the GPU with a backward GEMM.
            xs.wait_stream(compute)
            self._peer.step(0, m.grads.numel(), lr, blocks=0, stream=xs)
        loss = m.scaled_loss_sum(1.0 / (self.global_batch * self.seq))
        if self.world > 1:
            dist.all_reduce(loss, group=self.group)
        compute.wait_stream(xs)
        return loss

    def save_checkpoint(self, path, cfg) -> None:
        """Checkpoint v1 (the reference's TOML + little-endian f32 files,
        src/net/checkpoint/model.rs:138-148) of the model's parameters,
        described by `cfg` (models.TransformerConfig). Every rank holds the
        same parameters after a step, so rank 0 alone writes. Collective:
        every rank returns once the files are complete."""
        from .checkpoint import dump_transformer_params
        err = None
        if self.rank == 0:
            try:
                dump_transformer_params(path, cfg, self.model.params.detach().cpu().numpy())
            except Exception as ex:  # reported on every rank below
                err = ex
        self._agree(err is None, err, "rank 0 could not write the checkpoint")

    def load_checkpoint(self, path, cfg) -> None:
        """Rank 0 reads checkpoint v1 files (model.rs:150-172, with every
        validation of the format), refuses them unless they describe `cfg`,
        and every rank receives the parameters by broadcast (no shared file
        system needed). Collective; raises on every rank if rank 0 failed."""
        from .checkpoint import load_transformer_params
        params = self.model.params
        err = None
        if self.rank == 0:
            try:
                got, flat = load_transformer_params(path)
                if got != cfg:
                    raise ValueError(f"checkpoint describes {got}, not {cfg}")
                if flat.size != params.numel():
                    raise ValueError(f"checkpoint holds {flat.size} parameters, the model "
                                     f"{params.numel()}")
                params.copy_(torch.from_numpy(flat).to(params.device))
            except Exception as ex:  # reported on every rank below
                err = ex
        self._agree(err is None, err, "rank 0 could not load the checkpoint")
        self.broadcast_params(params)

    def _agree(self, ok: bool, err, message: str) -> None:
        """Rank 0's outcome, shared with every rank (raises on all of them)."""
        if self.world > 1:
            dev = self.model.params.device
            flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
            dist.broadcast(flag, 0, group=self.group)
            ok = bool(flag.item())
        if not ok:
            raise err if err is not None else RuntimeError(message)

    def close(self) -> None:
        """Releases the peer exchange (collective when exchange='peer')."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    def run_host(self, batches, stream: torch.cuda.Stream | None = None) -> list[float]:
        """Steps over host-resident batches, one step per (x, target) pair
        of pinned CPU tensors ([local_batch*seq, width] each). The inputs of
        step i+1 are copied host->device on a side stream while step i
        computes (two device buffer pairs); within a step the forward pass
        waits only for x, and the target's copy overlaps it. Each step's
        mean loss is copied back and read when the following step has been
        queued. Returns the losses in step order."""
        compute = stream or torch.cuda.current_stream()
        copy = torch.cuda.Stream(device=compute.device)
        bufs, ready, ready_t, free = [], [], [], []
        losses, pending = [], []
        lh = [torch.empty(1, pin_memory=True) for _ in range(2)]
        lev = [torch.cuda.Event() for _ in range(2)]

        def stage(i, xh, th):
            k = i % 2
            if len(bufs) <= k:
                bufs.append((torch.empty(xh.shape, device=compute.device),
                             torch.empty(th.shape, device=compute.device)))
                ready.append(torch.cuda.Event())
                ready_t.append(torch.cuda.Event())
                free.append(None)
            with torch.cuda.stream(copy):
                if free[k] is not None:
                    copy.wait_event(free[k])  # step i-2 is done with this pair
                bufs[k][0].copy_(xh, non_blocking=True)
                ready[k].record(copy)
                bufs[k][1].copy_(th, non_blocking=True)
                ready_t[k].record(copy)

        it = iter(batches)
        nxt = next(it, None)
        if nxt is None:
            return losses
        stage(0, *nxt)
        i = 0
        while nxt is not None:
            k = i % 2
            compute.wait_event(ready[k])
            with torch.cuda.stream(compute):
                loss = self.step(*bufs[k],
                                 _before_target=lambda k=k: compute.wait_event(ready_t[k]))
                ev = torch.cuda.Event()
                ev.record(compute)
                free[k] = ev
                lh[k].copy_(loss, non_blocking=True)
                lev[k].record(compute)
            nxt = next(it, None)
            if nxt is not None:
                stage(i + 1, *nxt)
            if pending:
                j, kk = pending.pop()
                lev[kk].synchronize()
                losses.append(float(lh[kk].item()))
            pending.append((i, k))
            i += 1
        for j, kk in pending:
            lev[kk].synchronize()
            losses.append(float(lh[kk].item()))
        return losses
