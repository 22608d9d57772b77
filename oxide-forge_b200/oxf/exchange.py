"""Fused gradient exchange + SGD across the GPUs of one node (liboxf.so).

`PeerExchange` is this process's side of `oxf_exchange_*` (include/oxf_host.h):
it exports its parameter arena, gradient arena and signal pad as CUDA IPC
handles, gathers every rank's handles over torch.distributed (host plumbing
only), maps them, and then launches one kernel per gradient bucket that
reads the bucket's gradients from every rank over NVLink, applies
    p -= lr * (g_0 + g_1 + ... + g_{world-1})
to the shard this rank owns, and stores the result into every rank's
parameter arena. It replaces "all-reduce the bucket, then SGD" in
`DataParallelTrainer` (exchange="peer"). There is no reference counterpart:
the reference trains on one GPU (src/cuda/runtime.rs:34-45) with the update
of Linear::learn (src/net/linear.rs:373-391).
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, lib


def _rank_world() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


class PeerExchange:
    """Maps every rank's arenas; `step` runs the fused exchange + SGD.

    params, grads: this rank's flat f32 CUDA arenas of equal length (the
    engine's, in cursor order). Collective: every rank constructs it at the
    same point, with the same arena length.
    """

    def __init__(self, params: torch.Tensor, grads: torch.Tensor, group=None,
                 timeout_us: int = 0):
        if not (params.is_cuda and grads.is_cuda):
            raise ValueError("PeerExchange needs CUDA arenas")
        if params.numel() != grads.numel():
            raise ValueError("parameter and gradient arenas differ in length")
        self.rank, self.world = _rank_world()
        if self.world > _lib.EXCHANGE_MAX_RANKS:
            raise ValueError(f"at most {_lib.EXCHANGE_MAX_RANKS} ranks")
        self.group = group
        self.count = params.numel()
        self._keep = (params, grads)
        self._h = None
        h = C.c_void_p()
        check(lib().oxf_exchange_create(self.rank, self.world, params.data_ptr(),
                                        grads.data_ptr(), self.count, C.byref(h)))
        self._h = h
        if timeout_us:
            check(lib().oxf_exchange_set_timeout(h, int(timeout_us)))
        if self.world > 1:
            mine = (_lib.IpcHandle * 3)()
            check(lib().oxf_exchange_handles(h, mine))
            blobs: list = [None] * self.world
            dist.all_gather_object(blobs, bytes(mine), group=group)
            every = (_lib.IpcHandle * (3 * self.world)).from_buffer_copy(b"".join(blobs))
            check(lib().oxf_exchange_connect(h, every))
            dist.barrier(group=group)  # every rank mapped before anyone signals

    def step(self, offset: int, count: int, lr: float, blocks: int = 0,
             stream: torch.cuda.Stream | None = None) -> None:
        """The fused exchange + SGD over [offset, offset+count) on `stream`
        (default: the current stream). Same arguments, same order, every rank."""
        s = stream or torch.cuda.current_stream()
        check(lib().oxf_exchange_step(self._h, int(offset), int(count), float(lr), int(blocks),
                                      C.c_void_p(s.cuda_stream)))

    def set_timeout(self, timeout_us: int) -> None:
        check(lib().oxf_exchange_set_timeout(self._h, int(timeout_us)))

    def close(self) -> None:
        """Collective: waits for this rank's work, then for every rank, before
        unmapping (no peer may still be reading or writing this memory)."""
        if self._h is None:
            return
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier(group=self.group)
        check(lib().oxf_exchange_destroy(self._h))
        self._h = None
