"""Batch-sharded data parallelism for the event path.

Every (batch, feature) channel is independent through extract -> scan ->
restore, so each rank runs the whole pipeline on its own batch shard with no
exchange; the only collective is one all-reduce of the parameter gradients
the path produces (A / A_log, W_B/W_C or W_BC, D, dt_idle/dt_active or the
softplus parameters).  They are flattened into a single contiguous bucket
(tens of KB per block, so one latency-bound collective) and reduced on a side
stream so the reduction can overlap whatever work the caller still has
queued on the compute stream.  The reference has no distributed code; its
only multi-GPU path is single-process nn.DataParallel on <= 2 GPUs
(spike_mamba/lra_impl.py:1750-1762).
"""
from __future__ import annotations

import datetime
import os
from typing import Iterable, List, Optional

import torch
import torch.distributed as dist


def shard_range(n: int, rank: int, world: int):
    """Contiguous [start, stop) of n items for `rank` (sizes differ by <= 1)."""
    base, rem = divmod(n, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def init_from_env(backend: Optional[str] = None, timeout_s: float = 120.0) -> tuple:
    """Initialise the default process group from torchrun's environment.

    Returns (rank, world_size, local_rank).  Single-process runs need no
    group and return (0, 1, 0)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local


class GradBucket:
    """One flat buffer holding the gradients of `params`, all-reduced at once."""

    def __init__(self, params: Iterable[torch.Tensor], average: bool = True, group=None):
        self.params: List[torch.Tensor] = [p for p in params]
        if not self.params:
            raise ValueError("GradBucket needs at least one parameter")
        dev = self.params[0].device
        dts = {p.dtype for p in self.params}
        if len(dts) != 1:
            raise ValueError(f"GradBucket parameters must share one dtype, got {dts}")
        self.numel = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(self.numel, dtype=self.params[0].dtype, device=dev)
        self.average = average
        self.group = group
        self._stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        self._work = None

    def _pack(self):
        off = 0
        for p in self.params:
            n = p.numel()
            if p.grad is None:
                self.flat[off:off + n].zero_()
            else:
                self.flat[off:off + n].copy_(p.grad.reshape(-1))
            off += n

    def _unpack(self):
        off = 0
        for p in self.params:
            n = p.numel()
            v = self.flat[off:off + n].view_as(p)
            if p.grad is None:
                p.grad = v.clone()
            else:
                p.grad.copy_(v)
            off += n

    def start(self):
        """Pack and launch the all-reduce (asynchronous with respect to the host)."""
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        if world == 1:
            return self
        if self._stream is not None:
            cur = torch.cuda.current_stream(self.flat.device)
            self._stream.wait_stream(cur)
            with torch.cuda.stream(self._stream):
                self._pack()
                if self.average:
                    self.flat.div_(world)
                self._work = dist.all_reduce(self.flat, group=self.group, async_op=True)
        else:
            self._pack()
            if self.average:
                self.flat.div_(world)
            self._work = dist.all_reduce(self.flat, group=self.group, async_op=True)
        return self

    def finish(self):
        """Wait for the reduction and write the result back into .grad."""
        if self._work is None:
            return
        self._work.wait()
        if self._stream is not None:
            torch.cuda.current_stream(self.flat.device).wait_stream(self._stream)
        self._unpack()
        self._work = None
