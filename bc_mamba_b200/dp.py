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
    """One flat buffer holding the gradients of `params`, all-reduced at once.

    The parameters' .grad tensors are views into the buffer (as DDP's
    gradient-as-bucket-view), so autograd accumulates straight into it and the
    reduction is a single collective with no packing copies.  Call
    `zero_grad()` instead of resetting .grad to None between steps (a None
    grad would make autograd allocate a fresh tensor outside the bucket)."""

    def __init__(self, params: Iterable[torch.Tensor], average: bool = True, group=None,
                 overlap: bool = False):
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
        self._views = []
        off = 0
        for p in self.params:
            n = p.numel()
            v = self.flat[off:off + n].view_as(p)
            if p.grad is not None:
                v.copy_(p.grad)
            p.grad = v
            self._views.append(v)
            off += n
        # overlap: launch the reduction from autograd as soon as every
        # parameter's gradient of this backward has been accumulated, so it
        # runs beside the rest of the backward (e.g. the input-gradient ops)
        self._pending = len(self.params)
        self._armed = overlap
        if overlap:
            for p in self.params:
                p.register_post_accumulate_grad_hook(self._on_accumulated)

    def _on_accumulated(self, p):
        if not self._armed or self._work is not None:
            return
        self._pending -= 1
        if self._pending == 0:
            self.start()

    def zero_grad(self):
        """Zero every gradient (one fill of the bucket) and re-arm the overlap."""
        self._rebind()
        self.flat.zero_()
        self._pending = len(self.params)

    def _rebind(self):
        # a caller that replaced .grad (e.g. set it to None) gets the view back
        for p, v in zip(self.params, self._views):
            if p.grad is None:
                v.zero_()
                p.grad = v
            elif p.grad.data_ptr() != v.data_ptr():
                v.copy_(p.grad)
                p.grad = v

    def start(self):
        """Launch the all-reduce (asynchronous with respect to the host)."""
        world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        if world == 1:
            return self
        self._rebind()
        op = dist.ReduceOp.SUM
        if self.average:
            if dist.get_backend(self.group) == "nccl":
                op = dist.ReduceOp.AVG
            else:
                self.flat.div_(world)
        if self._stream is not None:
            cur = torch.cuda.current_stream(self.flat.device)
            self._stream.wait_stream(cur)
            with torch.cuda.stream(self._stream):
                self._work = dist.all_reduce(self.flat, op=op, group=self.group, async_op=True)
        else:
            self._work = dist.all_reduce(self.flat, op=op, group=self.group, async_op=True)
        return self

    def finish(self):
        """Wait for the reduction (the result is already in .grad); launches it
        first when it has not been launched (no overlap, or some parameter got
        no gradient in this backward)."""
        if self._work is None:
            self.start()
        if self._work is None:
            return
        self._work.wait()
        if self._stream is not None:
            torch.cuda.current_stream(self.flat.device).wait_stream(self._stream)
        self._work = None
