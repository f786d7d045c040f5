"""Batch data parallelism for the SSM-scan ops (one process per GPU).

The reference has no multi-device code (it runs on one Apple GPU).  On a B200
box the scans shard naturally by batch: every batch row is independent, so
each rank runs the ops on its own rows with no data-path communication.  The
only exchange is the gradient of the parameters all rows share -- for the
Mamba-1 scan dA (dim, dstate), dD (dim) and d delta_bias (dim); for the SSD
scan dA, dD and d dt_bias -- which is summed over ranks with ONE all-reduce on
a flat fp32 bucket (NCCL over NVLink on the B200 box, gloo in the CPU tests).
Per-sample gradients (du, ddelta, dz, dB, dC, ...) stay local.
"""

from __future__ import annotations

import datetime
from typing import Iterable, Sequence

import torch
import torch.distributed as dist

__all__ = ["batch_slice", "shard_batch", "ParamGradBucket", "init_process_group"]


def batch_slice(batch: int, rank: int, world: int) -> slice:
    """Contiguous rows of ``batch`` owned by ``rank``; the first ``batch % world``
    ranks take one extra row."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(batch, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


def shard_batch(tensors: Sequence[torch.Tensor | None], rank: int, world: int,
                batch_dim: int = 0) -> list[torch.Tensor | None]:
    """This rank's rows of every per-sample tensor (``None`` passes through)."""
    out = []
    sl = None
    for t in tensors:
        if t is None:
            out.append(None)
            continue
        if sl is None:
            sl = batch_slice(t.shape[batch_dim], rank, world)
        out.append(t.narrow(batch_dim, sl.start, sl.stop - sl.start))
    return out


class ParamGradBucket:
    """One flat fp32 buffer for the shared-parameter gradients.

    ``reduce(grads)`` copies the gradients into the bucket, sums it over the
    process group with a single all-reduce, and returns views shaped like the
    inputs.  The bucket is allocated once and reused, so the collective is the
    same call every step with no per-step allocation.
    """

    def __init__(self, shapes: Iterable[torch.Size], device, group=None, dtype=torch.float32):
        self.shapes = [torch.Size(s) for s in shapes]
        self.sizes = [int(torch.Size(s).numel()) for s in self.shapes]
        self.buffer = torch.zeros(sum(self.sizes), dtype=dtype, device=device)
        self.group = group

    def reduce(self, grads: Sequence[torch.Tensor], async_op: bool = False):
        if len(grads) != len(self.sizes):
            raise ValueError("gradient count does not match the bucket")
        off = 0
        for g, n in zip(grads, self.sizes):
            if g.numel() != n:
                raise ValueError(f"gradient of {g.numel()} elements for a slot of {n}")
            self.buffer[off:off + n].copy_(g.reshape(-1))
            off += n
        work = None
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            work = dist.all_reduce(self.buffer, op=dist.ReduceOp.SUM, group=self.group,
                                   async_op=async_op)
        views, off = [], 0
        for n, shape in zip(self.sizes, self.shapes):
            views.append(self.buffer[off:off + n].view(shape))
            off += n
        return (views, work) if async_op else views


def init_process_group(backend: str = "nccl", timeout_s: float = 120.0, device_id=None):
    """Process group from the torchrun environment with a finite timeout, so that
    ranks waiting on a rank that failed end with an error instead of hanging."""
    kwargs = dict(backend=backend, timeout=datetime.timedelta(seconds=timeout_s))
    if device_id is not None:
        kwargs["device_id"] = device_id
    dist.init_process_group(**kwargs)
    return dist.get_rank(), dist.get_world_size()
