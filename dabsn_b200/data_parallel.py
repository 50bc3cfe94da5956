"""Data-parallel gradient averaging over one flat buffer.

The batch shards over ranks with replicated parameters (the reference's data
parallelism, distributed.py:515-580); the only exchange is the gradient
average.  Every parameter's ``.grad`` is a view of one flat FP32 buffer, so a
step zeroes one tensor and averages it with one all-reduce (NCCL over
NVLink on GPUs, gloo on CPU) -- the arithmetic of
``DistributedDataParallel`` without its per-bucket autograd hooks, which cost
more than the exchange itself on sub-millisecond steps.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class FlatGradAllReduce:
    """Owns the flat gradient buffer of ``params`` on ``device``."""

    def __init__(self, params, device, group=None, broadcast_from: int | None = 0):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        dtypes = {p.dtype for p in self.params}
        if dtypes != {torch.float32}:
            raise TypeError(f"flat gradient buffer expects FP32 parameters, got {dtypes}")
        self.flat = torch.zeros(sum(p.numel() for p in self.params), device=device,
                                dtype=torch.float32)
        self.attach()
        if broadcast_from is not None and dist.is_initialized() and dist.get_world_size(group) > 1:
            for p in self.params:
                dist.broadcast(p.data, src=broadcast_from, group=group)

    def attach(self) -> None:
        """(Re)bind every ``.grad`` to its slice of the flat buffer."""
        off = 0
        for p in self.params:
            p.grad = self.flat[off:off + p.numel()].view_as(p)
            off += p.numel()

    def zero(self) -> None:
        self.flat.zero_()

    def all_reduce(self) -> None:
        """Average the gradients over the ranks (no-op on one rank)."""
        if dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=self.group)
