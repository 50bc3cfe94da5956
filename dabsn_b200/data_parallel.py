"""Data-parallel gradient averaging over one flat buffer.

The batch shards over ranks with replicated parameters (the reference's data
parallelism, distributed.py:515-580); the only exchange is the gradient
average.  Every parameter's ``.grad`` is a view of one flat FP32 buffer, so a
step zeroes one tensor and averages it with all-reduces over contiguous
slices of it (NCCL over NVLink on GPUs, gloo on CPU).

Two schedules:

* one all-reduce of the whole buffer after the backward (``bucket_bytes``
  None): the cheapest on sub-millisecond steps, where per-bucket hooks cost
  more than the exchange;
* buckets (``bucket_bytes`` set): parameters are laid out in reverse
  registration order (roughly the order in which the backward finishes
  them) and cut into contiguous buckets; a post-accumulate hook on each
  parameter launches the asynchronous all-reduce of its bucket as soon as
  every gradient in it is final, so the exchange overlaps the rest of the
  backward (on a long step the model's readout and embedding gradients,
  finished early, cross NVLink while the core scan's reverse runs).
  ``all_reduce()`` launches the buckets no hook launched (parameters
  without a gradient this step) and waits for all of them.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class FlatGradAllReduce:
    """Owns the flat gradient buffer of ``params`` on ``device``."""

    def __init__(self, params, device, group=None, broadcast_from: int | None = 0,
                 bucket_bytes: int | None = None):
        params = [p for p in params if p.requires_grad]
        self.group = group
        dtypes = {p.dtype for p in params}
        if dtypes != {torch.float32}:
            raise TypeError(f"flat gradient buffer expects FP32 parameters, got {dtypes}")
        multi = dist.is_initialized() and dist.get_world_size(group) > 1
        self.overlap = bucket_bytes is not None and multi
        self.params = list(reversed(params)) if self.overlap else params
        self.flat = torch.zeros(sum(p.numel() for p in self.params), device=device,
                                dtype=torch.float32)
        self.attach()
        if broadcast_from is not None and multi:
            for p in self.params:
                dist.broadcast(p.data, src=broadcast_from, group=group)
        self.buckets: list[tuple[int, int, int]] = []  # (start, end, parameters)
        self._works: list = []
        self._pending: list[int] = []
        if self.overlap:
            self._build_buckets(int(bucket_bytes))

    def attach(self) -> None:
        """(Re)bind every ``.grad`` to its slice of the flat buffer."""
        off = 0
        for p in self.params:
            p.grad = self.flat[off:off + p.numel()].view_as(p)
            off += p.numel()

    def _build_buckets(self, bucket_bytes: int) -> None:
        off, start, count = 0, 0, 0
        owner = []
        for p in self.params:
            owner.append(len(self.buckets))
            off += p.numel()
            count += 1
            if (off - start) * 4 >= bucket_bytes:
                self.buckets.append((start, off, count))
                start, count = off, 0
        if count:
            self.buckets.append((start, off, count))
        for p, b in zip(self.params, owner):
            p.register_post_accumulate_grad_hook(self._hook_for(b))
        self._reset()

    def _reset(self) -> None:
        self._works = [None] * len(self.buckets)
        self._pending = [c for _, _, c in self.buckets]

    def _launch(self, b: int) -> None:
        s, e, _ = self.buckets[b]
        self._works[b] = dist.all_reduce(self.flat[s:e], op=dist.ReduceOp.AVG, group=self.group,
                                         async_op=True)

    def _hook_for(self, b: int):
        def hook(_param):
            self._pending[b] -= 1
            if self._pending[b] == 0 and self._works[b] is None:
                self._launch(b)
        return hook

    def zero(self) -> None:
        self.flat.zero_()
        if self.overlap:
            self._reset()

    def all_reduce(self) -> None:
        """Average the gradients over the ranks (no-op on one rank)."""
        if not (dist.is_initialized() and dist.get_world_size(self.group) > 1):
            return
        if not self.overlap:
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG, group=self.group)
            return
        for b in range(len(self.buckets)):
            if self._works[b] is None:
                self._launch(b)
        for w in self._works:
            w.wait()
        self._reset()
