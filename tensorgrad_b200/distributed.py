"""Data-parallel training: one process per GPU, gradients averaged over NCCL.

The reference is single-process; this module adds the exchange step that batch sharding
needs. Every parameter's gradient lives in a flat arena (see ``optim.arena``), so the
all-reduce runs in place on contiguous buckets of those buffers, with no gather or scatter.

Buckets are consecutive parameters of an arena, about ``bucket_bytes`` each. The engine's
leaf hook (``autograd.add_leaf_hook``) fires when a parameter's gradient is final; when the
last parameter of a bucket is final, that bucket's all-reduce is launched asynchronously on
NCCL's stream and overlaps the rest of the backward walk. ``reduce()`` (after ``backward``)
launches any bucket not yet launched, in bucket order, then waits for all of them. Every
rank runs the same graph, so the hooks fire in the same order and all ranks issue the same
collectives in the same order.
"""

from __future__ import annotations

import os
from collections.abc import Callable, Sequence
from typing import Any

from tensorgrad_b200.optim.arena import flatten_parameters
from tensorgrad_b200.tensor import Tensor

__all__ = ["BucketedAllReduce", "GradientAllReduce", "barrier", "max_over_ranks",
           "plan_buckets", "world_size"]


def _dist():
    import torch.distributed as dist

    return dist if dist.is_available() and dist.is_initialized() else None


def world_size() -> int:
    d = _dist()
    return d.get_world_size() if d is not None else int(os.environ.get("WORLD_SIZE", "1"))


def barrier() -> None:
    d = _dist()
    if d is not None:
        d.barrier()


def max_over_ranks(value: float) -> float:
    """The maximum of a host scalar over all ranks (timings are max over ranks)."""
    d = _dist()
    if d is None:
        return value
    import torch

    backend = d.get_backend()
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    d.all_reduce(t, op=d.ReduceOp.MAX)
    return float(t.item())


def plan_buckets(sizes: Sequence[int], offsets: Sequence[int], itemsize: int,
                 bucket_bytes: int) -> list[tuple[int, int, list[int]]]:
    """Group consecutive parameters (element ``sizes`` at element ``offsets`` of one flat
    buffer) into buckets of at least ``bucket_bytes`` (the last may be smaller). Returns
    ``(start, stop, member indices)`` per bucket, ``stop`` the next bucket's start (so the
    padding between slots is reduced too and the buckets tile the buffer)."""
    buckets: list[tuple[int, int, list[int]]] = []
    members: list[int] = []
    start = offsets[0] if offsets else 0
    for i, (size, off) in enumerate(zip(sizes, offsets, strict=True)):
        members.append(i)
        end = off + size
        if (end - start) * itemsize >= bucket_bytes:
            nxt = offsets[i + 1] if i + 1 < len(offsets) else end
            buckets.append((start, nxt, members))
            members, start = [], nxt
    if members:
        buckets.append((start, offsets[-1] + sizes[-1], members))
    return buckets


class BucketedAllReduce:
    """Averages flat gradient buffers across ranks bucket by bucket.

    ``buffers`` lists, per flat buffer, the torch tensor and the ids, element offsets and
    sizes of the parameters whose gradients live in it. ``ready(param_id)`` marks one
    parameter's gradient final; a bucket whose members are all final is launched at once
    (asynchronously). ``finish()`` launches the rest in bucket order and waits.
    """

    def __init__(self, buffers: Sequence[tuple[Any, list[int], list[int], list[int]]],
                 bucket_bytes: int = 32 << 20) -> None:
        self.views: list[Any] = []
        self.members: list[int] = []  # member count per bucket
        self.owner: dict[int, int] = {}
        for flat, ids, offsets, sizes in buffers:
            for start, stop, idx in plan_buckets(sizes, offsets, flat.element_size(),
                                                 bucket_bytes):
                b = len(self.views)
                self.views.append(flat[start:stop])
                self.members.append(len(idx))
                for i in idx:
                    self.owner[ids[i]] = b
        self.pending = list(self.members)
        self.launched = [False] * len(self.views)
        self.order: list[int] = []       # launch order of the current step
        self.last_order: list[int] = []  # launch order of the last finished step
        self.handles: list[Any] = []

    def _launch(self, b: int) -> None:
        d = _dist()
        self.launched[b] = True
        self.order.append(b)
        if d is None or d.get_world_size() == 1:
            return
        op = d.ReduceOp.AVG if d.get_backend() == "nccl" else d.ReduceOp.SUM
        self.handles.append((b, d.all_reduce(self.views[b], op=op, async_op=True), op))

    def ready(self, param_id: int) -> None:
        b = self.owner.get(param_id)
        if b is None or self.launched[b]:
            return
        self.pending[b] -= 1
        if self.pending[b] == 0:
            self._launch(b)

    def finish(self) -> None:
        for b in range(len(self.views)):
            if not self.launched[b]:
                self._launch(b)
        d = _dist()
        for b, work, op in self.handles:
            work.wait()
            if d is not None and op == d.ReduceOp.SUM:
                self.views[b].mul_(1.0 / d.get_world_size())
        self.handles.clear()
        self.pending = list(self.members)
        self.launched = [False] * len(self.views)
        self.last_order, self.order = self.order, []


class GradientAllReduce:
    """Averages every parameter gradient across ranks, in place in the gradient arenas,
    overlapping each bucket's all-reduce with the rest of the backward walk.

    Call ``reduce()`` once after every ``backward()`` (before clipping and the optimizer).
    """

    def __init__(self, params: Sequence[Tensor], bucket_bytes: int = 32 << 20,
                 overlap: bool = True) -> None:
        from tensorgrad_b200 import autograd

        self.arenas = flatten_parameters(list(params))
        buffers = []
        for arena in self.arenas:
            buffers.append((arena.grad_buf._t, [id(p) for p in arena.params],
                            list(arena.offsets), [p.size for p in arena.params]))
        self.buckets = BucketedAllReduce(buffers, bucket_bytes)
        self.closed = False
        self._remove: Callable[[], None] | None = None
        if overlap and world_size() > 1:
            self._remove = autograd.add_leaf_hook(lambda t: self.buckets.ready(id(t)))

    def reduce(self) -> None:
        for arena in self.arenas:
            arena.settle_clip()
        self.buckets.finish()

    def close(self) -> None:
        if self._remove is not None:
            self._remove()
            self._remove = None
        self.closed = True
