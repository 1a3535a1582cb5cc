"""Data-parallel training: one process per GPU, gradients averaged over NCCL.

The reference is single-process; this module adds the exchange step that batch sharding
needs. Every parameter's gradient lives in a flat arena (see ``optim.arena``), so the
all-reduce runs in place on a few large contiguous buffers, with no gather or scatter.
All ranks issue the same collectives in the same order.
"""

from __future__ import annotations

import os
from collections.abc import Sequence

from tensorgrad_b200.optim.arena import flatten_parameters
from tensorgrad_b200.tensor import Tensor

__all__ = ["GradientAllReduce", "barrier", "max_over_ranks", "world_size"]


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


class GradientAllReduce:
    """Averages every parameter gradient across ranks, in place in the gradient arenas."""

    def __init__(self, params: Sequence[Tensor]) -> None:
        self.arenas = flatten_parameters(list(params))
        self.closed = False

    def reduce(self) -> None:
        d = _dist()
        if d is None or d.get_world_size() == 1:
            return
        op = d.ReduceOp.AVG if d.get_backend() == "nccl" else d.ReduceOp.SUM
        for arena in self.arenas:
            t = arena.grad_buf._t
            d.all_reduce(t, op=op)
            if op == d.ReduceOp.SUM:
                arena.grad_buf *= 1.0 / d.get_world_size()

    def close(self) -> None:
        self.closed = True
