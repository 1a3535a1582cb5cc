"""Flat parameter and gradient arenas.

The parameters of a group are re-homed into one contiguous device buffer (each tensor
starting on a 16-byte boundary), and every parameter gets a matching slot in a gradient
buffer of the same layout. The engine accumulates leaf gradients straight into those slots,
so a whole group's optimizer update, gradient norm and data-parallel all-reduce each run as
one launch over one buffer, with no gather or copy.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200.device import DeviceArray
from tensorgrad_b200.tensor import Tensor

_ALIGN_BYTES = 16


class Arena:
    """One dtype's parameters in one buffer; ``offsets[i]`` is where ``params[i]`` starts."""

    def __init__(self, params: Sequence[Tensor]) -> None:
        if not params:
            raise ValueError("an arena needs at least one parameter")
        dtypes = {p.dtype for p in params}
        if len(dtypes) != 1:
            raise TypeError(f"an arena holds one dtype, got {sorted(map(str, dtypes))}")
        self.dtype: np.dtype[Any] = params[0].dtype
        align = max(_ALIGN_BYTES // self.dtype.itemsize, 1)
        self.params = list(params)
        self.index = {id(p): i for i, p in enumerate(self.params)}  # by identity, never ==
        self.offsets: list[int] = []
        total = 0
        for p in self.params:
            self.offsets.append(total)
            total += -(-p.size // align) * align
        self.numel = total
        self.param_buf = device.zeros((total,), self.dtype)
        self.grad_buf = device.zeros((total,), self.dtype)
        for p, off in zip(self.params, self.offsets, strict=True):
            view = self.param_buf.flat_view(off, p.size, p.shape)
            device.copy_into(view, p.data)
            p.data = view
            p._grad_slot = self.grad_buf.flat_view(off, p.size, p.shape)
            if p._grad is not None:
                device.copy_into(p._grad_slot, p._grad.data.astype(self.dtype, copy=False))
                p._grad = Tensor._wrap(p._grad_slot)
            p._arena = self  # type: ignore[attr-defined]
        # A clip_grad_norm_ rescale not yet written into grad_buf: (total norm as a float64
        # device scalar, max_norm, eps). AdamW applies it inside its update pass; anything
        # else that reads or adds to the gradients first calls settle_clip().
        self.pending_clip: tuple[DeviceArray, float, float] | None = None

    def settle_clip(self) -> None:
        """Write a pending clip rescale into the gradient buffer (the reference's in-place
        ``g *= scale``), so that the gradients read as clipped."""
        pend = self.pending_clip
        if pend is None:
            return
        self.pending_clip = None
        from tensorgrad_b200._lib import check, int64_array, lib, ptr_array

        total, max_norm, eps = pend
        check(lib.tg_clip_scale_multi(device.dtype_code(self.dtype), 1,
                                      ptr_array([self.grad_buf.ptr]), int64_array([self.numel]),
                                      total.ptr, max_norm, eps, None, device.stream()), "clip")

    def intact(self) -> bool:
        """Every parameter still lives in its slot (nobody re-assigned ``p.data``)."""
        base = self.param_buf.ptr
        es = self.dtype.itemsize
        return all(p.data.ptr == base + off * es
                   for p, off in zip(self.params, self.offsets, strict=True))

    def grads_in_slots(self) -> bool:
        """Every parameter has a gradient, and it is the one in its arena slot."""
        return all(p._grad is not None and p._grad.data is p._grad_slot for p in self.params)

    def grad_view(self, start: int, stop: int) -> DeviceArray:
        return self.grad_buf.flat_view(start, stop - start)


def arena_of(params: Sequence[Tensor]) -> Arena | None:
    """The arena holding exactly ``params`` (in any order), if there is one."""
    arenas = {id(getattr(p, "_arena", None)) for p in params}
    if len(arenas) != 1:
        return None
    arena = getattr(params[0], "_arena", None)
    if arena is None or len(arena.params) != len(params):
        return None
    return arena


def flatten_parameters(params: Sequence[Tensor]) -> list[Arena]:
    """Re-home ``params`` into arenas (one per dtype), unless they already live in arenas."""
    params = list(params)
    if all(getattr(p, "_arena", None) is not None for p in params):
        seen: dict[int, Arena] = {}
        for p in params:
            seen.setdefault(id(p._arena), p._arena)  # type: ignore[attr-defined]
        return list(seen.values())
    fresh = [p for p in params if getattr(p, "_arena", None) is None]
    by_dtype: dict[str, list[Tensor]] = {}
    for p in fresh:
        by_dtype.setdefault(str(p.dtype), []).append(p)
    return [Arena(group) for group in by_dtype.values()]
