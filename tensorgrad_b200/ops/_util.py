"""Helpers shared by the op implementations (the reference's ops/_util.py:12-92)."""

from __future__ import annotations

import math
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, int64_array, int_array, lib
from tensorgrad_b200.autograd import BackwardFn, GraphFn, Node, is_grad_enabled
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.tensor import Tensor

Need = tuple[bool, ...]


def as_tensor(x: Any, like: Tensor | None = None) -> Tensor:
    """``x`` as a tensor; Python scalars adopt the floating dtype of ``like``."""
    if isinstance(x, Tensor):
        return x
    if isinstance(x, int | float) and like is not None and np.issubdtype(like.dtype, np.floating):
        return Tensor._wrap(device.from_numpy(np.asarray(x, dtype=like.dtype)))
    return Tensor(x)


def coerce_pair(a: Any, b: Any) -> tuple[Tensor, Tensor]:
    ta = a if isinstance(a, Tensor) else None
    tb = b if isinstance(b, Tensor) else None
    return as_tensor(a, tb), as_tensor(b, ta)


def make_result(data: DeviceArray, parents: tuple[Tensor, ...], backward: BackwardFn,
                op: str, graph: GraphFn | None = None) -> Tensor:
    """Wrap an op's output, recording a graph node if any input requires grad
    (ops/_util.py:28-46). ``backward`` is the VJP on device arrays; ``graph`` (optional) the
    same VJP in differentiable tensor ops, for ``create_graph=True``."""
    out = Tensor._wrap(data)
    if is_grad_enabled() and any(p._requires_grad for p in parents):
        out._requires_grad = True
        out._node = Node(op, parents, backward, graph)
    return out


def grad_buffer(t: Tensor | None, shape: tuple[int, ...], dtype: Any) -> DeviceArray:
    """Where a VJP writes the gradient of parent ``t``: the leaf's arena slot when it can take
    the gradient directly (``Tensor._grad_target``; saves a buffer and a copy per parameter
    and step), else a new buffer. The caller must write every element."""
    if (t is not None and t._node is None and t._grad_slot is not None
            and tuple(shape) == t.shape and np.dtype(dtype) == t.dtype):
        slot = t._grad_target()
        if slot is not None:
            return slot
    return device.empty(shape, dtype)


def constant(data: DeviceArray) -> Tensor:
    """A tensor outside every graph (masks and saved values inside graph VJPs)."""
    return Tensor._wrap(data)


def identity(x: Tensor) -> Tensor:
    """A node that passes gradients straight through to ``x``: differentiating against it
    reaches ``x``'s own graph."""
    return make_result(x.data, (x,), lambda g, need: (g,), "identity",
                       lambda g, y, need: (g,))


def graph_by_composite(parents: tuple[Tensor, ...], composite: Any, g: Tensor,
                       need: Need) -> tuple[Tensor | None, ...]:
    """The differentiable VJP of a fused op, taken through ``composite``: the same function
    of ``parents`` written with differentiable ops. It runs on identity nodes over the
    parents that need a gradient, and its own graph VJPs (kept, ``create_graph``) give
    gradients that are differentiable again, in ``g`` and in the parents."""
    from tensorgrad_b200 import autograd

    with autograd.enable_grad():
        leaves = [identity(p) if n else p for p, n in zip(parents, need, strict=True)]
        y = composite(*leaves)
    wanted = [t for t, n in zip(leaves, need, strict=True) if n]
    if not wanted or not y.requires_grad:
        return (None,) * len(parents)
    found = iter(autograd.grad(y, wanted, grad_outputs=g, create_graph=True, allow_unused=True))
    return tuple(next(found) if n else None for n in need)


def unbroadcast(grad: DeviceArray, shape: tuple[int, ...]) -> DeviceArray:
    """Sum ``grad`` down to ``shape``: the adjoint of broadcasting (ops/_util.py:49-63).

    Summing over leading axes only (bias and position-embedding gradients) is a column sum;
    anything else goes through the keep-axis reduction.
    """
    if grad.shape == shape:
        return grad
    extra = grad.ndim - len(shape)
    full = (1,) * extra + tuple(shape)
    keep = [not (i < extra or (full[i] == 1 and grad.shape[i] != 1)) for i in range(grad.ndim)]
    code = dtype_code(grad.dtype)
    # Leading summed axes followed only by kept ones: a column sum over a 2-D view.
    first_keep = keep.index(True) if True in keep else grad.ndim
    if all(keep[first_keep:]):
        rows = math.prod(grad.shape[:first_keep])
        cols = math.prod(grad.shape[first_keep:])
        out = device.empty(shape, grad.dtype)
        scratch = device.scratch(lib.tg_colsum_scratch_bytes(code, rows, cols))
        check(lib.tg_colsum(code, grad.ptr, out.ptr, rows, cols, 0, scratch.ptr,
                            device.stream()), "unbroadcast")
        return out
    out = device.empty(shape, grad.dtype)
    check(lib.tg_reduce_sum(code, grad.ndim, int64_array(grad.shape), int_array(keep),
                            grad.ptr, out.ptr, device.stream()), "unbroadcast")
    return out


def normalize_axes(axis: Any, ndim: int) -> tuple[int, ...]:
    if axis is None:
        return tuple(range(ndim))
    axes = (axis,) if isinstance(axis, int) else tuple(axis)
    out = []
    for ax in axes:
        if not -ndim <= ax < max(ndim, 1):
            raise np.exceptions.AxisError(ax, ndim)
        out.append(ax % ndim if ndim else 0)
    return tuple(sorted(set(out)))


def normalize_axis(axis: int, ndim: int) -> int:
    if not -ndim <= axis < ndim:
        raise np.exceptions.AxisError(axis, ndim)
    return axis % ndim
