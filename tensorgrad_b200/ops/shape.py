"""Shape manipulation (the reference's ops/shape.py): views, permutes, broadcasts and basic
indexing. Reshapes share storage; everything that moves elements is one strided-copy kernel."""

from __future__ import annotations

import math
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, int64_array, lib
from tensorgrad_b200.device import DeviceArray
from tensorgrad_b200.ops._util import Need, as_tensor, make_result, normalize_axis, unbroadcast
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["broadcast_to", "concat", "flatten", "getitem", "masked_fill", "permute", "reshape",
           "squeeze", "stack", "sum_to", "transpose", "unsqueeze", "where"]


def strided_copy(src_ptr: int, src_strides: list[int], dst_ptr: int, dst_strides: list[int],
                 shape: tuple[int, ...], itemsize: int) -> None:
    check(lib.tg_strided_copy(itemsize, len(shape), int64_array(shape), src_ptr,
                              int64_array(src_strides), dst_ptr, int64_array(dst_strides),
                              device.stream()), "strided copy")


def broadcast_array(a: DeviceArray, shape: tuple[int, ...]) -> DeviceArray:
    """Materialise ``a`` broadcast to ``shape``."""
    if a.shape == shape:
        return a
    out = device.empty(shape, a.dtype)
    strides = device.contiguous_strides(a.shape)
    pad = len(shape) - a.ndim
    src = [0] * pad + [0 if (n == 1 and shape[pad + i] != 1) else strides[i]
                       for i, n in enumerate(a.shape)]
    strided_copy(a.ptr, src, out.ptr, device.contiguous_strides(shape), shape, a.itemsize)
    return out


def permute_array(a: DeviceArray, perm: tuple[int, ...]) -> DeviceArray:
    shape = tuple(a.shape[p] for p in perm)
    out = device.empty(shape, a.dtype)
    strides = device.contiguous_strides(a.shape)
    strided_copy(a.ptr, [strides[p] for p in perm], out.ptr, device.contiguous_strides(shape),
                 shape, a.itemsize)
    return out


@profiled("reshape")
def reshape(a: Any, shape: tuple[int, ...]) -> Tensor:
    """A view with a new shape (one entry may be -1) (ops/shape.py:45)."""
    ta = as_tensor(a)
    out = ta.data.reshape(shape)
    src_shape = ta.shape

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (g.reshape(src_shape),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (reshape(g, src_shape),)

    return make_result(out, (ta,), backward, "reshape", graph)


def flatten(a: Any, start_axis: int = 0, end_axis: int = -1) -> Tensor:
    ta = as_tensor(a)
    if ta.ndim == 0:
        return reshape(ta, (1,))
    s = normalize_axis(start_axis, ta.ndim)
    e = normalize_axis(end_axis, ta.ndim)
    if s > e:
        raise ValueError("flatten: start_axis must not come after end_axis")
    shape = ta.shape[:s] + (math.prod(ta.shape[s:e + 1]),) + ta.shape[e + 1:]
    return reshape(ta, shape)


@profiled("permute")
def permute(a: Any, dims: tuple[int, ...]) -> Tensor:
    ta = as_tensor(a)
    perm = tuple(normalize_axis(d, ta.ndim) for d in dims)
    if sorted(perm) != list(range(ta.ndim)):
        raise ValueError(f"permute: {dims} is not a permutation of {ta.ndim} axes")
    inv = tuple(np.argsort(perm))

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (permute_array(g, inv),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (permute(g, inv),)

    return make_result(permute_array(ta.data, perm), (ta,), backward, "permute", graph)


def transpose(a: Any, axis0: int, axis1: int) -> Tensor:
    ta = as_tensor(a)
    perm = list(range(ta.ndim))
    i, j = normalize_axis(axis0, ta.ndim), normalize_axis(axis1, ta.ndim)
    perm[i], perm[j] = perm[j], perm[i]
    return permute(ta, tuple(perm))


def unsqueeze(a: Any, axis: int) -> Tensor:
    ta = as_tensor(a)
    ax = normalize_axis(axis, ta.ndim + 1)
    return reshape(ta, ta.shape[:ax] + (1,) + ta.shape[ax:])


def squeeze(a: Any, axis: int | None = None) -> Tensor:
    ta = as_tensor(a)
    if axis is None:
        return reshape(ta, tuple(n for n in ta.shape if n != 1))
    ax = normalize_axis(axis, ta.ndim)
    if ta.shape[ax] != 1:
        return ta
    return reshape(ta, ta.shape[:ax] + ta.shape[ax + 1:])


@profiled("broadcast_to")
def broadcast_to(a: Any, shape: tuple[int, ...]) -> Tensor:
    ta = as_tensor(a)
    shape = tuple(shape)
    np.broadcast_shapes(ta.shape, shape)
    src = ta.shape

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (unbroadcast(g, src),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (sum_to(g, src),)

    return make_result(broadcast_array(ta.data, shape), (ta,), backward, "broadcast_to", graph)


def sum_to(a: Any, shape: tuple[int, ...]) -> Tensor:
    ta = as_tensor(a)
    shape = tuple(shape)
    if ta.shape == shape:
        return ta
    target = ta.shape

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (broadcast_array(g, target),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (broadcast_to(g, target),)

    return make_result(unbroadcast(ta.data, shape), (ta,), backward, "sum_to", graph)


def _basic_view(shape: tuple[int, ...], itemsize: int, index: Any) -> tuple[int, tuple[int, ...], list[int]]:
    """Element offset, shape and element strides of ``x[index]`` for basic indexing."""
    items = index if isinstance(index, tuple) else (index,)
    for it in items:
        if not (it is None or it is Ellipsis or isinstance(it, int | np.integer | slice)):
            raise NotImplementedError("getitem on device tensors supports basic indexing only")
    base = np.empty(0, dtype=np.dtype(f"V{itemsize}"))
    strides = tuple(s * itemsize for s in device.contiguous_strides(shape))
    fake = np.lib.stride_tricks.as_strided(base, shape=shape, strides=strides)
    view = fake[index]
    offset = view.__array_interface__["data"][0] - base.__array_interface__["data"][0]
    return offset // itemsize, view.shape, [s // itemsize for s in view.strides]


def _normalize_index(index: Any) -> tuple[Any, bool]:
    """Tensors and lists in an index as host arrays, boolean masks as their nonzero
    positions; whether the index is advanced (ops/shape.py:162-179)."""
    items = index if isinstance(index, tuple) else (index,)
    out: list[Any] = []
    advanced = False
    for item in items:
        value = item.data if isinstance(item, Tensor) else item
        if isinstance(value, DeviceArray):
            value = value.numpy()
        if isinstance(value, list):
            value = np.asarray(value)
        if isinstance(value, np.ndarray):
            advanced = True
            if value.dtype == np.bool_:
                out.extend(np.nonzero(value))
                continue
            if not np.issubdtype(value.dtype, np.integer):
                raise IndexError(f"index arrays must be integer or boolean, got {value.dtype}")
        out.append(value)
    return (tuple(out) if isinstance(index, tuple) or len(out) != 1 else out[0]), advanced


def _gather_elements(ta: Tensor, index: Any) -> Tensor:
    """``a[index]`` with integer or boolean arrays (NumPy's advanced indexing): the selected
    flat positions are worked out on the host from the index alone, the elements are gathered
    on the device, and the VJP scatter-adds the gradient (an element selected twice gets both
    contributions), as the embedding's row lookup and its adjoint with rows of one element."""
    from tensorgrad_b200.ops.layers import host_rows

    positions = np.arange(ta.size, dtype=np.int64).reshape(ta.shape)[index]
    rows = host_rows(positions, max(ta.size, 1), 1)
    x = ta.data
    if x.dtype.kind != "f":
        # Integer data moves bit for bit through the float gather of the same width.
        width = {8: np.float64, 4: np.float32}.get(x.itemsize)
        if width is None:
            return Tensor._wrap(device.from_numpy(x.numpy()[index]))
        raw = DeviceArray(x._buf, x._off, (x.size, 1), np.dtype(width))
        got = rows.gather_array(raw)
        return Tensor._wrap(DeviceArray(got._buf, got._off, positions.shape, x.dtype))
    out = rows.gather_array(x.reshape((x.size, 1))).reshape(positions.shape)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (rows.scatter_array(g.reshape((g.size, 1))).reshape(ta.shape),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (reshape(rows.scatter(reshape(g, (*positions.shape, 1))), ta.shape),)

    return make_result(out, (ta,), backward, "getitem", graph)


@profiled("getitem")
def getitem(a: Any, index: Any) -> Tensor:
    """``a[index]``: NumPy's basic indexing (ints, slices, ``...``, ``None``) as one strided
    copy whose VJP writes the gradient into zeros at the selected positions; integer / boolean
    arrays (and tensors) as a gather whose VJP is a scatter-add (ops/shape.py:182-235)."""
    ta = as_tensor(a)
    index, advanced = _normalize_index(index)
    if advanced:
        return _gather_elements(ta, index)
    x = ta.data
    offset, shape, strides = _basic_view(ta.shape, x.itemsize, index)
    out = device.empty(shape, x.dtype)
    strided_copy(x.ptr + offset * x.itemsize, strides, out.ptr, device.contiguous_strides(shape),
                 shape, x.itemsize)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        gx = device.zeros(ta.shape, g.dtype)
        strided_copy(g.ptr, device.contiguous_strides(shape), gx.ptr + offset * g.itemsize,
                     strides, shape, g.itemsize)
        return (gx,)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (_scatter(g, ta.shape, index),)

    return make_result(out, (ta,), backward, "getitem", graph)


def _scatter(g: Tensor, shape: tuple[int, ...], index: Any) -> Tensor:
    """Zeros of ``shape`` with ``g`` at ``[index]``: getitem's VJP as a differentiable op (its
    own VJP is getitem again), for gradients that carry a graph."""
    gd = g.data
    offset, view_shape, strides = _basic_view(shape, gd.itemsize, index)
    out = device.zeros(shape, gd.dtype)
    strided_copy(gd.ptr, device.contiguous_strides(view_shape), out.ptr + offset * gd.itemsize,
                 strides, view_shape, gd.itemsize)

    def backward(gg: DeviceArray, need: Need) -> tuple[DeviceArray]:
        piece = device.empty(view_shape, gg.dtype)
        strided_copy(gg.ptr + offset * gg.itemsize, strides, piece.ptr,
                     device.contiguous_strides(view_shape), view_shape, gg.itemsize)
        return (piece,)

    def graph(gg: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (getitem(gg, index),)

    return make_result(out, (g,), backward, "scatter", graph)


@profiled("stack")
def stack(tensors: Any, axis: int = 0) -> Tensor:
    """Join equally shaped tensors along a new axis (ops/shape.py:265-281); the VJP hands
    each input its slice of the gradient."""
    ts = [as_tensor(t) for t in tensors]
    if not ts:
        raise ValueError("stack needs at least one tensor")
    shape0 = ts[0].shape
    if any(t.shape != shape0 for t in ts):
        raise ValueError(f"stack: shapes differ: {[t.shape for t in ts]}")
    ax = normalize_axis(axis, len(shape0) + 1)
    dt = np.result_type(*[t.dtype for t in ts])
    out_shape = (*shape0[:ax], len(ts), *shape0[ax:])
    out = device.empty(out_shape, dt)
    ostr = device.contiguous_strides(out_shape)
    slot_strides = ostr[:ax] + ostr[ax + 1:]
    for k, t in enumerate(ts):
        src = t.data if t.dtype == dt else t.data.astype(dt)
        strided_copy(src.ptr, device.contiguous_strides(shape0), out.ptr + k * ostr[ax] * out.itemsize,
                     slot_strides, shape0, out.itemsize)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        grads: list[DeviceArray | None] = []
        for k in range(len(ts)):
            if not need[k]:
                grads.append(None)
                continue
            gk = device.empty(shape0, g.dtype)
            strided_copy(g.ptr + k * ostr[ax] * g.itemsize, slot_strides, gk.ptr,
                         device.contiguous_strides(shape0), shape0, g.itemsize)
            grads.append(gk)
        return tuple(grads)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        lead = (slice(None),) * ax
        return tuple(getitem(g, (*lead, k)) if need[k] else None for k in range(len(ts)))

    return make_result(out, tuple(ts), backward, "stack", graph)


@profiled("concat")
def concat(tensors: Any, axis: int = 0) -> Tensor:
    """Join tensors along an existing axis (ops/shape.py:243-262): one strided copy per input
    into its slab of the output; the VJP hands each input its slab of the gradient."""
    ts = [as_tensor(t) for t in tensors]
    if not ts:
        raise ValueError("concat needs at least one tensor")
    ax = normalize_axis(axis, ts[0].ndim)
    rest = ts[0].shape[:ax] + ts[0].shape[ax + 1:]
    for t in ts:
        if t.ndim != ts[0].ndim or t.shape[:ax] + t.shape[ax + 1:] != rest:
            raise ValueError(f"concat: shapes {[t.shape for t in ts]} differ off axis {ax}")
    dt = np.result_type(*[t.dtype for t in ts])
    sizes = [t.shape[ax] for t in ts]
    starts = [0, *np.cumsum(sizes)[:-1].tolist()]
    out_shape = (*ts[0].shape[:ax], int(sum(sizes)), *ts[0].shape[ax + 1:])
    out = device.empty(out_shape, dt)
    ostr = device.contiguous_strides(out_shape)
    for t, start in zip(ts, starts, strict=True):
        src = t.data if t.dtype == dt else t.data.astype(dt)
        strided_copy(src.ptr, device.contiguous_strides(t.shape),
                     out.ptr + start * ostr[ax] * out.itemsize, ostr, t.shape, out.itemsize)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        grads: list[DeviceArray | None] = []
        for t, start, wanted in zip(ts, starts, need, strict=True):
            if not wanted:
                grads.append(None)
                continue
            piece = device.empty(t.shape, g.dtype)
            strided_copy(g.ptr + start * ostr[ax] * g.itemsize, ostr, piece.ptr,
                         device.contiguous_strides(t.shape), t.shape, g.itemsize)
            grads.append(piece)
        return tuple(grads)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        lead = (slice(None),) * ax
        return tuple(getitem(g, (*lead, slice(start, start + t.shape[ax]))) if wanted else None
                     for t, start, wanted in zip(ts, starts, need, strict=True))

    return make_result(out, tuple(ts), backward, "concat", graph)


_COND_CODES = {np.dtype(np.bool_): -1, np.dtype(np.float32): 0, np.dtype(np.float64): 1,
               np.dtype(np.int64): 2}


def _condition(mask: Any) -> DeviceArray:
    """A condition on the device, read as ``!= 0``: a boolean, float or int64 device array
    as it is, anything else (host arrays, bools) uploaded as one byte per element."""
    data = mask.data if isinstance(mask, Tensor) else mask
    if isinstance(data, DeviceArray) and data.dtype in _COND_CODES:
        return data
    if isinstance(data, DeviceArray):
        data = data.numpy()
    return device.from_numpy(np.asarray(data).astype(np.bool_, copy=False))


def _bcast(shape: tuple[int, ...], out: tuple[int, ...]) -> list[int]:
    strides = device.contiguous_strides(shape)
    pad = len(out) - len(shape)
    return [0] * pad + [0 if (n == 1 and out[pad + i] != 1) else strides[i]
                        for i, n in enumerate(shape)]


def where_array(cond: DeviceArray, a: DeviceArray, b: DeviceArray) -> DeviceArray:
    """``cond ? a : b`` broadcast together; ``a`` and ``b`` share one floating dtype."""
    from tensorgrad_b200.device import dtype_code

    shape = tuple(np.broadcast_shapes(cond.shape, a.shape, b.shape))
    out = device.empty(shape, a.dtype)
    check(lib.tg_where(dtype_code(a.dtype), _COND_CODES[cond.dtype], len(shape),
                       int64_array(shape), cond.ptr, int64_array(_bcast(cond.shape, shape)),
                       a.ptr, int64_array(_bcast(a.shape, shape)), b.ptr,
                       int64_array(_bcast(b.shape, shape)), out.ptr, device.stream()), "where")
    return out


@profiled("where")
def where(condition: Any, a: Any, b: Any) -> Tensor:
    """Elements of ``a`` where ``condition`` holds, of ``b`` elsewhere, all three broadcast
    (ops/shape.py:290-309); the gradient goes to the branch that was picked."""
    from tensorgrad_b200.ops._util import coerce_pair
    from tensorgrad_b200.ops.elementwise import cast_array

    cond = _condition(condition)
    ta, tb = coerce_pair(a, b)
    dt = np.result_type(ta.dtype, tb.dtype)
    if dt.kind != "f":
        dt = np.dtype(np.float64)
    ad = ta.data if ta.dtype == dt else cast_array(ta.data, dt)
    bd = tb.data if tb.dtype == dt else cast_array(tb.data, dt)
    out = where_array(cond, ad, bd)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        zero = device.scalar_like(0.0, g.dtype)
        return (unbroadcast(where_array(cond, g, zero), ta.shape) if need[0] else None,
                unbroadcast(where_array(cond, zero, g), tb.shape) if need[1] else None)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        c = Tensor._wrap(cond)
        return (sum_to(where(c, g, 0.0), ta.shape) if need[0] else None,
                sum_to(where(c, 0.0, g), tb.shape) if need[1] else None)

    return make_result(out, (ta, tb), backward, "where", graph)


@profiled("masked_fill")
def masked_fill(a: Any, mask: Any, value: float) -> Tensor:
    """``a`` with ``value`` wherever ``mask`` (broadcastable to ``a``) holds
    (ops/shape.py:312-328); filled positions get no gradient."""
    from tensorgrad_b200.ops.elementwise import cast_array

    ta = as_tensor(a)
    cond = _condition(mask)
    xd = ta.data if ta.dtype.kind == "f" else cast_array(ta.data, np.dtype(np.float64))
    out = where_array(cond, device.scalar_like(value, xd.dtype), xd)
    if out.shape != ta.shape:
        raise ValueError(f"masked_fill: mask {cond.shape} does not broadcast to {ta.shape}")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (where_array(cond, device.scalar_like(0.0, g.dtype), g),)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (masked_fill(g, Tensor._wrap(cond), 0.0),)

    return make_result(out, (ta,), backward, "masked_fill", graph)
