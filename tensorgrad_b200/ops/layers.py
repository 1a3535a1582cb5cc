"""Fused building blocks used by :mod:`tensorgrad_b200.nn` (the reference's ops/layers.py):
linear, layer norm, batch norm, embedding and dropout."""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import MUL, check, lib
from tensorgrad_b200._random import dropout_threshold, get_rng, keep_mask, pcg64_take
from tensorgrad_b200.autograd import no_grad
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops import elementwise, reduce
from tensorgrad_b200.ops._util import Need, as_tensor, constant, grad_buffer, make_result
from tensorgrad_b200.ops.elementwise import binary_array, cast_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["batch_norm", "dropout", "embedding", "layer_norm", "linear"]


def _same_dtype(*arrays: DeviceArray | None) -> list[DeviceArray | None]:
    dt = np.result_type(*[a.dtype for a in arrays if a is not None])
    if dt.kind != "f":
        dt = np.dtype(np.float64)
    return [a if a is None or a.dtype == dt else cast_array(a, dt) for a in arrays]


@profiled("linear")
def linear(x: Any, weight: Any, bias: Any = None) -> Tensor:
    """``x @ weight.T + bias`` over flattened leading axes, as one GEMM with the bias in its
    epilogue (ops/layers.py:22-62). The VJP is two GEMMs and a column sum."""
    tx, tw = as_tensor(x), as_tensor(weight)
    tb = None if bias is None else as_tensor(bias)
    if tw.ndim != 2 or tx.ndim == 0 or tx.shape[-1] != tw.shape[1]:
        raise ValueError(f"linear: input {tx.shape} does not match weight {tw.shape}")
    xd, wd, bd = _same_dtype(tx.data, tw.data, None if tb is None else tb.data)
    assert xd is not None and wd is not None
    out_f, in_f = tw.shape
    rows = xd.size // in_f if in_f else 0
    code = dtype_code(xd.dtype)
    y = device.empty((*tx.shape[:-1], out_f), xd.dtype)
    fwd_bytes = lib.tg_linear_forward_scratch_bytes(code, rows, in_f, out_f)
    fwd_scratch = device.scratch(fwd_bytes) if fwd_bytes > 16 else None
    check(lib.tg_linear_forward(code, xd.ptr, wd.ptr, bd.ptr if bd is not None else None, y.ptr,
                                rows, in_f, out_f,
                                fwd_scratch.ptr if fwd_scratch is not None else None,
                                device.stream()), "linear")
    has_bias = tb is not None

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        if g.dtype != xd.dtype:
            g = cast_array(g, xd.dtype)
        gx = device.empty(tx.shape, xd.dtype) if need[0] else None
        gw = grad_buffer(tw, tw.shape, xd.dtype) if need[1] else None
        gb = grad_buffer(tb, (out_f,), xd.dtype) if has_bias and need[2] else None
        mask = (1 if gx is not None else 0) | (2 if gw is not None else 0) | (4 if gb is not None else 0)
        scratch = device.scratch(lib.tg_linear_backward_scratch_bytes(code, rows, in_f, out_f,
                                                                      mask))
        check(lib.tg_linear_backward(
            code, g.ptr, xd.ptr, wd.ptr, gx.ptr if gx is not None else None,
            gw.ptr if gw is not None else None, gb.ptr if gb is not None else None,
            rows, in_f, out_f, mask, 0.0, scratch.ptr,
            device.stream()), "linear backward")
        if gx is not None and gx.dtype != tx.dtype:
            gx = cast_array(gx, tx.dtype)
        return (gx, gw) if not has_bias else (gx, gw, gb)

    def graph(g: Tensor, out: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        # gx = g W, gW = g2^T x2 (leading axes flattened), gb = column sums of g2.
        from tensorgrad_b200.ops.linalg import matmul
        from tensorgrad_b200.ops.reduce import sum as tsum
        from tensorgrad_b200.ops.shape import reshape, transpose

        g2 = reshape(g, (rows, out_f))
        gx = reshape(matmul(g2, tw), tx.shape) if need[0] else None
        gw = matmul(transpose(g2, 0, 1), reshape(tx, (rows, in_f))) if need[1] else None
        if not has_bias:
            return gx, gw
        return gx, gw, (tsum(g2, axis=0) if need[2] else None)

    parents = (tx, tw) if tb is None else (tx, tw, tb)
    return make_result(y, parents, backward, "linear", graph)


@profiled("layer_norm")
def layer_norm(x: Any, weight: Any = None, bias: Any = None, eps: float = 1e-5) -> Tensor:
    """Normalise over the last axis, then scale and shift (ops/layers.py:65-141).

    Forward saves the per-row mean and ``rstd``; the VJP recomputes ``xhat`` from them:
    ``gx = rstd (gh - mean(gh) - xhat mean(gh xhat))`` with ``gh = g * weight``.
    """
    tx = as_tensor(x)
    tw = None if weight is None else as_tensor(weight)
    tb = None if bias is None else as_tensor(bias)
    xd = tx.data if tx.dtype.kind == "f" else cast_array(tx.data, np.dtype(np.float64))
    wd = None if tw is None else tw.data
    bd = None if tb is None else tb.data
    cols = tx.shape[-1]
    rows = xd.size // cols if cols else 0
    code = dtype_code(xd.dtype)
    y = device.empty(tx.shape, xd.dtype)
    mean = device.empty((rows,), xd.dtype)
    rstd = device.empty((rows,), xd.dtype)
    check(lib.tg_layer_norm_forward(code, xd.ptr, wd.ptr if wd is not None else None,
                                    bd.ptr if bd is not None else None, y.ptr, mean.ptr,
                                    rstd.ptr, rows, cols, eps, device.stream()), "layer_norm")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        k = 1
        need_w = need_b = False
        if tw is not None:
            need_w = need[k]
            k += 1
        if tb is not None:
            need_b = need[k]
        gx = device.empty(tx.shape, xd.dtype) if need[0] else None
        gw = grad_buffer(tw, (cols,), xd.dtype) if need_w else None
        gb = grad_buffer(tb, (cols,), xd.dtype) if need_b else None
        mask = (1 if gx is not None else 0) | (2 if gw is not None else 0) | (4 if gb is not None else 0)
        scratch = (device.scratch(lib.tg_layer_norm_scratch_bytes(code, rows, cols))
                   if (gw is not None or gb is not None) else None)
        check(lib.tg_layer_norm_backward(
            code, g.ptr, xd.ptr, wd.ptr if wd is not None else None, mean.ptr, rstd.ptr,
            gx.ptr if gx is not None else None, gw.ptr if gw is not None else None,
            gb.ptr if gb is not None else None, rows, cols, mask,
            scratch.ptr if scratch is not None else None, device.stream()), "layer_norm backward")
        grads: list[DeviceArray | None] = [gx]
        if tw is not None:
            grads.append(gw)
        if tb is not None:
            grads.append(gb)
        return tuple(grads)

    def graph(g: Tensor, y_: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        # The same closed form with the row statistics recomputed as differentiable ops
        # (ops/layers.py:120-138), so derivatives of any order flow through x as well.
        return _normalized_vjp(g, tx, tw, tb, (tx.ndim - 1,), eps, need, None)

    parents = tuple(t for t in (tx, tw, tb) if t is not None)
    return make_result(y, parents, backward, "layer_norm", graph)


def _normalized_vjp(g: Tensor, x: Tensor, w: Tensor | None, b: Tensor | None,
                    axes: tuple[int, ...], eps: float, need: Need,
                    view: tuple[int, ...] | None) -> tuple[Tensor | None, ...]:
    """Graph VJP of ``xhat * w + b`` with ``xhat`` normalised over ``axes`` (biased
    variance): ``gx = rstd (gh - mean(gh) - xhat mean(gh xhat))``, ``gh = g w``,
    ``gw = sum(g xhat)``, ``gb = sum(g)``. Without ``view`` (layer norm: parameters along the
    normalised axes) the parameter sums run over the other axes; with ``view`` (batch norm:
    one parameter per channel, ``w`` reshaped to ``view`` to broadcast) over ``axes``."""
    from tensorgrad_b200.ops.shape import reshape

    mul, sub, add = elementwise.mul, elementwise.sub, elementwise.add
    centred = sub(x, reduce.mean(x, axes, keepdims=True))
    rstd = elementwise.pow(add(reduce.mean(mul(centred, centred), axes, keepdims=True), eps),
                           -0.5)
    xhat = mul(centred, rstd)
    other = axes if view is not None else tuple(i for i in range(x.ndim) if i not in axes)
    grads: list[Tensor | None] = [None]
    if need[0]:
        gh = g if w is None else mul(g, w if view is None else reshape(w, view))
        inner = sub(sub(gh, reduce.mean(gh, axes, keepdims=True)),
                    mul(xhat, reduce.mean(mul(gh, xhat), axes, keepdims=True)))
        grads[0] = mul(rstd, inner)
    k = 1
    for param, term in ((w, lambda: mul(g, xhat)), (b, lambda: g)):
        if param is None:
            continue
        grads.append(reshape(reduce.sum(term(), other), param.shape) if need[k] else None)
        k += 1
    return tuple(grads)


@profiled("batch_norm")
def batch_norm(
    x: Tensor,
    running_mean: DeviceArray | None,
    running_var: DeviceArray | None,
    weight: Tensor | None = None,
    bias: Tensor | None = None,
    *,
    training: bool = True,
    momentum: float = 0.1,
    eps: float = 1e-5,
) -> Tensor:
    """Batch normalisation over ``(N, C, *spatial)`` with per-channel statistics
    (ops/layers.py:144-189).

    Training mode runs fused kernels: one pass for the float64 per-channel statistics (and
    the running-statistics update), one for the normalisation; the VJP is one reduction pass
    and one elementwise pass, the closed form of the composite the reference records
    (``mean``, ``var``, ``sub``, ``div``, ``sqrt``, ``mul``, ``add``). Evaluation mode is that
    composite, as in the reference.
    """
    if x.ndim < 2:
        raise ValueError(f"batch_norm expects (N, C, ...) input, got {x.shape}")
    axes = (0, *range(2, x.ndim))
    view = (1, -1, *([1] * (x.ndim - 2)))
    stats_ok = running_mean is None or running_var is None or (
        running_mean.dtype == x.dtype and running_var.dtype == x.dtype)
    if training and x.dtype.kind == "f" and stats_ok and x.size:
        return _batch_norm_train(x, running_mean, running_var, weight, bias, momentum, eps)
    if training:
        mean = reduce.mean(x, axes, keepdims=True)
        var = reduce.var(x, axes, keepdims=True, correction=0)
        if running_mean is not None and running_var is not None:
            n = x.size // x.shape[1]
            with no_grad():
                unbiased = var.data.reshape(-1) * (n / max(n - 1, 1))
                running_mean *= 1 - momentum
                running_mean += mean.data.reshape(-1) * momentum
                running_var *= 1 - momentum
                running_var += unbiased * momentum
    else:
        if running_mean is None or running_var is None:
            raise ValueError("evaluation-mode batch_norm needs running statistics")
        mean = Tensor._wrap(running_mean.astype(x.dtype, copy=False).reshape(view))
        var = Tensor._wrap(running_var.astype(x.dtype, copy=False).reshape(view))
    out = (x - mean) / elementwise.sqrt(var + eps)
    if weight is not None:
        out = out * weight.reshape(view)
    if bias is not None:
        out = out + bias.reshape(view)
    return out


def _batch_norm_train(x: Tensor, running_mean: DeviceArray | None,
                      running_var: DeviceArray | None, weight: Tensor | None,
                      bias: Tensor | None, momentum: float, eps: float) -> Tensor:
    n, c = x.shape[0], x.shape[1]
    hw = x.size // (n * c)
    xd = x.data
    wd = None if weight is None else (weight.data if weight.dtype == xd.dtype
                                      else cast_array(weight.data, xd.dtype))
    bd = None if bias is None else (bias.data if bias.dtype == xd.dtype
                                    else cast_array(bias.data, xd.dtype))
    if wd is not None and wd.size != c or bd is not None and bd.size != c:
        raise ValueError(f"batch_norm: weight/bias must have {c} elements")
    code = dtype_code(xd.dtype)
    y = device.empty(x.shape, xd.dtype)
    mean = device.empty((c,), xd.dtype)
    rstd = device.empty((c,), xd.dtype)
    track = running_mean is not None and running_var is not None
    scratch = device.scratch(lib.tg_batch_norm_scratch_bytes(code, n, c, hw))
    check(lib.tg_batch_norm_forward(
        code, n, c, hw, xd.ptr, wd.ptr if wd is not None else None,
        bd.ptr if bd is not None else None, y.ptr, mean.ptr, rstd.ptr,
        running_mean.ptr if track else None, running_var.ptr if track else None,
        momentum, eps, scratch.ptr, device.stream()), "batch_norm")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        if g.dtype != xd.dtype:
            g = cast_array(g, xd.dtype)
        k = 1
        need_w = need_b = False
        if weight is not None:
            need_w = need[k]
            k += 1
        if bias is not None:
            need_b = need[k]
        gx = device.empty(x.shape, xd.dtype) if need[0] else None
        gw = grad_buffer(weight, (c,), xd.dtype) if need_w and weight.shape == (c,) else (
            device.empty((c,), xd.dtype) if need_w else None)
        gb = grad_buffer(bias, (c,), xd.dtype) if need_b and bias.shape == (c,) else (
            device.empty((c,), xd.dtype) if need_b else None)
        scr = device.scratch(lib.tg_batch_norm_scratch_bytes(code, n, c, hw))
        check(lib.tg_batch_norm_backward(
            code, n, c, hw, g.ptr, xd.ptr, wd.ptr if wd is not None else None, mean.ptr,
            rstd.ptr, gx.ptr if gx is not None else None, gw.ptr if gw is not None else None,
            gb.ptr if gb is not None else None, scr.ptr, device.stream()), "batch_norm backward")
        grads: list[DeviceArray | None] = [gx]
        if weight is not None:
            grads.append(None if gw is None else gw.reshape(weight.shape))
        if bias is not None:
            grads.append(None if gb is None else gb.reshape(bias.shape))
        return tuple(grads)

    def graph(g: Tensor, y_: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        # The composite the reference records, differentiated as differentiable ops: per
        # channel statistics over the batch and spatial axes.
        view = (1, c, *([1] * (x.ndim - 2)))
        return _normalized_vjp(g, x, weight, bias, (0, *range(2, x.ndim)), eps, need, view)

    parents = tuple(t for t in (x, weight, bias) if t is not None)
    return make_result(y, parents, backward, "batch_norm", graph)


@profiled("embedding")
def embedding(indices: Any, weight: Any) -> Tensor:
    """Row lookup; the VJP is a scatter-add in the reference's sorted order
    (ops/layers.py:209-232).

    Host ids are checked before any device work, as the reference checks them, then uploaded.
    Device-resident ids (a Tensor or DeviceArray) stay on the device: the gather checks them
    (an out-of-range id raises IndexError at the next host synchronisation). Either way the
    VJP sorts the ids on the device (keys ``id * n + position``: the reference's stable
    order) and sums each run of equal ids, so the step needs no host work per call."""
    tw = as_tensor(weight)
    num, dim = tw.shape
    wd = tw.data
    code = dtype_code(wd.dtype)
    dev_ids = indices.data if isinstance(indices, Tensor) else indices
    if isinstance(dev_ids, DeviceArray):
        if dev_ids.dtype.kind not in "iu":
            raise TypeError(f"embedding indices must be integers, got {dev_ids.dtype}")
        ids_dev = dev_ids if dev_ids.dtype == np.int64 else cast_array(dev_ids, np.dtype(np.int64))
        shape, n = dev_ids.shape, dev_ids.size
        out = device.empty((*shape, dim), wd.dtype)
        check(lib.tg_embedding_forward(code, ids_dev.ptr, wd.ptr, out.ptr, n, num, dim,
                                       device.async_error_word(device.ASYNC_EMBEDDING_ID),
                                       device.stream()), "embedding")

        rows = _Rows(ids_dev, shape, num, dim, device.async_error_word(device.ASYNC_EMBEDDING_ID),
                     target=tw)
        return make_result(out, (tw,), rows.backward, "embedding", rows.graph)
    idx = np.asarray(indices)
    if not np.issubdtype(idx.dtype, np.integer):
        raise TypeError(f"embedding indices must be integers, got {idx.dtype}")
    if idx.size and (idx.min() < 0 or idx.max() >= num):
        raise IndexError(f"embedding ids must be in [0, {num}), got {idx.min()}..{idx.max()}")
    rows = host_rows(idx, num, dim)
    rows.target = tw
    return make_result(rows.gather_array(wd), (tw,), rows.backward, "embedding", rows.graph)


def host_rows(idx: np.ndarray, num: int, dim: int) -> _Rows:
    """``_Rows`` for host ids already checked against ``num``: uploaded once."""
    flat = np.ascontiguousarray(idx.reshape(-1), dtype=np.int64)
    return _Rows(device.from_numpy(flat), idx.shape, num, dim, None)


class _Rows:
    """An embedding call's ids: the row lookup (a gather) and its adjoint, the scatter-add of
    gradient rows, as array functions and as differentiable ops whose VJPs are each other
    (the reference's graph VJP is its ``scatter_add`` op, ops/layers.py:229-232)."""

    def __init__(self, ids: DeviceArray, shape: tuple[int, ...], num: int, dim: int,
                 err_word: Any, target: Tensor | None = None) -> None:
        self.ids, self.shape, self.num, self.dim = ids, tuple(shape), num, dim
        self.err_word = err_word
        self.target = target  # the table whose VJP this is (its gradient may go to its slot)

    def scatter_array(self, g: DeviceArray, out: DeviceArray | None = None) -> DeviceArray:
        """``gw[num, dim]`` (into ``out`` when given) with row ``i`` of ``g`` added into row
        ``ids[i]``, in the stable id order (a device sort of the keys ``id * n + position``);
        every row is written (zeros where no id points)."""
        n, num, dim = self.ids.size, self.num, self.dim
        scr = device.scratch(lib.tg_embedding_sort_scratch_bytes(n, num))
        keys = device.empty((n,), np.int64)  # uint64 sort keys
        check(lib.tg_embedding_sort(self.ids.ptr, n, num, keys.ptr, None, scr.ptr, scr.nbytes,
                                    device.stream()), "embedding sort")
        gw = device.empty((num, dim), g.dtype) if out is None else out
        check(lib.tg_embedding_backward_sorted(dtype_code(g.dtype), g.ptr, keys.ptr, n, gw.ptr,
                                               num, dim, 0, device.stream()),
              "embedding backward")
        return gw

    def gather_array(self, u: DeviceArray) -> DeviceArray:
        out = device.empty((*self.shape, self.dim), u.dtype)
        check(lib.tg_embedding_forward(dtype_code(u.dtype), self.ids.ptr, u.ptr, out.ptr,
                                       self.ids.size, self.num, self.dim, self.err_word,
                                       device.stream()), "embedding")
        return out

    def backward(self, g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        out = None if self.target is None else grad_buffer(self.target, (self.num, self.dim),
                                                           g.dtype)
        return (self.scatter_array(g, out),)

    def graph(self, g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (self.scatter(g),)

    def scatter(self, g: Tensor) -> Tensor:
        return make_result(self.scatter_array(g.data), (g,),
                           lambda u, need: (self.gather_array(u),), "embedding_backward",
                           lambda u, y, need: (self.gather(u),))

    def gather(self, u: Tensor) -> Tensor:
        return make_result(self.gather_array(u.data), (u,),
                           lambda v, need: (self.scatter_array(v),), "embedding", self.graph)


@profiled("dropout")
def dropout(x: Any, p: float = 0.5, training: bool = True,
            rng: np.random.Generator | None = None) -> Tensor:
    """Inverted dropout with the reference's quantised keep-mask (ops/layers.py:235-259); the
    identity when ``p == 0`` or not training. With a PCG64 generator (NumPy's default, and
    the global one) the mask is generated on the device from the generator's state, equal to
    the reference's bit for bit, and regenerated by the VJP instead of stored; other
    generators draw it on the host and upload it."""
    tx = as_tensor(x)
    if not 0.0 <= p <= 1.0:
        raise ValueError(f"dropout probability must be in [0, 1], got {p}")
    if not training or p == 0.0:
        return tx
    gen = rng or get_rng()
    threshold, scale = dropout_threshold(p)
    n = tx.size
    # keep_mask draws nothing when every element is dropped.
    state = (np.zeros(4, np.uint64) if threshold >= 65536
             else pcg64_take(gen, (n + 3) // 4))
    if state is None:
        # Not a PCG64 generator: the reference's mask drawn on the host and uploaded.
        keep, scale = keep_mask(tx.shape, p, gen)
        mask = device.from_numpy((keep * np.asarray(scale, dtype=tx.dtype)).astype(tx.dtype))

        def backward_host(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
            return (binary_array(g, mask, MUL),)

        def graph_host(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
            return (elementwise.mul(g, constant(mask)),)

        return make_result(binary_array(tx.data, mask, MUL), (tx,), backward_host, "dropout",
                           graph_host)

    def apply(src: DeviceArray) -> DeviceArray:
        out = device.empty(src.shape, src.dtype)
        check(lib.tg_dropout_pcg64(dtype_code(src.dtype), n, src.ptr, out.ptr,
                                   state.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), 0,
                                   threshold, scale, device.stream()), "dropout")
        return out

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        # The VJP multiplies by the same mask, regenerated from the same generator state.
        return (apply(g if g.dtype == tx.dtype else g.astype(tx.dtype)),)

    def masked(t: Tensor) -> Tensor:
        """The same mask applied to ``t`` as a differentiable op (self-adjoint)."""
        return make_result(apply(t.data if t.dtype == tx.dtype else t.data.astype(tx.dtype)),
                           (t,), backward, "dropout", graph)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        return (masked(g),)

    return make_result(apply(tx.data), (tx,), backward, "dropout", graph)
