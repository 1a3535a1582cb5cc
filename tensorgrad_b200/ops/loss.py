"""Loss functions (the reference's ops/loss.py)."""

from __future__ import annotations

from typing import Any, Literal

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops import reduce
from tensorgrad_b200.ops._util import Need, as_tensor, coerce_pair, make_result
from tensorgrad_b200.ops.elementwise import cast_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["Reduction", "binary_cross_entropy_with_logits", "cross_entropy", "mse_loss"]

Reduction = Literal["mean", "sum", "none"]
_RED = {"mean": 0, "sum": 1, "none": 2}


@profiled("cross_entropy")
def cross_entropy(logits: Any, target: Any, *, ignore_index: int = -100,
                  reduction: Reduction = "mean") -> Tensor:
    """Softmax cross-entropy from unnormalised logits, class axis last (ops/loss.py:23-97).

    One kernel pass per row computes the log-sum-exp (online max and sum) and the row loss;
    the mean over non-ignored rows is a fixed-order float64 sum. The VJP is one pass writing
    ``(softmax - onehot) * g / n_valid``. Host targets are validated on the host, as the
    reference does, before any device work; device-resident targets are validated by the
    kernel and an out-of-range one raises at the next host synchronisation.
    """
    tl = as_tensor(logits)
    classes = tl.shape[-1]
    dev_t = target.data if isinstance(target, Tensor) else target
    bad = None
    if isinstance(dev_t, DeviceArray):
        # Device-resident targets stay on the device: the kernel checks them and an
        # out-of-range target raises IndexError at the next host synchronisation.
        if dev_t.dtype.kind not in "iu":
            raise TypeError(f"cross_entropy targets must be integers, got {dev_t.dtype}")
        if tl.shape[:-1] != dev_t.shape:
            raise ValueError(f"logits {tl.shape} and targets {dev_t.shape} are incompatible")
        if reduction not in _RED:
            raise ValueError(f"unknown reduction {reduction!r}")
        tgt = dev_t if dev_t.dtype == np.int64 else cast_array(dev_t, np.dtype(np.int64))
        t_shape = dev_t.shape
        bad = device.async_error_word(device.ASYNC_CLASS_TARGET)
    else:
        t = np.asarray(target)
        if not np.issubdtype(t.dtype, np.integer):
            raise TypeError(f"cross_entropy targets must be integers, got {t.dtype}")
        if tl.shape[:-1] != t.shape:
            raise ValueError(f"logits {tl.shape} and targets {t.shape} are incompatible")
        if reduction not in _RED:
            raise ValueError(f"unknown reduction {reduction!r}")
        flat_t = np.ascontiguousarray(t.reshape(-1), dtype=np.int64)
        valid = flat_t != ignore_index
        safe = np.where(valid, flat_t, 0)
        if np.any((safe < 0) | (safe >= classes)):
            raise IndexError(f"target out of range for {classes} classes")
        tgt = device.from_numpy(flat_t)
        t_shape = t.shape
    x = tl.data if tl.dtype.kind == "f" else cast_array(tl.data, np.dtype(np.float64))
    rows = tgt.size
    code = dtype_code(x.dtype)
    red = _RED[reduction]
    lse = device.empty((rows,), x.dtype)
    row_loss = device.empty((rows,), x.dtype)
    n_valid = device.empty((1,), np.int64)
    out = row_loss.reshape(t_shape) if red == 2 else device.empty((), x.dtype)
    check(lib.tg_cross_entropy_forward(code, x.ptr, tgt.ptr, lse.ptr, row_loss.ptr, out.ptr,
                                       rows, classes, ignore_index, red, n_valid.ptr, bad,
                                       device.stream()), "cross_entropy")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        if g.dtype != x.dtype:
            g = cast_array(g, x.dtype)
        grad = device.empty(tl.shape, x.dtype)
        check(lib.tg_cross_entropy_backward(code, x.ptr, tgt.ptr, lse.ptr, g.ptr, n_valid.ptr,
                                            grad.ptr, rows, classes, ignore_index, red,
                                            device.stream()), "cross_entropy backward")
        return (grad if grad.dtype == tl.dtype else cast_array(grad, tl.dtype),)

    host_targets = None if isinstance(dev_t, DeviceArray) else flat_t

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor]:
        # (softmax(x) - onehot) * valid * weight in differentiable ops: softmax as e / sum(e)
        # with e = exp(x - lse), the saved log-sum-exp a constant shift; the one-hot rows
        # (host targets) uploaded once.
        from tensorgrad_b200.ops.elementwise import exp, mul, sub
        from tensorgrad_b200.ops.shape import reshape

        if host_targets is None:
            raise NotImplementedError("create_graph=True: cross_entropy with device-resident "
                                      "targets has no differentiable VJP; pass host targets")
        keep = host_targets != ignore_index
        onehot = np.zeros((rows, classes), dtype=x.dtype)
        onehot[np.flatnonzero(keep), host_targets[keep]] = 1.0
        x2 = reshape(tl, (rows, classes))
        e = exp(sub(x2, Tensor._wrap(lse.reshape((rows, 1)))))
        probs = e / reduce.sum(e, axis=-1, keepdims=True)
        diff = mul(sub(probs, Tensor(onehot)), Tensor(keep.astype(x.dtype).reshape(rows, 1)))
        if red == 2:
            weight = reshape(g, (rows, 1))
        elif red == 0:
            weight = g / float(max(int(keep.sum()), 1))
        else:
            weight = g
        return (reshape(mul(diff, weight), tl.shape),)

    return make_result(out, (tl,), backward, "cross_entropy", graph)


@profiled("mse_loss")
def mse_loss(prediction: Any, target: Any, *, reduction: Reduction = "mean") -> Tensor:
    """``(prediction - target) ** 2`` reduced, composed as the reference composes it
    (ops/loss.py:148-161)."""
    tp, tt = coerce_pair(prediction, target)
    sq = (tp - tt) ** 2
    if reduction == "mean":
        return reduce.mean(sq)
    if reduction == "sum":
        return reduce.sum(sq)
    if reduction == "none":
        return sq
    raise ValueError(f"unknown reduction {reduction!r}")


@profiled("binary_cross_entropy")
def binary_cross_entropy_with_logits(logits: Any, target: Any, *,
                                     reduction: Reduction = "mean") -> Tensor:
    """Binary cross entropy of ``sigmoid(logits)`` against ``target`` in [0, 1]
    (ops/loss.py:100-145): ``max(z, 0) - z y + log1p(exp(-|z|))`` on the device, so nothing
    overflows; the gradient is ``sigmoid(z) - y`` for the logits and ``-z`` for the targets."""
    from tensorgrad_b200._lib import ABS, ADD, EXP, LOG1P, MUL, NEG, RELU, SIGMOID, SUB
    from tensorgrad_b200.ops.elementwise import _unary, binary_array, scale_array

    tz, ty = coerce_pair(logits, target)
    if tz.shape != ty.shape:
        raise ValueError(f"logits {tz.shape} and target {ty.shape} must have the same shape")
    if reduction not in ("mean", "sum", "none"):
        raise ValueError(f"unknown reduction {reduction!r}")
    dt = np.result_type(tz.dtype, ty.dtype)
    if dt.kind != "f":
        dt = np.dtype(np.float64)
    z = tz.data if tz.dtype == dt else cast_array(tz.data, dt)
    y = ty.data if ty.dtype == dt else cast_array(ty.data, dt)
    softplus_tail = _unary(_unary(_unary(_unary(z, ABS), NEG), EXP), LOG1P)
    losses = binary_array(binary_array(_unary(z, RELU), binary_array(z, y, MUL), SUB),
                          softplus_tail, ADD)
    n = max(losses.size, 1)
    if reduction == "none":
        out = losses
    else:
        total = reduce.sum_array(losses, tuple(range(losses.ndim))).reshape(())
        out = scale_array(total, 1.0 / n) if reduction == "mean" else total
    scale = 1.0 / n if reduction == "mean" else 1.0

    def upstream_array(g: DeviceArray) -> DeviceArray:
        if reduction == "none":
            return g
        from tensorgrad_b200.ops.shape import broadcast_array

        return broadcast_array(scale_array(g, scale), z.shape)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        up = upstream_array(g)
        return (binary_array(binary_array(_unary(z, SIGMOID), y, SUB), up, MUL)
                if need[0] else None,
                binary_array(_unary(z, NEG), up, MUL) if need[1] else None)

    def graph(g: Tensor, y_: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        from tensorgrad_b200.ops.elementwise import sigmoid
        from tensorgrad_b200.ops.shape import broadcast_to

        up = g if reduction == "none" else broadcast_to(g * scale, tz.shape)
        return ((sigmoid(tz) - ty) * up if need[0] else None,
                -tz * up if need[1] else None)

    return make_result(out, (tz, ty), backward, "binary_cross_entropy", graph)
