"""Gradient-norm clipping (the reference's optim/clip.py:15-31) on the device.

The global L2 norm is accumulated in float64 over all gradients (one launch for a flat
arena, or a multi-tensor launch), and the rescale ``g *= max_norm / (total + eps)`` (the
factor rounded to the gradient dtype, as the reference casts it) applies only when that
factor is below 1, decided on the device. For a flat arena the rescale is left pending:
AdamW's update pass reads the gradients rescaled (clip and update in one pass), and any
other reader of a gradient writes the rescale first, so the gradients always read as the
reference's clipped ones. Returning the norm as a Python float reads 8 bytes back, which
synchronises the stream once per call.
"""

from __future__ import annotations

from collections.abc import Iterable

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, int64_array, lib, ptr_array
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.optim.arena import arena_of
from tensorgrad_b200.tensor import Tensor

__all__ = ["clip_grad_norm_", "grad_norm_device"]


def _segments(params: list[Tensor]) -> dict[str, list[DeviceArray]]:
    """Gradient buffers to reduce, per dtype: the whole flat arena when it is exact."""
    arena = arena_of(params)
    if arena is not None and arena.grads_in_slots():
        arena.settle_clip()
        return {str(arena.dtype): [arena.grad_buf]}
    out: dict[str, list[DeviceArray]] = {}
    for p in params:
        if p.grad is not None:
            out.setdefault(str(p.grad.dtype), []).append(p.grad.data)
    return out


def grad_norm_device(params: Iterable[Tensor]) -> tuple[DeviceArray, dict[str, list[DeviceArray]]]:
    """Total gradient norm as a float64 device scalar, and the buffers it covered."""
    segs = _segments(list(params))
    total = device.zeros((1,), np.float64)
    parts: list[DeviceArray] = []
    for bufs in segs.values():
        code = dtype_code(bufs[0].dtype)
        part = device.empty((1,), np.float64)
        scratch = device.scratch(lib.tg_sumsq_scratch_bytes(len(bufs)))
        check(lib.tg_sumsq_multi(code, len(bufs), ptr_array(b.ptr for b in bufs),
                                 int64_array(b.size for b in bufs), part.ptr, scratch.ptr,
                                 device.stream()), "grad norm")
        parts.append(part)
    if len(parts) == 1:
        total = parts[0]
    elif parts:
        # sqrt(a^2 + b^2) across dtypes, on the device.
        from tensorgrad_b200._lib import ADD, MUL, SQRT
        from tensorgrad_b200.ops.elementwise import binary_array

        acc = binary_array(parts[0], parts[0], MUL)
        for p in parts[1:]:
            acc = binary_array(acc, binary_array(p, p, MUL), ADD)
        total = device.empty((1,), np.float64)
        check(lib.tg_unary(1, SQRT, 1, acc.ptr, 0.0, total.ptr, device.stream()), "grad norm")
    return total, segs


def clip_grad_norm_(params: Iterable[Tensor], max_norm: float, eps: float = 1e-6, *,
                    sync: bool = True) -> float | Tensor:
    """Rescale gradients in place so their global L2 norm is at most ``max_norm``.

    The norm and the scale stay on the device. ``sync=False`` returns the norm as a 0-d device
    tensor instead of a float, so a training step does not wait for the device here.

    Returns:
        The total norm before clipping.
    """
    params = list(params)
    total, segs = grad_norm_device(params)
    arena = arena_of(params)
    if (arena is not None and len(segs) == 1
            and next(iter(segs.values()))[0] is arena.grad_buf):
        # One flat arena: the rescale stays pending, and AdamW's update pass applies it while
        # it reads the gradients (one pass over them instead of two); reading a gradient
        # first writes it.
        arena.pending_clip = (total, float(max_norm), float(eps))
        segs = {}
    for bufs in segs.values():
        code = dtype_code(bufs[0].dtype)
        check(lib.tg_clip_scale_multi(code, len(bufs), ptr_array(b.ptr for b in bufs),
                                      int64_array(b.size for b in bufs), total.ptr, max_norm,
                                      eps, None, device.stream()), "clip")
    if not sync:
        return Tensor._wrap(total.reshape(()))
    return float(total.item())
