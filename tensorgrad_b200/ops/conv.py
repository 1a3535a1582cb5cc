"""2-D convolution and max pooling on device tensors (the reference's ops/conv.py).

``conv2d`` lowers to an im2col patch matrix and one tensor-core GEMM per direction; the
patch matrix is kept for the weight gradient, as the reference keeps it
(ops/conv.py:91-116). ``max_pool2d`` records the winning window cell per output so the VJP
is a gather instead of a recomputation of the hit masks (ops/conv.py:300-357); the winner is
the same: the first maximum in row-major order, a NaN counting as the maximum.
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import ConvShape, check, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import Need, as_tensor, make_result
from tensorgrad_b200.ops.elementwise import cast_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["conv2d", "max_pool2d"]

IntPair = int | tuple[int, int]


def _pair(value: IntPair, name: str) -> tuple[int, int]:
    pair = (value, value) if isinstance(value, int) else tuple(int(v) for v in value)
    if len(pair) != 2:
        raise ValueError(f"{name} must be an int or a pair of ints")
    return pair  # type: ignore[return-value]


def _out_size(size: int, kernel: int, stride: int, padding: int) -> int:
    out = (size + 2 * padding - kernel) // stride + 1
    if out <= 0:
        raise ValueError(
            f"kernel {kernel} with padding {padding} does not fit an input of size {size}"
        )
    return out


def _shape(x_shape: tuple[int, ...], c_out: int, kernel: tuple[int, int],
           stride: tuple[int, int], padding: tuple[int, int]) -> ConvShape:
    n, c, h, w = x_shape
    oh = _out_size(h, kernel[0], stride[0], padding[0])
    ow = _out_size(w, kernel[1], stride[1], padding[1])
    return ConvShape(n, c, h, w, c_out, kernel[0], kernel[1], stride[0], stride[1], padding[0],
                     padding[1], oh, ow)


def _float_pair(a: DeviceArray, b: DeviceArray) -> tuple[DeviceArray, DeviceArray]:
    dt = np.result_type(a.dtype, b.dtype)
    if dt.kind != "f":
        dt = np.dtype(np.float64)
    return (a if a.dtype == dt else cast_array(a, dt)), (b if b.dtype == dt else cast_array(b, dt))


@profiled("conv2d")
def conv2d(x: Any, weight: Any, bias: Any = None, stride: IntPair = 1,
           padding: IntPair = 0) -> Tensor:
    """2-D cross-correlation of ``(N, C_in, H, W)`` input with ``(C_out, C_in, KH, KW)``
    filters (ops/conv.py:128-177). Returns ``(N, C_out, OH, OW)``."""
    tx, tw = as_tensor(x), as_tensor(weight)
    tb = None if bias is None else as_tensor(bias)
    if tx.ndim != 4 or tw.ndim != 4:
        raise ValueError(f"conv2d expects 4-D input and weight, got {tx.shape} and {tw.shape}")
    if tx.shape[1] != tw.shape[1]:
        raise ValueError(f"input has {tx.shape[1]} channels but weight expects {tw.shape[1]}")
    st, pad = _pair(stride, "stride"), _pair(padding, "padding")
    c_out = tw.shape[0]
    if tb is not None and tb.shape != (c_out,):
        raise ValueError(f"bias must have shape ({c_out},), got {tb.shape}")
    xd, wd = _float_pair(tx.data, tw.data)
    bd = None if tb is None else (tb.data if tb.dtype == xd.dtype else cast_array(tb.data, xd.dtype))
    s = _shape(tx.shape, c_out, (tw.shape[2], tw.shape[3]), st, pad)
    code = dtype_code(xd.dtype)
    ref = ctypes.byref(s)
    rows, ld = ctypes.c_int64(), ctypes.c_int64()
    check(lib.tg_conv2d_cols_shape(ref, ctypes.byref(rows), ctypes.byref(ld)), "conv2d")
    cols = device.empty((rows.value, ld.value), xd.dtype)
    y = device.empty((s.n, c_out, s.oh, s.ow), xd.dtype)
    scratch = device.scratch(lib.tg_conv2d_forward_scratch_bytes(code, ref))
    check(lib.tg_conv2d_forward(code, ref, xd.ptr, wd.ptr, bd.ptr if bd is not None else None,
                                y.ptr, cols.ptr, scratch.ptr, device.stream()), "conv2d")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        if g.dtype != xd.dtype:
            g = cast_array(g, xd.dtype)
        gx = device.empty(tx.shape, xd.dtype) if need[0] else None
        gw = device.empty(tw.shape, xd.dtype) if need[1] else None
        gb = device.empty((c_out,), xd.dtype) if tb is not None and need[2] else None
        scr = device.scratch(lib.tg_conv2d_backward_scratch_bytes(code, ref, int(gx is not None)))
        check(lib.tg_conv2d_backward(
            code, ref, g.ptr, cols.ptr, wd.ptr, gx.ptr if gx is not None else None,
            gw.ptr if gw is not None else None, gb.ptr if gb is not None else None, scr.ptr,
            device.stream()), "conv2d backward")
        if gx is not None and gx.dtype != tx.dtype and tx.dtype.kind == "f":
            gx = cast_array(gx, tx.dtype)
        return (gx, gw) if tb is None else (gx, gw, gb)

    parents = (tx, tw) if tb is None else (tx, tw, tb)
    return make_result(y, parents, backward, "conv2d")


@profiled("max_pool2d")
def max_pool2d(x: Any, kernel_size: IntPair, stride: IntPair | None = None,
               padding: IntPair = 0) -> Tensor:
    """Max pooling over ``(N, C, H, W)``; ``stride`` defaults to ``kernel_size``; ``-inf``
    padding of at most half the kernel (ops/conv.py:300-357)."""
    tx = as_tensor(x)
    if tx.ndim != 4:
        raise ValueError(f"max_pool2d expects 4-D input, got {tx.shape}")
    kh, kw = _pair(kernel_size, "kernel_size")
    sh, sw = _pair(kernel_size if stride is None else stride, "stride")
    ph, pw = _pair(padding, "padding")
    if ph > kh // 2 or pw > kw // 2:
        raise ValueError(
            f"padding {(ph, pw)} must be at most half the kernel size {(kh, kw)}; larger "
            "padding creates windows that contain only padding"
        )
    if kh * kw > 256:
        raise ValueError(f"max_pool2d supports windows of at most 256 cells, got {(kh, kw)}")
    xd = tx.data if tx.dtype.kind == "f" else cast_array(tx.data, np.dtype(np.float64))
    s = _shape(tx.shape, 0, (kh, kw), (sh, sw), (ph, pw))
    code = dtype_code(xd.dtype)
    ref = ctypes.byref(s)
    y = device.empty((s.n, s.c, s.oh, s.ow), xd.dtype)
    arg = device.empty((s.n, s.c, s.oh, s.ow), np.uint8)
    check(lib.tg_max_pool2d_forward(code, ref, xd.ptr, y.ptr, arg.ptr, device.stream()),
          "max_pool2d")

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        if g.dtype != xd.dtype:
            g = cast_array(g, xd.dtype)
        gx = device.empty(tx.shape, xd.dtype)
        check(lib.tg_max_pool2d_backward(code, ref, g.ptr, arg.ptr, gx.ptr, device.stream()),
              "max_pool2d backward")
        return (gx,)

    return make_result(y, (tx,), backward, "max_pool2d")
