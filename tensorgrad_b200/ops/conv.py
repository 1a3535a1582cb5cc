"""2-D convolution and max pooling on device tensors (the reference's ops/conv.py).

``conv2d`` lowers to an im2col patch matrix and one tensor-core GEMM per direction; the
patch matrix is kept for the weight gradient, as the reference keeps it
(ops/conv.py:91-116). ``max_pool2d`` records the winning window cell per output so the VJP
is a gather instead of a recomputation of the hit masks (ops/conv.py:300-357); the winner is
the same: the first maximum in row-major order, a NaN counting as the maximum.

Both are differentiable to any order (``create_graph=True``), as in the reference: the
convolution's two gradients are ops of their own, ``conv2d_input_grad`` (a transposed
convolution) and ``conv2d_weight_grad``, and the three form a family closed under taking
VJPs (each is bilinear in its two tensor arguments). Pooling's VJP scatters ``g`` to the
recorded winners; that scatter and its adjoint, a gather from the winners, are ops whose VJPs
are each other.
"""

from __future__ import annotations

import ctypes
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import ConvShape, check, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import Need, as_tensor, grad_buffer, make_result
from tensorgrad_b200.ops import reduce
from tensorgrad_b200.ops.elementwise import cast_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["conv2d", "conv2d_input_grad", "conv2d_weight_grad", "max_pool2d"]

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


def _cast(a: DeviceArray, dtype: np.dtype[Any]) -> DeviceArray:
    return a if a.dtype == dtype else cast_array(a, dtype)


def _patches(xd: DeviceArray, s: ConvShape) -> DeviceArray:
    """The im2col patch matrix of ``xd`` (``tg_conv2d_cols_shape`` rows x ld)."""
    ref = ctypes.byref(s)
    rows, ld = ctypes.c_int64(), ctypes.c_int64()
    check(lib.tg_conv2d_cols_shape(ref, ctypes.byref(rows), ctypes.byref(ld)), "conv2d")
    return device.empty((rows.value, ld.value), xd.dtype)


def _conv_array(xd: DeviceArray, wd: DeviceArray, bd: DeviceArray | None,
                s: ConvShape) -> tuple[DeviceArray, DeviceArray]:
    """``y = conv(x, w) + b`` and the patch matrix the weight gradient reads."""
    code, ref = dtype_code(xd.dtype), ctypes.byref(s)
    cols = _patches(xd, s)
    y = device.empty((s.n, s.c_out, s.oh, s.ow), xd.dtype)
    scratch = device.scratch(lib.tg_conv2d_forward_scratch_bytes(code, ref))
    check(lib.tg_conv2d_forward(code, ref, xd.ptr, wd.ptr, bd.ptr if bd is not None else None,
                                y.ptr, cols.ptr, scratch.ptr, device.stream()), "conv2d")
    return y, cols


def _input_grad_array(g: DeviceArray, wd: DeviceArray, s: ConvShape) -> DeviceArray:
    """``(n, c, h, w)`` input gradient of an output gradient ``g`` (no patch matrix needed)."""
    code, ref = dtype_code(wd.dtype), ctypes.byref(s)
    gx = device.empty((s.n, s.c, s.h, s.w), wd.dtype)
    scr = device.scratch(lib.tg_conv2d_backward_scratch_bytes(code, ref, 1))
    check(lib.tg_conv2d_backward(code, ref, _cast(g, wd.dtype).ptr, None, wd.ptr, gx.ptr, None,
                                 None, scr.ptr, device.stream()), "conv2d input gradient")
    return gx


def _weight_grad_array(cols: DeviceArray, g: DeviceArray, s: ConvShape) -> DeviceArray:
    """``(c_out, c, kh, kw)`` weight gradient from the patch matrix and ``g``."""
    code, ref = dtype_code(cols.dtype), ctypes.byref(s)
    gw = device.empty((s.c_out, s.c, s.kh, s.kw), cols.dtype)
    scr = device.scratch(lib.tg_conv2d_backward_scratch_bytes(code, ref, 0))
    check(lib.tg_conv2d_backward(code, ref, _cast(g, cols.dtype).ptr, cols.ptr, None, None,
                                 gw.ptr, None, scr.ptr, device.stream()),
          "conv2d weight gradient")
    return gw


def _im2col(xd: DeviceArray, s: ConvShape) -> DeviceArray:
    cols = _patches(xd, s)
    check(lib.tg_conv2d_im2col(dtype_code(xd.dtype), ctypes.byref(s), xd.ptr, cols.ptr,
                               device.stream()), "conv2d(im2col)")
    return cols


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
    bd = None if tb is None else _cast(tb.data, xd.dtype)
    s = _shape(tx.shape, c_out, (tw.shape[2], tw.shape[3]), st, pad)
    code = dtype_code(xd.dtype)
    ref = ctypes.byref(s)
    y, cols = _conv_array(xd, wd, bd, s)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        g = _cast(g, xd.dtype)
        gx = device.empty(tx.shape, xd.dtype) if need[0] else None
        gw = grad_buffer(tw, tw.shape, xd.dtype) if need[1] else None
        gb = grad_buffer(tb, (c_out,), xd.dtype) if tb is not None and need[2] else None
        scr = device.scratch(lib.tg_conv2d_backward_scratch_bytes(code, ref, int(gx is not None)))
        check(lib.tg_conv2d_backward(
            code, ref, g.ptr, cols.ptr, wd.ptr, gx.ptr if gx is not None else None,
            gw.ptr if gw is not None else None, gb.ptr if gb is not None else None, scr.ptr,
            device.stream()), "conv2d backward")
        if gx is not None and gx.dtype != tx.dtype and tx.dtype.kind == "f":
            gx = cast_array(gx, tx.dtype)
        return (gx, gw) if tb is None else (gx, gw, gb)

    def graph(g: Tensor, y_: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        gx = conv2d_input_grad(g, tw, tx.shape, st, pad) if need[0] else None
        gw = conv2d_weight_grad(tx, g, tw.shape, st, pad) if need[1] else None
        gb = reduce.sum(g, axis=(0, 2, 3)) if tb is not None and need[2] else None
        return (gx, gw) if tb is None else (gx, gw, gb)

    parents = (tx, tw) if tb is None else (tx, tw, tb)
    return make_result(y, parents, backward, "conv2d", graph)


def _grad_shape(input_shape: Any, weight_shape: Any, out: tuple[int, ...], st: tuple[int, int],
                pad: tuple[int, int], what: str) -> ConvShape:
    n, c, h, w = (int(v) for v in input_shape)
    c_out, c_w, kh, kw = (int(v) for v in weight_shape)
    if c_w != c:
        raise ValueError(f"{what}: input has {c} channels but weight expects {c_w}")
    s = _shape((n, c, h, w), c_out, (kh, kw), st, pad)
    if tuple(out) != (n, c_out, s.oh, s.ow):
        raise ValueError(f"{what}: output gradient of shape {tuple(out)}, expected "
                         f"{(n, c_out, s.oh, s.ow)}")
    return s


@profiled("conv2d_input_grad")
def conv2d_input_grad(grad_output: Any, weight: Any, input_shape: tuple[int, ...],
                      stride: IntPair = 1, padding: IntPair = 0) -> Tensor:
    """The gradient of ``conv2d(x, weight)`` with respect to ``x`` for an output gradient
    (a transposed convolution, ops/conv.py:180-213): ``(N, C_out, OH, OW)`` to
    ``input_shape``. Differentiable in both arguments."""
    tg_, tw = as_tensor(grad_output), as_tensor(weight)
    st, pad = _pair(stride, "stride"), _pair(padding, "padding")
    s = _grad_shape(input_shape, tw.shape, tg_.shape, st, pad, "conv2d_input_grad")
    gd, wd = _float_pair(tg_.data, tw.data)
    out = _input_grad_array(gd, wd, s)

    def backward(u: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        u = _cast(u, wd.dtype)
        # d/dg <u, T(g, w)> = conv(u, w); d/dw = the weight gradient of (u, g).
        g_u = _conv_array(u, wd, None, s)[0] if need[0] else None
        w_u = _weight_grad_array(_im2col(u, s), gd, s) if need[1] else None
        return g_u, w_u

    def graph(u: Tensor, y_: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        return (conv2d(u, tw, stride=st, padding=pad) if need[0] else None,
                conv2d_weight_grad(u, tg_, tw.shape, st, pad) if need[1] else None)

    return make_result(out, (tg_, tw), backward, "conv2d_input_grad", graph)


@profiled("conv2d_weight_grad")
def conv2d_weight_grad(x: Any, grad_output: Any, weight_shape: tuple[int, ...],
                       stride: IntPair = 1, padding: IntPair = 0) -> Tensor:
    """The gradient of ``conv2d(x, w)`` with respect to ``w`` for an output gradient
    (ops/conv.py:216-250): a ``weight_shape`` tensor. Differentiable in both arguments."""
    tx, tg_ = as_tensor(x), as_tensor(grad_output)
    st, pad = _pair(stride, "stride"), _pair(padding, "padding")
    if tx.ndim != 4:
        raise ValueError(f"conv2d_weight_grad expects 4-D input, got {tx.shape}")
    s = _grad_shape(tx.shape, weight_shape, tg_.shape, st, pad, "conv2d_weight_grad")
    xd, gd = _float_pair(tx.data, tg_.data)
    out = _weight_grad_array(_im2col(xd, s), gd, s)

    def backward(m: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        m = _cast(m, xd.dtype)
        # d/dx <m, W(x, g)> = the input gradient of (g, m); d/dg = conv(x, m).
        x_m = _input_grad_array(gd, m, s) if need[0] else None
        g_m = _conv_array(xd, m, None, s)[0] if need[1] else None
        return x_m, g_m

    def graph(m: Tensor, y_: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        return (conv2d_input_grad(tg_, m, tx.shape, st, pad) if need[0] else None,
                conv2d(tx, m, stride=st, padding=pad) if need[1] else None)

    return make_result(out, (tx, tg_), backward, "conv2d_weight_grad", graph)


class _Winners:
    """A pooling call's recorded winners, with the scatter (the VJP) and its adjoint gather
    as differentiable ops of their own."""

    def __init__(self, s: ConvShape, arg: DeviceArray, dtype: np.dtype[Any]) -> None:
        self.s, self.arg, self.dtype, self.code = s, arg, dtype, dtype_code(dtype)

    def scatter_array(self, g: DeviceArray) -> DeviceArray:
        s = self.s
        gx = device.empty((s.n, s.c, s.h, s.w), self.dtype)
        check(lib.tg_max_pool2d_backward(self.code, ctypes.byref(s), _cast(g, self.dtype).ptr,
                                         self.arg.ptr, gx.ptr, device.stream()),
              "max_pool2d backward")
        return gx

    def gather_array(self, u: DeviceArray) -> DeviceArray:
        s = self.s
        out = device.empty((s.n, s.c, s.oh, s.ow), self.dtype)
        check(lib.tg_max_pool2d_gather(self.code, ctypes.byref(s), _cast(u, self.dtype).ptr,
                                       self.arg.ptr, out.ptr, device.stream()),
              "max_pool2d gather")
        return out

    def scatter(self, g: Tensor) -> Tensor:
        return make_result(self.scatter_array(g.data), (g,),
                           lambda u, need: (self.gather_array(u),), "max_pool2d_scatter",
                           lambda u, y, need: (self.gather(u),))

    def gather(self, u: Tensor) -> Tensor:
        return make_result(self.gather_array(u.data), (u,),
                           lambda v, need: (self.scatter_array(v),), "max_pool2d_gather",
                           lambda v, y, need: (self.scatter(v),))


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
    y = device.empty((s.n, s.c, s.oh, s.ow), xd.dtype)
    arg = device.empty((s.n, s.c, s.oh, s.ow), np.uint8)
    check(lib.tg_max_pool2d_forward(code, ctypes.byref(s), xd.ptr, y.ptr, arg.ptr,
                                    device.stream()), "max_pool2d")
    winners = _Winners(s, arg, xd.dtype)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        return (winners.scatter_array(g),)

    def graph(g: Tensor, y_: Tensor, need: Need) -> tuple[Tensor]:
        # The winners are locally constant in x, so the VJP is linear in g alone.
        return (winners.scatter(g),)

    return make_result(y, (tx,), backward, "max_pool2d", graph)
