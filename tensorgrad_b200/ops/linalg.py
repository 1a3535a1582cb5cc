"""Matrix product (the reference's ops/linalg.py:16-63) on the GEMM kernels."""

from __future__ import annotations

import math
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import check, lib
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import Need, coerce_pair, make_result, unbroadcast
from tensorgrad_b200.ops.elementwise import cast_array
from tensorgrad_b200.ops.shape import broadcast_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["matmul"]


def _bmm(a: DeviceArray, b: DeviceArray, ta: int, tb: int, m: int, n: int, k: int,
         batch: int) -> DeviceArray:
    """``batch`` products op(a_i) @ op(b_i) of contiguous stacks."""
    out = device.empty((batch, m, n), a.dtype)
    lda = m if ta else k
    ldb = k if tb else n
    check(lib.tg_gemm_batched(dtype_code(a.dtype), ta, tb, m, n, k, 1.0, a.ptr, lda, m * k,
                              b.ptr, ldb, k * n, 0.0, out.ptr, n, m * n, batch,
                              device.stream()), "matmul")
    return out


@profiled("matmul")
def matmul(a: Any, b: Any) -> Tensor:
    """``a @ b`` with NumPy's rules (ops/linalg.py:16-63): leading axes broadcast; a 1-D
    ``a`` is a row and a 1-D ``b`` a column, whose axis is dropped from the result (two
    vectors give their dot product)."""
    ta, tb = coerce_pair(a, b)
    if ta.ndim == 0 or tb.ndim == 0:
        raise ValueError("matmul does not accept 0-d tensors; use mul instead")
    dt = np.result_type(ta.dtype, tb.dtype)
    ad = ta.data if ta.dtype == dt else cast_array(ta.data, dt)
    bd = tb.data if tb.dtype == dt else cast_array(tb.data, dt)
    a_vec, b_vec = ta.ndim == 1, tb.ndim == 1
    a2 = ad.reshape((1, ad.shape[0])) if a_vec else ad
    b2 = bd.reshape((bd.shape[0], 1)) if b_vec else bd
    m, k = a2.shape[-2:]
    k2, n = b2.shape[-2:]
    if k != k2:
        raise ValueError(f"matmul: shapes {ta.shape} and {tb.shape} are not aligned")
    batch = tuple(np.broadcast_shapes(a2.shape[:-2], b2.shape[:-2]))
    nb = math.prod(batch)
    af = broadcast_array(a2, (*batch, m, k))
    bf = broadcast_array(b2, (*batch, k, n))
    full = (*batch, m, n)
    shape = (*batch, *(() if a_vec else (m,)), *(() if b_vec else (n,)))
    out = _bmm(af, bf, 0, 0, m, n, k, nb).reshape(shape)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, DeviceArray | None]:
        g = g.reshape(full)
        ga = gb = None
        if need[0]:  # g @ b^T
            ga = unbroadcast(_bmm(g, bf, 0, 1, m, k, n, nb).reshape((*batch, m, k)), a2.shape)
            ga = ga.reshape(ta.shape)
        if need[1]:  # a^T @ g
            gb = unbroadcast(_bmm(af, g, 1, 0, k, n, m, nb).reshape((*batch, k, n)), b2.shape)
            gb = gb.reshape(tb.shape)
        return ga, gb

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, Tensor | None]:
        from tensorgrad_b200.ops.shape import reshape, sum_to, transpose

        g2 = reshape(g, full)
        ra = reshape(ta, a2.shape) if a_vec else ta
        rb = reshape(tb, b2.shape) if b_vec else tb
        ga = reshape(sum_to(matmul(g2, transpose(rb, -1, -2)), a2.shape), ta.shape) \
            if need[0] else None
        gb = reshape(sum_to(matmul(transpose(ra, -1, -2), g2), b2.shape), tb.shape) \
            if need[1] else None
        return ga, gb

    return make_result(out, (ta, tb), backward, "matmul", graph)
