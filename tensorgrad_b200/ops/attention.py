"""Fused scaled-dot-product attention (the reference's ops/attention.py:40-272).

``softmax(q k^T / sqrt(d) + causal mask) v`` as one graph node backed by the flash-style
kernels of ``attention.cu``: the forward keeps the output and one log-sum-exp per query row
instead of the ``(T_q, T_k)`` probabilities, and the VJP recomputes them.
:func:`packed_self_attention` reads Q, K and V as strided views of the packed ``(B, T, 3D)``
QKV projection and writes their gradients straight into one ``(B, T, 3D)`` buffer, as the
reference does.

Both are differentiable to any order (``create_graph=True``): their graph VJPs differentiate
the same function written with differentiable ops (``q k^T`` and ``P v`` products, the
softmax normalised against the forward's saved log-sum-exp, the causal mask as a ``-inf``
bias, the dropout keep-mask regenerated from the call's generator state as a constant), as
the reference's graph VJPs do (ops/attention.py:118-160). That path materialises the
``(T_q, T_k)`` probabilities; first-order training never takes it.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200._lib import AttnShape, check, lib
from tensorgrad_b200._random import dropout_threshold, get_rng, pcg64_take
from tensorgrad_b200.device import DeviceArray, dtype_code
from tensorgrad_b200.ops._util import (
    Need, as_tensor, constant, graph_by_composite, make_result, unbroadcast,
)
from tensorgrad_b200.ops.elementwise import cast_array
from tensorgrad_b200.profiler import profiled
from tensorgrad_b200.tensor import Tensor

__all__ = ["causal_mask", "packed_self_attention", "scaled_dot_product_attention"]


def causal_mask(q_len: int, k_len: int) -> np.ndarray:
    """Boolean mask, ``True`` where attention is forbidden (ops/attention.py:40-49)."""
    return np.triu(np.ones((q_len, k_len), dtype=np.bool_), k=1 + k_len - q_len)


def _shape(b: int, h: int, tq: int, tk: int, d: int, q: tuple[int, int, int],
           k: tuple[int, int, int], v: tuple[int, int, int], o: tuple[int, int, int],
           causal: bool) -> AttnShape:
    return AttnShape(b, h, tq, tk, d, *q, *k, *v, *o, 1 if causal else 0)


def _forward(shape: AttnShape, code: int, q: int, k: int, v: int, o: int, lse: int) -> None:
    scratch = device.scratch(lib.tg_attention_forward_scratch_bytes(code, shape))
    check(lib.tg_attention_forward(code, shape, q, k, v, o, lse, scratch.ptr, device.stream()),
          "attention")


def _backward(shape: AttnShape, code: int, q: int, k: int, v: int, o: int, lse: int, do: int,
              dq: int, dk: int, dv: int) -> None:
    scratch = device.scratch(lib.tg_attention_backward_scratch_bytes(code, shape))
    check(lib.tg_attention_backward(code, shape, q, k, v, o, lse, do, dq, dk, dv, scratch.ptr,
                                    device.stream()), "attention backward")


def _dropout_state(score_shape: tuple[int, ...], p: float, training: bool,
                   rng: np.random.Generator | None) -> tuple[np.ndarray, int, float] | None:
    """The attention-dropout draw (ops/attention.py:59-68): ``None`` when inactive, else the
    PCG64 state before the reference's keep-mask over ``score_shape`` (the host generator
    moves past the mask), the 16-bit threshold and the survivor scale."""
    if not training or p == 0.0:
        return None
    if not 0.0 <= p < 1.0:
        raise ValueError(f"attention dropout must be in [0, 1), got {p}")
    threshold, scale = dropout_threshold(p)
    if threshold >= 65536:  # every weight dropped: keep_mask draws nothing
        return np.zeros(4, np.uint64), threshold, scale
    state = pcg64_take(rng or get_rng(), (math.prod(score_shape) + 3) // 4)
    if state is None:
        raise NotImplementedError("attention dropout on the device needs a PCG64 generator "
                                  "(NumPy's default)")
    return state, threshold, scale


def _forward_dropout(shape: AttnShape, code: int, q: int, k: int, v: int, o: int, lse: int,
                     drop: tuple[np.ndarray, int, float]) -> None:
    state, threshold, scale = drop
    scratch = device.scratch(lib.tg_attention_dropout_scratch_bytes(code, shape))
    check(lib.tg_attention_forward_dropout(
        code, shape, q, k, v, o, lse, state.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)),
        threshold, scale, scratch.ptr, device.stream()), "attention (dropout)")


def _backward_dropout(shape: AttnShape, code: int, q: int, k: int, v: int, do: int, dq: int,
                      dk: int, dv: int, drop: tuple[np.ndarray, int, float]) -> None:
    state, threshold, scale = drop
    scratch = device.scratch(lib.tg_attention_dropout_scratch_bytes(code, shape))
    check(lib.tg_attention_backward_dropout(
        code, shape, q, k, v, do, dq, dk, dv,
        state.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), threshold, scale, scratch.ptr,
        device.stream()), "attention backward (dropout)")


def _causal_bias(n_q: int, n_k: int, dtype: np.dtype[Any]) -> Tensor:
    """0 where attention is allowed, ``-inf`` where the causal mask forbids it."""
    bias = np.where(causal_mask(n_q, n_k), -np.inf, 0.0).astype(dtype)
    return constant(device.from_numpy(bias))


def _keep_scaled(score_shape: tuple[int, ...], dtype: np.dtype[Any],
                 drop: tuple[np.ndarray, int, float]) -> Tensor:
    """The call's attention-dropout keep-mask times the survivor scale over ``score_shape``,
    regenerated from its PCG64 state (the same element order as the fused kernels)."""
    from tensorgrad_b200.ops.shape import broadcast_array

    state, threshold, scale = drop
    ones = broadcast_array(device.scalar_like(1.0, dtype), score_shape)
    out = device.empty(score_shape, dtype)
    check(lib.tg_dropout_pcg64(dtype_code(dtype), ones.size, ones.ptr, out.ptr,
                               state.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), 0,
                               threshold, scale, device.stream()), "attention dropout mask")
    return constant(out)


def _composite(q: Tensor, k: Tensor, v: Tensor, bias: Tensor | None, lse: Tensor,
               keep: Tensor | None) -> Tensor:
    """Attention in differentiable ops: ``softmax(q k^T / sqrt(d) + bias) [* keep] v`` with
    the softmax shifted by the forward's row log-sum-exp (a constant: any shift gives the same
    function, this one keeps every exponent <= 0)."""
    from tensorgrad_b200.ops import elementwise as E
    from tensorgrad_b200.ops import reduce as R
    from tensorgrad_b200.ops.linalg import matmul
    from tensorgrad_b200.ops.shape import transpose

    scores = E.mul(matmul(q, transpose(k, -1, -2)), 1.0 / math.sqrt(q.shape[-1]))
    if bias is not None:
        scores = E.add(scores, bias)
    e = E.exp(E.sub(scores, lse))
    p = E.div(e, R.sum(e, -1, keepdims=True))
    if keep is not None:
        p = E.mul(p, keep)
    return matmul(p, v)


def _unfused_attention(tq: Tensor, tk: Tensor, tv: Tensor, causal: bool, mask: Any,
                       dropout_p: float, training: bool,
                       rng: np.random.Generator | None) -> Tensor:
    """``softmax(q k^T / sqrt(d)`` with forbidden scores at ``-inf``) ``[* keep] v`` in
    differentiable ops (matmul, masked_fill, softmax), for masks and value widths the fused
    kernels do not take (ops/attention.py:52-90, 163-208)."""
    from tensorgrad_b200.ops import elementwise as E
    from tensorgrad_b200.ops.activation import softmax
    from tensorgrad_b200.ops.linalg import matmul
    from tensorgrad_b200.ops.shape import masked_fill, transpose

    n_q, n_k, d = tq.shape[-2], tk.shape[-2], tq.shape[-1]
    if tk.shape[-1] != d or tv.shape[-2] != n_k:
        raise ValueError(f"attention: incompatible q {tq.shape}, k {tk.shape}, v {tv.shape}")
    forbidden = None
    if mask is not None:
        m = mask.numpy() if isinstance(mask, Tensor) else mask
        forbidden = np.asarray(m, dtype=np.bool_)
    if causal:
        cm = causal_mask(n_q, n_k)
        forbidden = cm if forbidden is None else forbidden | cm
    batch = tuple(np.broadcast_shapes(tq.shape[:-2], tk.shape[:-2]))
    drop = _dropout_state((*batch, n_q, n_k), dropout_p, training, rng)
    scores = E.mul(matmul(tq, transpose(tk, -1, -2)), 1.0 / math.sqrt(d))
    if forbidden is not None:
        scores = masked_fill(scores, forbidden, -np.inf)
    weights = softmax(scores, -1)
    if drop is not None:
        weights = E.mul(weights, _keep_scaled((*batch, n_q, n_k), weights.dtype, drop))
    return matmul(weights, tv)


def _as_bhtd(shape: tuple[int, ...]) -> tuple[int, int]:
    """(B, H) of a ``(..., T, d)`` array: the batch axes collapse into B (and H = 1) unless
    there are exactly two."""
    lead = shape[:-2]
    if len(lead) == 2:
        return lead[0], lead[1]
    return math.prod(lead), 1


@profiled("attention")
def scaled_dot_product_attention(
    q: Any, k: Any, v: Any, *, causal: bool = False, mask: Any = None, dropout_p: float = 0.0,
    training: bool = False, rng: np.random.Generator | None = None,
) -> Tensor:
    """``softmax(q k^T / sqrt(d)) v`` over the last two axes, fused (ops/attention.py:163-208).

    ``q, k, v`` share their batch axes, or ``k``/``v`` broadcast over them (e.g. shared
    across heads); their gradients are then summed back (ops/attention.py:211-213). Dropout
    on the attention weights (``training`` and ``dropout_p > 0``) uses the reference's
    keep-mask, generated on the device from the global (or given) PCG64 generator and
    regenerated by the VJP. An extra boolean ``mask`` (broadcastable to the scores, ``True``
    = forbidden, combined with ``causal``) or values of another width than the queries take
    the unfused path: the same function in differentiable device ops, the scores
    materialised.
    """
    tq, tk, tv = as_tensor(q), as_tensor(k), as_tensor(v)
    if mask is not None or tv.shape[-1] != tq.shape[-1]:
        return _unfused_attention(tq, tk, tv, causal, mask, dropout_p, training, rng)
    dt = np.result_type(tq.dtype, tk.dtype, tv.dtype)
    qd, kd, vd = (t.data if t.dtype == dt else cast_array(t.data, dt) for t in (tq, tk, tv))
    batch = tuple(np.broadcast_shapes(tq.shape[:-2], tk.shape[:-2], tv.shape[:-2]))
    n_q, d = tq.shape[-2], tq.shape[-1]
    n_k = tk.shape[-2]
    if tk.shape[-1] != d or tv.shape[-1] != d or tv.shape[-2] != n_k:
        raise ValueError(f"attention: incompatible q {tq.shape}, k {tk.shape}, v {tv.shape}")
    full_shapes = [(*batch, n_q, d), (*batch, n_k, d), (*batch, n_k, d)]

    def materialise(a: DeviceArray, full: tuple[int, ...]) -> DeviceArray:
        if a.shape == full:
            return a
        from tensorgrad_b200.ops.shape import broadcast_array

        return broadcast_array(a, full)

    qf, kf, vf = (materialise(a, s) for a, s in zip((qd, kd, vd), full_shapes, strict=True))
    b, h = _as_bhtd(full_shapes[0])
    qs = (h * n_q * d, n_q * d, d)
    ks = (h * n_k * d, n_k * d, d)
    shp = _shape(b, h, n_q, n_k, d, qs, ks, ks, qs, causal)
    code = dtype_code(dt)
    drop = _dropout_state((*batch, n_q, n_k), dropout_p, training, rng)
    out = device.empty(full_shapes[0], dt)
    lse = device.empty((b * h * n_q,), dt)
    if drop is None:
        _forward(shp, code, qf.ptr, kf.ptr, vf.ptr, out.ptr, lse.ptr)
    else:
        _forward_dropout(shp, code, qf.ptr, kf.ptr, vf.ptr, out.ptr, lse.ptr, drop)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        if g.dtype != dt:
            g = cast_array(g, dt)
        dq = device.empty(full_shapes[0], dt)
        dk = device.empty(full_shapes[1], dt)
        dv = device.empty(full_shapes[2], dt)
        if drop is None:
            _backward(shp, code, qf.ptr, kf.ptr, vf.ptr, out.ptr, lse.ptr, g.ptr, dq.ptr,
                      dk.ptr, dv.ptr)
        else:
            _backward_dropout(shp, code, qf.ptr, kf.ptr, vf.ptr, g.ptr, dq.ptr, dk.ptr, dv.ptr,
                              drop)
        grads = []
        for gr, t, wanted in zip((dq, dk, dv), (tq, tk, tv), need, strict=True):
            if not wanted:
                grads.append(None)
                continue
            gr = unbroadcast(gr, t.shape)
            grads.append(gr if gr.dtype == t.dtype else cast_array(gr, t.dtype))
        return tuple(grads)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        bias = _causal_bias(n_q, n_k, dt) if causal else None
        keep = None if drop is None else _keep_scaled((*batch, n_q, n_k), dt, drop)
        lse_t = constant(lse.reshape((*batch, n_q, 1)))
        return graph_by_composite((tq, tk, tv),
                                  lambda a, b_, c: _composite(a, b_, c, bias, lse_t, keep),
                                  g, need)

    return make_result(out, (tq, tk, tv), backward, "attention", graph)


@profiled("self_attention")
def packed_self_attention(
    qkv: Any, num_heads: int, *, causal: bool = True, dropout_p: float = 0.0,
    training: bool = False, rng: np.random.Generator | None = None,
) -> Tensor:
    """Multi-head self-attention on a packed ``(B, T, 3 * D)`` QKV projection; returns merged
    heads ``(B, T, D)`` (ops/attention.py:223-272). Attention dropout as in
    :func:`scaled_dot_product_attention`, with the mask over ``(B, H, T, T)``."""
    tqkv = as_tensor(qkv)
    if tqkv.ndim != 3 or tqkv.shape[-1] % (3 * num_heads):
        raise ValueError(
            f"expected (B, T, 3 * D) with D divisible by {num_heads}, got {tqkv.shape}"
        )
    b, t, d3 = tqkv.shape
    d = d3 // 3
    hd = d // num_heads
    x = tqkv.data
    code = dtype_code(x.dtype)
    es = x.itemsize
    src = (t * d3, hd, d3)           # strides of q, k, v inside the packed buffer
    dst = (t * d, hd, d)             # strides of the merged-head output
    shp = _shape(b, num_heads, t, t, hd, src, src, src, dst, causal)
    drop = _dropout_state((b, num_heads, t, t), dropout_p, training, rng)
    out = device.empty((b, t, d), x.dtype)
    lse = device.empty((b * num_heads * t,), x.dtype)
    base = x.ptr
    if drop is None:
        _forward(shp, code, base, base + d * es, base + 2 * d * es, out.ptr, lse.ptr)
    else:
        _forward_dropout(shp, code, base, base + d * es, base + 2 * d * es, out.ptr, lse.ptr,
                         drop)

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray]:
        if g.dtype != x.dtype:
            g = cast_array(g, x.dtype)
        dqkv = device.empty((b, t, d3), x.dtype)
        gb = dqkv.ptr
        if drop is None:
            _backward(shp, code, base, base + d * es, base + 2 * d * es, out.ptr, lse.ptr,
                      g.ptr, gb, gb + d * es, gb + 2 * d * es)
        else:
            _backward_dropout(shp, code, base, base + d * es, base + 2 * d * es, g.ptr, gb,
                              gb + d * es, gb + 2 * d * es, drop)
        return (dqkv,)

    def graph(g: Tensor, y: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        from tensorgrad_b200.ops.shape import permute, reshape

        bias = _causal_bias(t, t, x.dtype) if causal else None
        keep = None if drop is None else _keep_scaled((b, num_heads, t, t), x.dtype, drop)
        lse_t = constant(lse.reshape((b, num_heads, t, 1)))

        def composite(packed: Tensor) -> Tensor:
            parts = permute(reshape(packed, (b, t, 3, num_heads, hd)), (2, 0, 3, 1, 4))
            o = _composite(parts[0], parts[1], parts[2], bias, lse_t, keep)
            return reshape(permute(o, (0, 2, 1, 3)), (b, t, d))

        return graph_by_composite((tqkv,), composite, g, need)

    return make_result(out, (tqkv,), backward, "self_attention", graph)
