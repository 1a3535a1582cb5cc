"""Finite-difference checks of first (:func:`gradcheck`) and second (:func:`gradgradcheck`)
derivatives of device functions (the reference's utils/gradcheck.py:19-192).

The function's output is projected onto fixed random weights, so the whole vector-Jacobian
product is checked, not only the gradient of a sum. Central differences perturb one element
of a device input at a time (one 8-byte host-to-device write per perturbation) and evaluate
the projection on the device; only the scalar projections and the compared gradients come
back to the host. Inputs that are checked must be float64.
"""

from __future__ import annotations

import ctypes
from collections.abc import Callable, Sequence

import numpy as np

from tensorgrad_b200 import autograd, device
from tensorgrad_b200._lib import check, lib
from tensorgrad_b200.autograd import enable_grad, no_grad
from tensorgrad_b200.tensor import Tensor

__all__ = ["GradcheckError", "gradcheck", "gradgradcheck", "numerical_grad"]


class GradcheckError(AssertionError):
    """Analytical and numerical derivatives disagree."""


def _projection(fn: Callable[..., Tensor], inputs: Sequence[Tensor], weights: Tensor) -> float:
    with no_grad():
        return float((fn(*inputs) * weights).sum().item())


def _write(x: Tensor, i: int, value: np.ndarray) -> None:
    """Element ``i`` (flat) of ``x``'s device data := ``value`` (a 0-d host array)."""
    data = x.data
    check(lib.tg_memcpy_h2d(ctypes.c_void_p(data.ptr + i * data.itemsize),
                            value.ctypes.data_as(ctypes.c_void_p), data.itemsize,
                            device.stream()), "gradcheck perturbation")
    device.synchronize()  # the host scalar must outlive the copy


def numerical_grad(fn: Callable[..., Tensor], inputs: Sequence[Tensor], index: int,
                   weights: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """Central-difference estimate of ``d sum(fn(*inputs) * weights) / d inputs[index]``;
    the input is perturbed in place on the device and restored."""
    x = inputs[index]
    original = x.numpy().reshape(-1)
    w = Tensor(np.asarray(weights))
    grad = np.zeros(original.size, dtype=np.float64)
    for i in range(original.size):
        v = original[i]
        _write(x, i, np.asarray(v + eps, dtype=original.dtype))
        plus = _projection(fn, inputs, w)
        _write(x, i, np.asarray(v - eps, dtype=original.dtype))
        minus = _projection(fn, inputs, w)
        _write(x, i, np.asarray(v, dtype=original.dtype))
        grad[i] = (plus - minus) / (2 * eps)
    return grad.reshape(x.shape)


def _agree(analytical: np.ndarray, expected: np.ndarray, what: str, atol: float, rtol: float,
           raise_exception: bool) -> bool:
    if np.allclose(analytical, expected, atol=atol, rtol=rtol):
        return True
    if not raise_exception:
        return False
    diff = np.abs(analytical - expected)
    worst = np.unravel_index(int(np.argmax(diff)), diff.shape) if diff.ndim else ()
    raise GradcheckError(
        f"{what}: max abs diff {diff.max():.3e} at {worst}; "
        f"analytical={np.asarray(analytical)[worst]!r}, expected={np.asarray(expected)[worst]!r}"
    )


def _checked(inputs: Sequence[Tensor], name: str) -> list[int]:
    idx = [i for i, t in enumerate(inputs) if t.requires_grad]
    if not idx:
        raise ValueError(f"{name} needs at least one input with requires_grad=True")
    for i in idx:
        if inputs[i].dtype != np.float64:
            raise TypeError(f"{name} input {i} is {inputs[i].dtype}; use float64")
    return idx


def gradcheck(fn: Callable[..., Tensor], inputs: Sequence[Tensor], *, eps: float = 1e-6,
              atol: float = 1e-6, rtol: float = 1e-4, seed: int = 0,
              raise_exception: bool = True) -> bool:
    """Backpropagated gradients of ``sum(fn(*inputs) * w)`` (``w`` fixed random weights)
    against central finite differences, for every input with ``requires_grad`` (float64).
    Returns ``True``, or raises :class:`GradcheckError` (``False`` with
    ``raise_exception=False``) on a mismatch."""
    idx = _checked(inputs, "gradcheck")
    for t in inputs:
        t.zero_grad()
    out = fn(*inputs)
    weights = np.random.default_rng(seed).standard_normal(out.shape)
    (out * Tensor(weights)).sum().backward()
    for i in idx:
        grad = inputs[i].grad
        analytical = np.zeros(inputs[i].shape) if grad is None else grad.numpy()
        numerical = numerical_grad(fn, inputs, i, weights, eps)
        what = f"gradient mismatch for input {i} (shape {inputs[i].shape})"
        if not _agree(analytical, numerical, what, atol, rtol, raise_exception):
            return False
    return True


def gradgradcheck(fn: Callable[..., Tensor], inputs: Sequence[Tensor], *, eps: float = 1e-6,
                  atol: float = 1e-5, rtol: float = 1e-4, seed: int = 0,
                  raise_exception: bool = True) -> bool:
    """Second derivatives: with a fixed random cotangent ``v``, the differentiable VJP
    ``G(x, v) = J(x)^T v`` (``create_graph=True``) must equal the plain VJP, and
    :func:`gradcheck` of ``G`` in both ``x`` and ``v`` must pass (double backward against
    central differences of the gradient)."""
    from tensorgrad_b200.ops.shape import concat, reshape

    idx = _checked(inputs, "gradgradcheck")
    wrt = [inputs[i] for i in idx]
    with enable_grad():
        out = fn(*inputs)
    v = np.random.default_rng(seed + 1).standard_normal(out.shape)
    with enable_grad():
        plain = autograd.grad(fn(*inputs), wrt, grad_outputs=v, allow_unused=True)
        graph = autograd.grad(fn(*inputs), wrt, grad_outputs=Tensor(v), create_graph=True,
                              allow_unused=True)
    for i, f, g in zip(idx, plain, graph, strict=True):
        zeros = np.zeros(inputs[i].shape)
        what = f"create_graph VJP disagrees with the plain VJP for input {i}"
        f_arr = zeros if f is None else f.numpy()
        g_arr = zeros if g is None else g.numpy()
        if not _agree(g_arr, f_arr, what, 1e-12, 1e-10, raise_exception):
            return False

    def first_derivative(*args: Tensor) -> Tensor:
        *xs, cotangent = args
        with enable_grad():
            grads = autograd.grad(fn(*xs), [xs[i] for i in idx], grad_outputs=cotangent,
                                  create_graph=True, allow_unused=True)
        flat = [reshape(Tensor(np.zeros(xs[i].shape)) if g is None else g, (-1,))
                for i, g in zip(idx, grads, strict=True)]
        return concat(flat)

    return gradcheck(first_derivative, [*inputs, Tensor(v, requires_grad=True)], eps=eps,
                     atol=atol, rtol=rtol, seed=seed + 2, raise_exception=raise_exception)
