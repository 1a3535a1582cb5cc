"""Function transforms on the device engine (API of the reference's func.py): ``grad``,
``value_and_grad``, ``vjp``, ``jvp``, ``jacobian``, ``hessian``, ``hvp``.

Each transform runs the function with grad mode on, differentiates with respect to a fresh
alias of every differentiated argument (an identity op on top of it, so nested transforms
differentiate only through their own argument), and returns results that carry a graph
exactly when grad mode is on at the call (``create_graph`` then). Forward-mode products use
two reverse passes: ``u -> J^T u`` is linear in ``u``, so its VJP in direction ``v`` is
``J v``. Every gradient is built from the ops' differentiable VJPs, so the functions may use
the elementwise, matrix, reduction, shape, linear and cross-entropy ops (the fused
attention, layer-norm, convolution and recurrent kernels have none and raise).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from typing import Any, TypeAlias

import numpy as np

from tensorgrad_b200 import autograd, device
from tensorgrad_b200.autograd import enable_grad, is_grad_enabled
from tensorgrad_b200.tensor import Tensor

__all__ = ["grad", "hessian", "hvp", "jacobian", "jvp", "value_and_grad", "vjp"]

TensorLike: TypeAlias = Tensor | np.ndarray | float
Argnums: TypeAlias = int | tuple[int, ...]


def _tensor(value: TensorLike) -> Tensor:
    return value if isinstance(value, Tensor) else Tensor(value)


def _alias(x: Tensor) -> Tensor:
    """The tensor to differentiate with respect to: a fresh leaf over ``x``'s storage, or, when
    ``x`` already has a graph, an identity op on top of it (results stay differentiable in
    ``x``)."""
    from tensorgrad_b200.ops._util import make_result

    if not x.requires_grad:
        return Tensor._wrap(x.data).requires_grad_()
    return make_result(x.data, (x,), lambda g, need: (g,), "alias",
                       lambda g, y, need: (g,))


def _zeros(x: Tensor) -> Tensor:
    return Tensor._wrap(device.zeros(x.shape, x.dtype))


def _pull(outputs: Sequence[Tensor], inputs: Sequence[Tensor],
          cotangents: Sequence[Any] | None, *, create_graph: bool,
          retain_graph: bool | None = None) -> tuple[Tensor, ...]:
    """``autograd.grad`` with zeros for inputs nothing depends on."""
    idx = [i for i, o in enumerate(outputs) if o.requires_grad]
    if not idx:
        return tuple(_zeros(x) for x in inputs)
    seeds = None if cotangents is None else [cotangents[i] for i in idx]
    got = autograd.grad([outputs[i] for i in idx], list(inputs), grad_outputs=seeds,
                        retain_graph=retain_graph, create_graph=create_graph,
                        allow_unused=True)
    return tuple(_zeros(x) if g is None else g for x, g in zip(inputs, got, strict=True))


def _positions(argnums: Argnums, count: int) -> tuple[int, ...]:
    pos = (argnums,) if isinstance(argnums, int) else tuple(argnums)
    if not pos:
        raise ValueError("argnums must name at least one argument")
    for p in pos:
        if not -count <= p < count:
            raise IndexError(f"argnums {p} is out of range for {count} arguments")
    return pos


def _with_aliases(args: Sequence[TensorLike], argnums: Argnums) -> tuple[list[Tensor], list[Tensor]]:
    tensors = [_tensor(a) for a in args]
    wrt = []
    for p in _positions(argnums, len(tensors)):
        tensors[p] = _alias(tensors[p])
        wrt.append(tensors[p])
    return tensors, wrt


def _shape_result(values: tuple[Tensor, ...], argnums: Argnums) -> Tensor | tuple[Tensor, ...]:
    return values[0] if isinstance(argnums, int) else values


def _settle(value: Tensor, keep_graph: bool) -> Tensor:
    return value if keep_graph else value.detach()


def value_and_grad(f: Callable[..., Tensor], argnums: Argnums = 0
                   ) -> Callable[..., tuple[Tensor, Tensor | tuple[Tensor, ...]]]:
    """``f`` and its gradient at once: the new function returns ``(f(*args), gradient)``."""

    def run(*args: TensorLike) -> tuple[Tensor, Tensor | tuple[Tensor, ...]]:
        keep = is_grad_enabled()
        with enable_grad():
            tensors, wrt = _with_aliases(args, argnums)
            out = f(*tensors)
            if not isinstance(out, Tensor) or out.size != 1:
                shape = getattr(out, "shape", type(out).__name__)
                raise ValueError(f"grad needs a function returning one scalar, got {shape}")
            grads = _pull([out], wrt, None, create_graph=keep)
        return _settle(out, keep), _shape_result(grads, argnums)

    return run


def grad(f: Callable[..., Tensor], argnums: Argnums = 0) -> Callable[..., Any]:
    """The gradient of the scalar function ``f`` with respect to argument(s) ``argnums``."""
    both = value_and_grad(f, argnums)
    return lambda *args: both(*args)[1]


def vjp(f: Callable[..., Tensor], *primals: TensorLike
        ) -> tuple[Tensor, Callable[[TensorLike], tuple[Tensor, ...]]]:
    """``f(*primals)`` and ``u -> (u^T df/dprimal_i)_i`` (callable repeatedly)."""
    keep = is_grad_enabled()
    with enable_grad():
        xs = [_alias(_tensor(p)) for p in primals]
        out = f(*xs)

    def pullback(cotangent: TensorLike) -> tuple[Tensor, ...]:
        with enable_grad():
            return _pull([out], xs, [_tensor(cotangent)], create_graph=is_grad_enabled(),
                         retain_graph=True)

    return _settle(out, keep), pullback


def jvp(f: Callable[..., Tensor], primals: Sequence[TensorLike],
        tangents: Sequence[TensorLike]) -> tuple[Tensor, Tensor]:
    """``f(*primals)`` and the Jacobian-vector product ``sum_i J_i v_i`` (two reverse passes:
    the VJP with a dummy cotangent ``u``, built with a graph, is linear in ``u``)."""
    if len(primals) != len(tangents):
        raise ValueError(f"got {len(primals)} primals but {len(tangents)} tangents")
    keep = is_grad_enabled()
    with enable_grad():
        xs = [_alias(_tensor(p)) for p in primals]
        vs = [_tensor(t) for t in tangents]
        for x, v in zip(xs, vs, strict=True):
            if x.shape != v.shape:
                raise ValueError(f"tangent shape {v.shape} does not match primal {x.shape}")
        out = f(*xs)
        u = _zeros(out).requires_grad_()
        pulled = _pull([out], xs, [u], create_graph=True)
        live = [(g, v) for g, v in zip(pulled, vs, strict=True) if g.requires_grad]
        if not live:
            return _settle(out, keep), _zeros(out)
        (forward,) = _pull([g for g, _ in live], [u], [v for _, v in live], create_graph=keep)
    return _settle(out, keep), forward


def jacobian(f: Callable[..., Any], argnums: Argnums = 0) -> Callable[..., Any]:
    """The Jacobian of ``f`` by reverse mode, one backward pass per output element: shape
    ``O + I`` for an output of shape ``O`` and an argument of shape ``I``; a tuple result
    for a function returning a tuple."""
    from tensorgrad_b200.ops.shape import reshape, stack

    def run(*args: TensorLike) -> Any:
        keep = is_grad_enabled()
        with enable_grad():
            tensors, wrt = _with_aliases(args, argnums)
            result = f(*tensors)
            outputs = result if isinstance(result, tuple) else (result,)
            blocks_per_output = []
            for out in outputs:
                rows = []
                for i in range(out.size):
                    seed = np.zeros(out.size, dtype=out.dtype)
                    seed[i] = 1.0
                    rows.append(_pull([out], wrt, [seed.reshape(out.shape)], create_graph=keep,
                                      retain_graph=True))
                blocks = tuple(
                    reshape(stack([row[j] for row in rows]), out.shape + x.shape) if rows
                    else Tensor._wrap(device.zeros(out.shape + x.shape, out.dtype))
                    for j, x in enumerate(wrt))
                if not keep:
                    blocks = tuple(b.detach() for b in blocks)
                blocks_per_output.append(_shape_result(blocks, argnums))
        return tuple(blocks_per_output) if isinstance(result, tuple) else blocks_per_output[0]

    return run


def hessian(f: Callable[..., Tensor], argnums: Argnums = 0) -> Callable[..., Any]:
    """The Hessian of the scalar ``f``: ``jacobian(grad(f))``."""
    return jacobian(grad(f, argnums), argnums)


def hvp(f: Callable[..., Tensor], primals: Sequence[TensorLike],
        tangents: Sequence[TensorLike]) -> tuple[Tensor, tuple[Tensor, ...]]:
    """``f(*primals)`` and the Hessian-vector products ``H v`` (reverse over reverse:
    ``d <grad f, v> / dx``, no Hessian materialised)."""
    if len(primals) != len(tangents):
        raise ValueError(f"got {len(primals)} primals but {len(tangents)} tangents")
    keep = is_grad_enabled()
    with enable_grad():
        xs = [_alias(_tensor(p)) for p in primals]
        vs = [_tensor(t) for t in tangents]
        out = f(*xs)
        if out.size != 1:
            raise ValueError(f"hvp needs a function returning one scalar, got shape {out.shape}")
        grads = _pull([out], xs, None, create_graph=True)
        terms = [(g * v).sum() for g, v in zip(grads, vs, strict=True) if g.requires_grad]
        if not terms:
            return _settle(out, keep), tuple(_zeros(x) for x in xs)
        total = terms[0]
        for term in terms[1:]:
            total = total + term
        products = _pull([total], xs, None, create_graph=keep)
    return _settle(out, keep), products
