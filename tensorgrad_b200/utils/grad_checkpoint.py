"""Gradient checkpointing on the device: keep a function's output, recompute its insides in
the backward pass (the reference's utils/grad_checkpoint.py:39-135).

``checkpoint(fn, *args)`` runs ``fn`` with graph recording off, so none of the device buffers
its ops would save for their VJPs (attention probabilities, LayerNorm statistics, GELU
inputs, dropout masks ...) outlive the call; the result is one graph node whose parents are
the arguments and the parameters ``fn`` uses. When the backward pass reaches that node it
runs ``fn`` again with recording on and walks the fresh graph with the same engine, asking
only for the gradients the outer pass needs; the recomputed buffers are freed as that inner
walk goes. Checkpointing every block of a GPT keeps only the residual stream between blocks
alive, at the cost of one more forward pass per block.

Dropout masks come out identical in both passes: the device dropout kernels take their PCG64
state from the global generator, and the recomputation runs under a copy of the generator
taken just before the forward pass (a fresh copy for every recomputation, so a graph kept
with ``retain_graph`` replays the same masks each time). Under ``create_graph=True`` the
recomputed graph is connected to the original inputs through identity nodes and kept, so
second derivatives go through checkpoints too.
"""

from __future__ import annotations

import copy
from collections.abc import Callable, Iterable, Sequence
from typing import Any

from tensorgrad_b200 import autograd
from tensorgrad_b200._random import get_rng, replaying
from tensorgrad_b200.autograd import enable_grad, no_grad
from tensorgrad_b200.device import DeviceArray
from tensorgrad_b200.ops._util import as_tensor, identity, make_result
from tensorgrad_b200.tensor import Tensor

__all__ = ["checkpoint"]

Need = tuple[bool, ...]


def _unique(tensors: Iterable[Tensor]) -> list[Tensor]:
    seen: set[int] = set()
    out = []
    for t in tensors:
        if id(t) not in seen:
            seen.add(id(t))
            out.append(t)
    return out


def checkpoint(fn: Callable[..., Tensor], *args: Any, params: Iterable[Tensor] | None = None,
               preserve_rng_state: bool = True) -> Tensor:
    """``fn(*args)`` whose intermediate device buffers are not kept for the backward pass.

    Args:
        fn: A function of tensors returning one tensor, or a module.
        args: Its tensor arguments.
        params: Leaf tensors ``fn`` uses besides its arguments that need gradients; by
            default ``fn.parameters()`` when ``fn`` has that method, else none.
        preserve_rng_state: Recompute under a copy of the global generator taken before the
            forward pass, so dropout draws the same masks in both passes.

    Raises:
        ValueError: A tensor in ``params`` is not a leaf.
        TypeError: ``fn`` does not return a tensor.
        RuntimeError: In the backward pass, when ``fn`` used a tensor that requires grad and is
            neither an argument nor in ``params`` (its gradient would be lost).
    """
    inputs = [as_tensor(a) for a in args]
    if params is None:
        owned = getattr(fn, "parameters", None)
        params = owned() if callable(owned) else ()
    weights = _unique(params)
    for w in weights:
        if w._node is not None:
            raise ValueError("checkpoint params must be leaf tensors (parameters), got the "
                             f"result of op '{w._node.op}'")
    generator = copy.deepcopy(get_rng()) if preserve_rng_state else None
    with no_grad():
        out = fn(*inputs)
    if not isinstance(out, Tensor):
        raise TypeError(f"the checkpointed function must return a Tensor, got "
                        f"{type(out).__name__}")
    parents = (*inputs, *weights)

    def rerun(connect: bool) -> tuple[list[Tensor], Tensor]:
        """``fn`` again, recording a graph. Returns one tensor per parent to differentiate
        against (fresh leaves for the arguments, or identity nodes on them with ``connect``)
        and the recomputed output."""
        with enable_grad():
            if connect:
                leaves = [identity(x) if x._requires_grad else x for x in inputs]
            else:
                leaves = [Tensor._wrap(x.data).requires_grad_() if x._requires_grad else x
                          for x in inputs]
            if generator is None:
                y = fn(*leaves)
            else:
                with replaying(copy.deepcopy(generator)):
                    y = fn(*leaves)
        _check_captures(y, [*leaves, *weights])
        return [*leaves, *weights], y

    def backward(g: DeviceArray, need: Need) -> tuple[DeviceArray | None, ...]:
        wrt, y = rerun(connect=False)
        wanted = [t for t, n in zip(wrt, need, strict=True) if n]
        if not wanted or not y._requires_grad:
            return (None,) * len(wrt)
        # The same engine over the recomputed graph, gradients captured for ``wanted`` only
        # (nothing is accumulated into ``.grad`` there); the graph is freed as it goes.
        got = autograd._run_backward([y], [g], retain_graph=False, targets=wanted)
        return tuple(got.get(id(t)) if n else None for t, n in zip(wrt, need, strict=True))

    def graph(g: Tensor, y_out: Tensor, need: Need) -> tuple[Tensor | None, ...]:
        wrt, y = rerun(connect=True)
        wanted = [t for t, n in zip(wrt, need, strict=True) if n]
        if not wanted or not y._requires_grad:
            return (None,) * len(wrt)
        found = iter(autograd.grad(y, wanted, grad_outputs=g, create_graph=True,
                                   allow_unused=True))
        return tuple(next(found) if n else None for n in need)

    return make_result(out.data, parents, backward, "checkpoint", graph=graph)


def _check_captures(y: Tensor, allowed: Sequence[Tensor]) -> None:
    """Raise when the recomputed graph reaches a leaf that requires grad and is neither an
    argument nor a declared parameter: the outer pass has no edge to deliver its gradient."""
    stop = {id(t) for t in allowed}
    seen: set[int] = set()
    stack = [y]
    while stack:
        t = stack.pop()
        if id(t) in seen or id(t) in stop:
            continue
        seen.add(id(t))
        node = t._node
        if node is None:
            if t._requires_grad:
                raise RuntimeError(
                    f"the checkpointed function uses a tensor of shape {t.shape} that requires "
                    "grad but is neither an argument nor in params; its gradient would be lost")
            continue
        stack.extend(p for p in node.parents if p._requires_grad)
