"""The reverse-mode engine: graph nodes, grad mode, ``backward`` and ``grad``.

Same contract as the reference engine (autograd.py:119-465 of tensorgrad 0.2.0): a
:class:`Node` holds an op's parents and its VJP closure; the engine walks the tensors that
require grad in reverse topological order (iterative post-order DFS), sums fan-out
contributions, accumulates leaf gradients, and frees each node's saved state unless
``retain_graph``. The walk runs on the host; the gradients it carries are device arrays and
every sum is a device kernel. Error messages match the reference's, word for word.

``create_graph=True`` runs a second walk whose gradients are tensors built from differentiable
device ops (each op's ``graph`` VJP), so they carry their own graph and can be differentiated
again (double backward, ``func.hessian`` ...). Every op has one: the fused kernels (attention,
layer and batch norm, convolution, pooling, recurrent layers, dropout, embedding) give theirs
as differentiable ops of their own or as the same function composed of differentiable ops. A
hook lets data-parallel training start a gradient all-reduce the moment a leaf's gradient is
final.
"""

from __future__ import annotations

import functools
import threading
from collections.abc import Callable, Sequence
from typing import TYPE_CHECKING, Any, TypeAlias, TypeVar

import numpy as np

from tensorgrad_b200 import profiler as _profiler

if TYPE_CHECKING:
    from tensorgrad_b200.device import DeviceArray
    from tensorgrad_b200.tensor import Tensor

__all__ = ["BackwardFn", "GradOutputs", "Node", "backward", "enable_grad", "grad", "is_grad_enabled",
           "no_grad"]

#: VJP of one op on device arrays: given d(loss)/d(output) and, per input, whether its
#: gradient is needed, return d(loss)/d(input_i) (``None`` where not needed).
BackwardFn = Callable[["DeviceArray", tuple[bool, ...]], tuple["DeviceArray | None", ...]]
#: The same VJP written with differentiable tensor ops: ``graph(g, out, need)`` with the
#: output tensor ``out``; used when gradients must carry a graph (``create_graph=True``).
GraphFn = Callable[["Tensor", "Tensor", tuple[bool, ...]], tuple["Tensor | None", ...]]
GradOutputs: TypeAlias = "Tensor | np.ndarray | Sequence[Tensor | np.ndarray | None] | None"

_R = TypeVar("_R")


class _GradMode(threading.local):
    enabled: bool = True


_grad_mode = _GradMode()


def is_grad_enabled() -> bool:
    """Return ``True`` if ops currently record the graph needed for ``backward``."""
    return _grad_mode.enabled


class _GradModeContext:
    _target: bool

    def __init__(self) -> None:
        self._previous: list[bool] = []

    def __enter__(self) -> None:
        self._previous.append(_grad_mode.enabled)
        _grad_mode.enabled = self._target

    def __exit__(self, *exc: object) -> None:
        _grad_mode.enabled = self._previous.pop()

    def __call__(self, fn: Callable[..., _R]) -> Callable[..., _R]:
        @functools.wraps(fn)
        def wrapper(*args: Any, **kwargs: Any) -> _R:
            with type(self)():
                return fn(*args, **kwargs)

        return wrapper


class no_grad(_GradModeContext):  # noqa: N801
    """Disable graph recording (context manager or decorator)."""

    _target = False


class enable_grad(_GradModeContext):  # noqa: N801
    """Re-enable graph recording inside a :class:`no_grad` region."""

    _target = True


class Node:
    """A recorded op: its inputs and the VJP that maps the output gradient to theirs."""

    __slots__ = ("_backward", "_graph", "op", "parents")

    def __init__(self, op: str, parents: tuple[Tensor, ...], backward: BackwardFn,
                 graph_backward: GraphFn | None = None) -> None:
        self.op = op
        self.parents = parents
        self._backward: BackwardFn | None = backward
        self._graph: GraphFn | None = graph_backward

    @property
    def released(self) -> bool:
        """``True`` once a backward pass without ``retain_graph`` freed the saved state."""
        return self._backward is None

    def check_alive(self) -> None:
        if self._backward is None:
            raise self._freed_error()

    def _freed_error(self) -> RuntimeError:
        return RuntimeError(
            f"Trying to backward through the graph a second time (op '{self.op}'); "
            "the saved intermediate values were freed. Pass retain_graph=True to the "
            "first backward() call if you need to backpropagate through it again."
        )

    def apply(self, grad: DeviceArray, need: tuple[bool, ...]) -> tuple[DeviceArray | None, ...]:
        self.check_alive()
        assert self._backward is not None
        return self._backward(grad, need)

    def apply_graph(self, grad: Tensor, output: Tensor,
                    need: tuple[bool, ...]) -> tuple[Tensor | None, ...]:
        """The VJP in differentiable ops (``create_graph``): the gradients carry a graph."""
        self.check_alive()
        if self._graph is None:
            raise NotImplementedError(
                f"create_graph=True: op '{self.op}' has no differentiable VJP on the device")
        return self._graph(grad, output, need)

    def release(self) -> None:
        """Drop the closures (and the device buffers they saved) and the parent references."""
        self._backward = None
        self._graph = None
        self.parents = ()

    def __repr__(self) -> str:
        return f"<Node {self.op}>"


# ---------------------------------------------------------------------------- engine
def _topological_order(roots: Sequence[Tensor]) -> list[Tensor]:
    """Every tensor the roots depend on (requiring grad), inputs before outputs."""
    order: list[Tensor] = []
    seen: set[int] = set()
    stack: list[tuple[Tensor, bool]] = [(r, False) for r in roots]
    while stack:
        t, done = stack.pop()
        if done:
            order.append(t)
            continue
        if id(t) in seen:
            continue
        seen.add(id(t))
        stack.append((t, True))
        node = t._node
        if node is not None:
            for p in node.parents:
                if p._requires_grad and id(p) not in seen:
                    stack.append((p, False))
    return _leaves_before_first_use(order)


def _leaves_before_first_use(order: list[Tensor]) -> list[Tensor]:
    """The same order with every leaf moved to just before its first consumer.

    The backward walk visits ``order`` reversed, so a leaf is then finalised right after the
    last op that contributes to its gradient, not wherever the depth-first search happened
    to reach it (the last parameters a backward pass sees, e.g. the earliest blocks' weights,
    are otherwise reached first and processed last). The ops' order, and therefore every
    sum, is unchanged; only the moment a leaf's ``.grad`` is written (and the leaf hooks of
    data-parallel bucketing fire) moves earlier.
    """
    placed: set[int] = set()
    out: list[Tensor] = []
    for t in order:
        node = t._node
        if node is None:
            continue
        for p in node.parents:
            if p._node is None and p._requires_grad and id(p) not in placed:
                placed.add(id(p))
                out.append(p)
        out.append(t)
    # Leaves nobody consumes (e.g. a root that is a leaf) keep their place at the end.
    for t in order:
        if t._node is None and id(t) not in placed:
            out.append(t)
    return out


def _leads_to(order: list[Tensor], targets: set[int]) -> set[int]:
    """Ids of tensors in ``order`` that are targets or have a target among their inputs."""
    live: set[int] = set()
    for t in order:
        node = t._node
        if id(t) in targets or (node is not None and any(id(p) in live for p in node.parents)):
            live.add(id(t))
    return live


#: Called as ``hook(leaf)`` right after a leaf's gradient for this backward pass is final.
_leaf_hooks: list[Callable[[Tensor], None]] = []


def add_leaf_hook(hook: Callable[[Tensor], None]) -> Callable[[], None]:
    """Register ``hook(leaf)`` (used by data-parallel gradient bucketing); returns a remover."""
    _leaf_hooks.append(hook)
    return lambda: _leaf_hooks.remove(hook)


def _run_backward(
    roots: Sequence[Tensor],
    seeds: Sequence[DeviceArray],
    *,
    retain_graph: bool,
    targets: Sequence[Tensor] | None,
    create_graph: bool = False,
) -> dict[int, Any]:
    if create_graph:
        return _graph_pass(roots, seeds, retain_graph, targets)
    prof = _profiler.active()
    if prof is None:
        return _backward_pass(roots, seeds, retain_graph, targets, None)
    return prof.timed(_profiler.ENGINE, True, _backward_pass, roots, seeds, retain_graph, targets,
                      prof)


def _backward_pass(
    roots: Sequence[Tensor],
    seeds: Sequence[DeviceArray],
    retain_graph: bool,
    targets: Sequence[Tensor] | None,
    prof: Any,
) -> dict[int, DeviceArray]:
    order = _topological_order(roots)
    target_ids = None if targets is None else {id(t) for t in targets}
    live = None if target_ids is None else _leads_to(order, target_ids)
    pending: dict[int, DeviceArray] = {}
    for root, seed in zip(roots, seeds, strict=True):
        prev = pending.get(id(root))
        pending[id(root)] = seed if prev is None else prev + seed
    captured: dict[int, DeviceArray] = {}
    hooks = _leaf_hooks
    for t in reversed(order):
        g = pending.pop(id(t), None)
        if g is None:
            continue
        node = t._node
        if target_ids is not None:
            if id(t) in target_ids:
                captured[id(t)] = g
        elif node is None or t._retains_grad:
            t._accumulate_grad(g)
            if node is None and hooks:
                for h in hooks:
                    h(t)
        if node is None:
            continue
        fn = node._backward
        if fn is None:
            raise node._freed_error()
        parents = node.parents
        if live is None:
            need = tuple([p._requires_grad for p in parents])
        else:
            need = tuple([p._requires_grad and id(p) in live for p in parents])
        if not any(need):
            continue
        if prof is None:
            grads = fn(g, need)
        else:
            grads = prof.timed(node.op, True, fn, g, need)
        if len(grads) != len(parents):
            raise RuntimeError(
                f"op '{node.op}' returned {len(grads)} gradients for {len(parents)} inputs"
            )
        for p, pg, wanted in zip(parents, grads, need, strict=True):
            if pg is None or not wanted:
                continue
            if pg.shape != p.shape:
                raise RuntimeError(
                    f"op '{node.op}' produced a gradient of shape {pg.shape} "
                    f"for an input of shape {p.shape}"
                )
            prev = pending.get(id(p))
            pending[id(p)] = pg if prev is None else prev + pg
        if not retain_graph:
            node.release()
    return captured


def _graph_pass(
    roots: Sequence[Tensor],
    seeds: Sequence[Any],
    retain_graph: bool,
    targets: Sequence[Tensor] | None,
) -> dict[int, Tensor]:
    """The walk of ``_backward_pass`` with tensor gradients built from differentiable ops
    (grad mode on), so every gradient it produces has a graph of its own. A leaf's gradient is
    then a plain tensor (not a slot of a flat arena): ``leaf.grad = leaf.grad + g``."""
    from tensorgrad_b200.tensor import Tensor

    order = _topological_order(roots)
    target_ids = None if targets is None else {id(t) for t in targets}
    live = None if target_ids is None else _leads_to(order, target_ids)
    captured: dict[int, Tensor] = {}
    with enable_grad():
        pending: dict[int, Tensor] = {}
        for root, seed in zip(roots, seeds, strict=True):
            # A tensor seed keeps its own graph (e.g. the dummy cotangent of a forward-mode
            # product, which is differentiated against afterwards).
            g0 = seed if isinstance(seed, Tensor) else Tensor._wrap(seed)
            prev = pending.get(id(root))
            pending[id(root)] = g0 if prev is None else prev + g0
        for t in reversed(order):
            g = pending.pop(id(t), None)
            if g is None:
                continue
            node = t._node
            if target_ids is not None:
                if id(t) in target_ids:
                    captured[id(t)] = g
            elif node is None or t._retains_grad:
                t.grad = g if t._grad is None else t._grad + g
            if node is None:
                continue
            if node._backward is None:
                raise node._freed_error()
            parents = node.parents
            need = tuple([p._requires_grad and (live is None or id(p) in live)
                          for p in parents])
            if not any(need):
                continue
            if node._graph is None:
                raise NotImplementedError(
                    f"create_graph=True: op '{node.op}' has no differentiable VJP on the device")
            grads = node._graph(g, t, need)
            if len(grads) != len(parents):
                raise RuntimeError(
                    f"op '{node.op}' returned {len(grads)} gradients for {len(parents)} inputs"
                )
            for p, pg, wanted in zip(parents, grads, need, strict=True):
                if pg is None or not wanted:
                    continue
                if pg.shape != p.shape:
                    raise RuntimeError(
                        f"op '{node.op}' produced a gradient of shape {pg.shape} "
                        f"for an input of shape {p.shape}"
                    )
                prev = pending.get(id(p))
                pending[id(p)] = pg if prev is None else prev + pg
            if not retain_graph:
                node.release()
    return captured


# ---------------------------------------------------------------------------- public API
def _as_tensors(value: Any, what: str) -> tuple[Tensor, ...]:
    from tensorgrad_b200.tensor import Tensor

    items = (value,) if isinstance(value, Tensor) else tuple(value)
    if not items:
        raise ValueError(f"{what} must contain at least one tensor")
    for item in items:
        if not isinstance(item, Tensor):
            raise TypeError(f"{what} must be tensors, got {type(item).__name__}")
    return items


def _graph_seeds(seeds: list[DeviceArray], grad_outputs: GradOutputs) -> list[Any]:
    """For ``create_graph``: the checked seeds, with every seed given as a tensor that
    requires grad passed as that tensor (its graph kept)."""
    from tensorgrad_b200.tensor import Tensor

    if grad_outputs is None or isinstance(grad_outputs, Tensor | np.ndarray):
        given: list[Any] = [grad_outputs]
    else:
        given = list(grad_outputs)
    return [g if isinstance(g, Tensor) and g.requires_grad and g.dtype == s.dtype else s
            for g, s in zip(given, seeds, strict=False)] + seeds[len(given):]


def _seeds(outputs: tuple[Tensor, ...], grad_outputs: GradOutputs) -> list[DeviceArray]:
    from tensorgrad_b200 import device
    from tensorgrad_b200.tensor import Tensor

    if grad_outputs is None:
        given: list[Any] = [None] * len(outputs)
    elif isinstance(grad_outputs, Tensor | np.ndarray | device.DeviceArray):
        given = [grad_outputs]
    else:
        given = list(grad_outputs)
    if len(given) != len(outputs):
        raise ValueError(f"got {len(given)} grad_outputs for {len(outputs)} outputs")
    seeds: list[DeviceArray] = []
    for out, g in zip(outputs, given, strict=True):
        if g is None:
            if out.size != 1:
                raise RuntimeError(
                    "grad can be implicitly created only for single-element outputs; "
                    f"got shape {out.shape}"
                )
            seeds.append(device.from_numpy(np.ones(out.shape, dtype=out.dtype)))
            continue
        if isinstance(g, Tensor):
            g = g.data
        if isinstance(g, device.DeviceArray):
            seed = g if g.dtype == out.dtype else g.astype(out.dtype)
        else:
            seed = device.from_numpy(np.asarray(g, dtype=out.dtype))
        if seed.shape != out.shape:
            raise ValueError(f"grad has shape {seed.shape}, expected {out.shape}")
        seeds.append(seed)
    return seeds


def backward(
    tensors: Tensor | Sequence[Tensor],
    grad_tensors: GradOutputs = None,
    retain_graph: bool | None = None,
    create_graph: bool = False,
) -> None:
    """Accumulate d(sum of ``tensors``)/d(leaf) into the ``.grad`` of every leaf; with
    ``create_graph`` the accumulated gradients carry a graph (``retain_graph`` then defaults
    to True, as in the reference)."""
    outputs = _as_tensors(tensors, "tensors")
    for out in outputs:
        if not out.requires_grad:
            raise RuntimeError("backward() called on a tensor that does not require grad")
    seeds: list[Any] = _seeds(outputs, grad_tensors)
    if create_graph:
        seeds = _graph_seeds(seeds, grad_tensors)
    keep = create_graph if retain_graph is None else bool(retain_graph)
    _run_backward(outputs, seeds, retain_graph=keep, targets=None, create_graph=create_graph)


def grad(
    outputs: Tensor | Sequence[Tensor],
    inputs: Tensor | Sequence[Tensor],
    grad_outputs: GradOutputs = None,
    retain_graph: bool | None = None,
    create_graph: bool = False,
    allow_unused: bool = False,
) -> tuple[Tensor | None, ...]:
    """Gradients of ``outputs`` with respect to ``inputs``, returned instead of accumulated."""
    from tensorgrad_b200.tensor import Tensor

    outs = _as_tensors(outputs, "outputs")
    ins = _as_tensors(inputs, "inputs")
    for i, out in enumerate(outs):
        if not out.requires_grad:
            raise RuntimeError(f"output {i} does not require grad and has no graph")
    for i, inp in enumerate(ins):
        if not inp.requires_grad:
            raise RuntimeError(f"input {i} does not require grad")
    seeds: list[Any] = _seeds(outs, grad_outputs)
    if create_graph:
        seeds = _graph_seeds(seeds, grad_outputs)
    keep = create_graph if retain_graph is None else bool(retain_graph)
    captured = _run_backward(outs, seeds, retain_graph=keep, targets=ins,
                             create_graph=create_graph)
    result: list[Tensor | None] = []
    for i, inp in enumerate(ins):
        g = captured.get(id(inp))
        if g is None:
            if not allow_unused:
                raise RuntimeError(
                    f"input {i} was not used to compute the outputs; pass allow_unused=True "
                    "to get None for it instead"
                )
            result.append(None)
        elif create_graph:
            result.append(g)  # a tensor with its own graph
        else:
            # A fresh array: the engine may hand back aliases of other gradients.
            result.append(Tensor._wrap(g.astype(inp.dtype, copy=True)))
    return tuple(result)
