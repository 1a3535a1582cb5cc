"""``Module`` and ``Parameter`` for device-resident models (API of the reference's
nn/module.py:16-244).

Every module keeps one ordered registry, attribute name -> member kind (parameter, child
module or buffer); the values themselves are ordinary attributes. Walking the tree with a
kind filter gives the reference's traversal orders: per kind, members in assignment order,
a re-assigned member moved to the end, children depth-first, shared tensors once where the
reference dedupes them. Buffers are device arrays (host arrays are uploaded when assigned).

State dicts move between host and device in bulk: ``state_dict`` queues one device-to-host
copy per tensor into page-locked staging and synchronises once, instead of once per tensor.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator, Mapping
from typing import Any, NamedTuple, Self

import numpy as np

from tensorgrad_b200 import device
from tensorgrad_b200.device import DeviceArray
from tensorgrad_b200.tensor import Tensor

__all__ = ["IncompatibleKeys", "Module", "Parameter"]

_PARAM, _CHILD, _BUFFER = "parameter", "module", "buffer"


class Parameter(Tensor):
    """A tensor that a :class:`Module` registers as trainable (``requires_grad`` by default)."""

    __slots__ = ()

    def __init__(self, data: object, requires_grad: bool = True) -> None:
        super().__init__(data, requires_grad=requires_grad)


class IncompatibleKeys(NamedTuple):
    """Keys a non-strict :meth:`Module.load_state_dict` could not match."""

    missing_keys: list[str]
    unexpected_keys: list[str]


def _as_device_buffer(name: str, value: object) -> DeviceArray:
    if isinstance(value, DeviceArray):
        return value
    if isinstance(value, np.ndarray):
        return device.from_numpy(value)
    raise TypeError(f"buffer '{name}' must be an array")


class Module:
    """Base class for layers and models: assigning a :class:`Parameter`, a sub-module or a
    registered buffer to an attribute registers it for traversal, state dicts and modes."""

    training: bool

    def __init__(self) -> None:
        object.__setattr__(self, "_registry", {})
        object.__setattr__(self, "training", True)

    # ------------------------------------------------------------------ registration
    def __setattr__(self, name: str, value: object) -> None:
        registry: dict[str, str] | None = self.__dict__.get("_registry")
        if registry is None:
            if isinstance(value, Parameter | Module):
                raise AttributeError("call Module.__init__() before assigning parameters/modules")
            object.__setattr__(self, name, value)
            return
        if registry.get(name) == _BUFFER:
            value = _as_device_buffer(name, value)
        else:
            kind = _PARAM if isinstance(value, Parameter) else (
                _CHILD if isinstance(value, Module) else None)
            registry.pop(name, None)  # re-registration moves the member to the end
            if kind is not None:
                registry[name] = kind
        object.__setattr__(self, name, value)

    def __delattr__(self, name: str) -> None:
        self.__dict__["_registry"].pop(name, None)
        object.__delattr__(self, name)

    def register_buffer(self, name: str, value: Any) -> None:
        """Register a non-trainable array (e.g. running statistics) saved in the state dict."""
        self.__dict__["_registry"][name] = _BUFFER
        object.__setattr__(self, name, _as_device_buffer(name, value))

    def _own(self, kind: str) -> Iterator[tuple[str, Any]]:
        for name, k in self.__dict__["_registry"].items():
            if k == kind:
                yield name, self.__dict__[name]

    # ------------------------------------------------------------------ traversal
    def named_children(self) -> Iterator[tuple[str, Module]]:
        """Direct sub-modules with their attribute names."""
        yield from self._own(_CHILD)

    def children(self) -> Iterator[Module]:
        for _, child in self._own(_CHILD):
            yield child

    def named_modules(self, prefix: str = "") -> Iterator[tuple[str, Module]]:
        """This module and every descendant once (depth first), with dotted names."""
        visited: set[int] = set()
        stack: list[tuple[str, Module]] = [(prefix, self)]
        while stack:
            path, module = stack.pop()
            if id(module) in visited:
                continue
            visited.add(id(module))
            yield path, module
            kids = [(f"{path}.{n}" if path else n, c) for n, c in module._own(_CHILD)]
            stack.extend(reversed(kids))

    def modules(self) -> Iterator[Module]:
        for _, module in self.named_modules():
            yield module

    def _members(self, kind: str, prefix: str, recurse: bool, once: bool) -> Iterator[tuple[str, Any]]:
        """Members of ``kind`` with dotted names: this module's own first, then each child's
        subtree in order (a child reached twice is walked twice); ``once`` skips a value
        already yielded (a tied parameter)."""
        yielded: set[int] = set()

        def visit(module: Module, path: str) -> Iterator[tuple[str, Any]]:
            for name, value in module._own(kind):
                if once and id(value) in yielded:
                    continue
                yielded.add(id(value))
                yield (f"{path}.{name}" if path else name), value
            if recurse:
                for name, child in module._own(_CHILD):
                    yield from visit(child, f"{path}.{name}" if path else name)

        yield from visit(self, prefix)

    def named_parameters(self, prefix: str = "", recurse: bool = True) -> Iterator[tuple[str, Parameter]]:
        """Parameters with dotted names; a parameter shared by several modules appears once."""
        yield from self._members(_PARAM, prefix, recurse, once=True)

    def parameters(self, recurse: bool = True) -> Iterator[Parameter]:
        for _, p in self._members(_PARAM, "", recurse, once=True):
            yield p

    def named_buffers(self, prefix: str = "", recurse: bool = True) -> Iterator[tuple[str, Any]]:
        yield from self._members(_BUFFER, prefix, recurse, once=True)

    def num_parameters(self) -> int:
        """Scalar parameters in the model, shared ones counted once."""
        return sum(p.size for p in self.parameters())

    # ------------------------------------------------------------------ state
    def _state_targets(self) -> dict[str, DeviceArray]:
        """Every parameter and buffer under every name it has (a tied parameter twice)."""
        out = {name: p.data for name, p in self._members(_PARAM, "", True, once=False)}
        out.update(self._members(_BUFFER, "", True, once=False))
        return out

    def state_dict(self) -> dict[str, np.ndarray]:
        """Host copies of every parameter and buffer, keyed by dotted name (a parameter shared
        by two modules appears under both names)."""
        targets = self._state_targets()
        return dict(zip(targets, device.numpy_many(list(targets.values())), strict=True))

    def load_state_dict(self, state: Mapping[str, Any], strict: bool = True) -> IncompatibleKeys:
        """Copy arrays from ``state`` into the parameters and buffers, in place (uploads)."""
        targets = self._state_targets()
        missing = [name for name in targets if name not in state]
        unexpected = [name for name in state if name not in targets]
        if strict and (missing or unexpected):
            raise KeyError(f"state dict mismatch: missing={missing}, unexpected={unexpected}")
        for name, target in targets.items():
            if name in state:
                value = np.asarray(state[name])
                if value.shape != target.shape:
                    raise ValueError(f"shape mismatch for '{name}': expected {target.shape}, "
                                     f"got {value.shape}")
                target[...] = value
        return IncompatibleKeys(missing, unexpected)

    # ------------------------------------------------------------------ modes / helpers
    def train(self, mode: bool = True) -> Self:
        for module in self.modules():
            object.__setattr__(module, "training", mode)
        return self

    def eval(self) -> Self:
        return self.train(False)

    def zero_grad(self) -> None:
        for p in self.parameters():
            p.grad = None

    def apply(self, fn: Callable[[Module], None]) -> Self:
        """Call ``fn`` on every descendant, children before parents, ``self`` last."""
        for module in list(self.modules())[::-1]:
            fn(module)
        return self

    def forward(self, *args: Any, **kwargs: Any) -> Tensor:
        raise NotImplementedError(f"{type(self).__name__} does not implement forward()")

    def __call__(self, *args: Any, **kwargs: Any) -> Tensor:
        return self.forward(*args, **kwargs)

    def extra_repr(self) -> str:
        return ""

    def __repr__(self) -> str:
        inner = [f"  ({name}): " + repr(child).replace("\n", "\n  ")
                 for name, child in self._own(_CHILD)]
        head = f"{type(self).__name__}({self.extra_repr()}"
        return head + ")" if not inner else "\n".join([head, *inner]) + "\n)"
