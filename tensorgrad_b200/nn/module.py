"""``Module`` and ``Parameter`` (the reference's nn/module.py:16-244), with device storage.

Registration, traversal (tied parameters listed once), ``train``/``eval`` and the state dict
behave as in the reference. ``state_dict()`` returns host NumPy copies; ``load_state_dict``
uploads into the existing device buffers in place.
"""

from __future__ import annotations

from collections.abc import Callable, Iterator, Mapping
from typing import Any, NamedTuple, Self

import numpy as np

from tensorgrad_b200.device import DeviceArray
from tensorgrad_b200.tensor import Tensor

__all__ = ["IncompatibleKeys", "Module", "Parameter"]


class Parameter(Tensor):
    """A tensor that a :class:`Module` registers as trainable (``requires_grad`` by default)."""

    __slots__ = ()

    def __init__(self, data: object, requires_grad: bool = True) -> None:
        super().__init__(data, requires_grad=requires_grad)


class IncompatibleKeys(NamedTuple):
    missing_keys: list[str]
    unexpected_keys: list[str]


class Module:
    """Base class for layers and models (same contract as the reference's ``Module``)."""

    training: bool

    def __init__(self) -> None:
        object.__setattr__(self, "_parameters", {})
        object.__setattr__(self, "_modules", {})
        object.__setattr__(self, "_buffers", {})
        object.__setattr__(self, "training", True)

    def __setattr__(self, name: str, value: object) -> None:
        state = self.__dict__
        if "_parameters" not in state:
            if isinstance(value, Parameter | Module):
                raise AttributeError("call Module.__init__() before assigning parameters/modules")
            object.__setattr__(self, name, value)
            return
        params, modules, buffers = state["_parameters"], state["_modules"], state["_buffers"]
        if name in buffers:
            if not isinstance(value, DeviceArray | np.ndarray):
                raise TypeError(f"buffer '{name}' must be an array")
            if isinstance(value, np.ndarray):
                from tensorgrad_b200 import device

                value = device.from_numpy(value)
            buffers[name] = value
        else:
            params.pop(name, None)
            modules.pop(name, None)
            if isinstance(value, Parameter):
                params[name] = value
            elif isinstance(value, Module):
                modules[name] = value
        object.__setattr__(self, name, value)

    def __delattr__(self, name: str) -> None:
        for registry in ("_parameters", "_modules", "_buffers"):
            self.__dict__[registry].pop(name, None)
        object.__delattr__(self, name)

    def register_buffer(self, name: str, value: Any) -> None:
        """Register a non-trainable array (e.g. running statistics) saved in the state dict."""
        if isinstance(value, np.ndarray):
            from tensorgrad_b200 import device

            value = device.from_numpy(value)
        self.__dict__["_buffers"][name] = value
        object.__setattr__(self, name, value)

    # ------------------------------------------------------------------ traversal
    def named_children(self) -> Iterator[tuple[str, Module]]:
        yield from self.__dict__["_modules"].items()

    def children(self) -> Iterator[Module]:
        for _, m in self.named_children():
            yield m

    def named_modules(self, prefix: str = "") -> Iterator[tuple[str, Module]]:
        seen: set[int] = set()

        def walk(module: Module, name: str) -> Iterator[tuple[str, Module]]:
            if id(module) in seen:
                return
            seen.add(id(module))
            yield name, module
            for child_name, child in module.named_children():
                yield from walk(child, f"{name}.{child_name}" if name else child_name)

        yield from walk(self, prefix)

    def modules(self) -> Iterator[Module]:
        for _, m in self.named_modules():
            yield m

    def _named_members(self, registry: str, prefix: str, recurse: bool,
                       dedupe: bool) -> Iterator[tuple[str, Any]]:
        seen: set[int] = set()

        def walk(module: Module, name: str) -> Iterator[tuple[str, Any]]:
            for key, value in module.__dict__[registry].items():
                if dedupe and id(value) in seen:
                    continue
                seen.add(id(value))
                yield (f"{name}.{key}" if name else key), value
            if recurse:
                for child_name, child in module.named_children():
                    yield from walk(child, f"{name}.{child_name}" if name else child_name)

        yield from walk(self, prefix)

    def named_parameters(self, prefix: str = "", recurse: bool = True) -> Iterator[tuple[str, Parameter]]:
        """Parameters with dotted names; a parameter shared by several modules appears once."""
        yield from self._named_members("_parameters", prefix, recurse, dedupe=True)

    def parameters(self, recurse: bool = True) -> Iterator[Parameter]:
        for _, p in self.named_parameters(recurse=recurse):
            yield p

    def named_buffers(self, prefix: str = "", recurse: bool = True) -> Iterator[tuple[str, Any]]:
        yield from self._named_members("_buffers", prefix, recurse, dedupe=True)

    def num_parameters(self) -> int:
        return sum(p.size for p in self.parameters())

    # ------------------------------------------------------------------ state
    def state_dict(self) -> dict[str, np.ndarray]:
        """Host copies of every parameter and buffer (tied parameters under both names)."""
        state: dict[str, np.ndarray] = {}
        for name, p in self._named_members("_parameters", "", True, dedupe=False):
            state[name] = p.data.numpy()
        for name, b in self._named_members("_buffers", "", True, dedupe=False):
            state[name] = b.numpy() if isinstance(b, DeviceArray) else np.array(b, copy=True)
        return state

    def load_state_dict(self, state: Mapping[str, Any], strict: bool = True) -> IncompatibleKeys:
        """Copy arrays from ``state`` into the parameters and buffers, in place."""
        targets: dict[str, DeviceArray] = {}
        for name, p in self._named_members("_parameters", "", True, dedupe=False):
            targets[name] = p.data
        for name, b in self._named_members("_buffers", "", True, dedupe=False):
            targets[name] = b
        missing = [k for k in targets if k not in state]
        unexpected = [k for k in state if k not in targets]
        if strict and (missing or unexpected):
            raise KeyError(f"state dict mismatch: missing={missing}, unexpected={unexpected}")
        for name, target in targets.items():
            if name not in state:
                continue
            value = np.asarray(state[name])
            if value.shape != target.shape:
                raise ValueError(
                    f"shape mismatch for '{name}': expected {target.shape}, got {value.shape}"
                )
            target[...] = value
        return IncompatibleKeys(missing, unexpected)

    # ------------------------------------------------------------------ modes / helpers
    def train(self, mode: bool = True) -> Self:
        for m in self.modules():
            object.__setattr__(m, "training", mode)
        return self

    def eval(self) -> Self:
        return self.train(False)

    def zero_grad(self) -> None:
        for p in self.parameters():
            p.grad = None

    def apply(self, fn: Callable[[Module], None]) -> Self:
        for m in reversed(list(self.modules())):
            fn(m)
        return self

    def forward(self, *args: Any, **kwargs: Any) -> Tensor:
        raise NotImplementedError(f"{type(self).__name__} does not implement forward()")

    def __call__(self, *args: Any, **kwargs: Any) -> Tensor:
        return self.forward(*args, **kwargs)

    def extra_repr(self) -> str:
        return ""

    def __repr__(self) -> str:
        children = list(self.named_children())
        head = f"{type(self).__name__}({self.extra_repr()}"
        if not children:
            return head + ")"
        lines = [head]
        for name, child in children:
            body = repr(child).replace("\n", "\n  ")
            lines.append(f"  ({name}): {body}")
        return "\n".join(lines) + "\n)"
