"""Optimizer base class and parameter groups (the reference's optim/optimizer.py:15-116)."""

from __future__ import annotations

from abc import ABC, abstractmethod
from collections.abc import Iterable
from dataclasses import dataclass, field
from typing import Any, Generic, NotRequired, TypedDict, TypeVar, cast

from tensorgrad_b200.tensor import Tensor

__all__ = ["Optimizer", "ParamGroup", "ParamGroupSpec"]


class ParamGroupSpec(TypedDict):
    params: Iterable[Tensor]
    lr: NotRequired[float]
    weight_decay: NotRequired[float]


@dataclass(eq=False)
class ParamGroup:
    """Parameters sharing a learning rate and weight decay; schedulers scale ``initial_lr``."""

    params: list[Tensor]
    lr: float
    weight_decay: float
    initial_lr: float = field(init=False)

    def __post_init__(self) -> None:
        self.initial_lr = self.lr


StateT = TypeVar("StateT")


class Optimizer(ABC, Generic[StateT]):
    """Owns parameter groups and per-parameter state; same validation and messages as the
    reference. Subclasses implement :meth:`step` with device kernels."""

    def __init__(self, params: Iterable[Any], lr: float, weight_decay: float) -> None:
        if lr < 0:
            raise ValueError(f"invalid learning rate {lr}")
        if weight_decay < 0:
            raise ValueError(f"invalid weight decay {weight_decay}")
        items = list(params)
        if not items:
            raise ValueError("optimizer got an empty parameter list")
        if all(isinstance(item, dict) for item in items):
            specs = cast(list[ParamGroupSpec], items)
        elif any(isinstance(item, dict) for item in items):
            raise TypeError("mix of tensors and parameter-group dicts")
        else:
            specs = [{"params": cast(list[Tensor], items)}]
        self.param_groups: list[ParamGroup] = []
        seen: set[int] = set()
        for spec in specs:
            group_params = list(spec["params"])
            for p in group_params:
                if not isinstance(p, Tensor) or not p.requires_grad:
                    raise TypeError("optimizers can only update tensors with requires_grad=True")
                if id(p) in seen:
                    raise ValueError("a parameter appears in more than one parameter group")
                seen.add(id(p))
            self.param_groups.append(ParamGroup(group_params, lr=spec.get("lr", lr),
                                                weight_decay=spec.get("weight_decay",
                                                                      weight_decay)))
        self.state: dict[int, StateT] = {}

    def zero_grad(self) -> None:
        """Reset the gradient of every managed parameter (``grad = None``)."""
        cleared = {id(p) for group in self.param_groups for p in group.params}
        for group in self.param_groups:
            for p in group.params:
                arena = p._arena
                # A clip rescale still pending on gradients that are all being dropped
                # needs no writing.
                if (arena is not None and arena.pending_clip is not None
                        and all(id(q) in cleared for q in arena.params)):
                    arena.pending_clip = None
                p.grad = None

    @abstractmethod
    def step(self) -> None:
        """Apply one update to every parameter that has a gradient."""
