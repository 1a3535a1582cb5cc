"""Optimizer base and parameter groups (API and checks of the reference's
optim/optimizer.py:15-116), for device optimizers.

The constructor accepts a list of tensors or a list of group dicts (``params`` plus optional
``lr`` / ``weight_decay``) and validates them with the reference's exception types and
messages. Subclasses implement ``step`` as device kernels over the groups; the per-parameter
state is keyed by the parameter's identity.
"""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass, field
from typing import Any, Generic, NotRequired, TypedDict, TypeVar

from tensorgrad_b200.tensor import Tensor

__all__ = ["Optimizer", "ParamGroup", "ParamGroupSpec"]


class ParamGroupSpec(TypedDict):
    params: Iterable[Tensor]
    lr: NotRequired[float]
    weight_decay: NotRequired[float]


@dataclass(eq=False)
class ParamGroup:
    """Parameters that share a learning rate and weight decay; ``initial_lr`` is the learning
    rate the group started with (what schedules scale)."""

    params: list[Tensor]
    lr: float
    weight_decay: float
    initial_lr: float = field(init=False)

    def __post_init__(self) -> None:
        self.initial_lr = self.lr


StateT = TypeVar("StateT")


def _group_specs(items: list[Any]) -> list[dict[str, Any]]:
    """The constructor's argument as group dicts: one group for a plain list of tensors."""
    dicts = [isinstance(item, dict) for item in items]
    if all(dicts):
        return [dict(item) for item in items]
    if any(dicts):
        raise TypeError("mix of tensors and parameter-group dicts")
    return [{"params": items}]


class Optimizer(Generic[StateT]):
    """Parameter groups and per-parameter state; ``step`` is the subclass's update."""

    def __init__(self, params: Iterable[Any], lr: float, weight_decay: float) -> None:
        if lr < 0:
            raise ValueError(f"invalid learning rate {lr}")
        if weight_decay < 0:
            raise ValueError(f"invalid weight decay {weight_decay}")
        items = list(params)
        if not items:
            raise ValueError("optimizer got an empty parameter list")
        claimed: set[int] = set()
        self.param_groups: list[ParamGroup] = []
        for spec in _group_specs(items):
            members = list(spec["params"])
            for p in members:
                if not isinstance(p, Tensor) or not p.requires_grad:
                    raise TypeError("optimizers can only update tensors with requires_grad=True")
                if id(p) in claimed:  # listed twice, in one group or in two
                    raise ValueError("a parameter appears in more than one parameter group")
                claimed.add(id(p))
            self.param_groups.append(ParamGroup(members, spec.get("lr", lr),
                                                spec.get("weight_decay", weight_decay)))
        self.state: dict[int, StateT] = {}

    def zero_grad(self) -> None:
        """Drop every managed parameter's gradient (``grad = None``)."""
        everything = [p for g in self.param_groups for p in g.params]
        ids = {id(p) for p in everything}
        for p in everything:
            arena = p._arena
            # A clip rescale still pending on gradients that all go away needs no writing.
            if (arena is not None and arena.pending_clip is not None
                    and all(id(q) in ids for q in arena.params)):
                arena.pending_clip = None
            p.grad = None

    def step(self) -> None:
        """Apply one update to every parameter that has a gradient."""
        raise NotImplementedError
