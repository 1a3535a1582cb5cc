"""Learning-rate schedules (API of the reference's optim/lr_scheduler.py).

A schedule maps its step count to a multiplier of every parameter group's ``initial_lr``.
Building one applies step 0; each ``step()`` advances the count and rewrites the groups'
``lr``, which the next optimizer launch passes to its kernel as a scalar. Host-only.
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod
from typing import Any

from tensorgrad_b200.optim.optimizer import Optimizer

__all__ = ["CosineWarmupLR", "LRScheduler", "StepLR"]


class LRScheduler(ABC):
    """Subclasses give ``factor(step)``, the multiplier of the initial learning rate (an
    abstract method: the base class cannot be built on its own)."""

    def __init__(self, optimizer: Optimizer[Any]) -> None:
        self.optimizer = optimizer
        self.last_step = 0
        self._set_rates()

    @abstractmethod
    def factor(self, step: int) -> float:
        """The multiplier at ``step``."""

    def step(self) -> None:
        """One optimizer update later."""
        self.last_step += 1
        self._set_rates()

    def get_last_lr(self) -> list[float]:
        """The learning rate each group has now."""
        return [group.lr for group in self.optimizer.param_groups]

    def _set_rates(self) -> None:
        scale = self.factor(self.last_step)
        for group in self.optimizer.param_groups:
            group.lr = scale * group.initial_lr


class StepLR(LRScheduler):
    """Decay by ``gamma`` once every ``step_size`` steps."""

    def __init__(self, optimizer: Optimizer[Any], step_size: int, gamma: float = 0.1) -> None:
        if step_size <= 0:
            raise ValueError("step_size must be positive")
        self.step_size = step_size
        self.gamma = gamma
        super().__init__(optimizer)

    def factor(self, step: int) -> float:
        decays = step // self.step_size
        return float(self.gamma ** decays)


class CosineWarmupLR(LRScheduler):
    """Warm up linearly, ``(step + 1) / warmup_steps``, then fall along half a cosine from 1
    to ``min_lr_ratio``, reached at ``total_steps`` and kept from then on."""

    def __init__(self, optimizer: Optimizer[Any], warmup_steps: int, total_steps: int,
                 min_lr_ratio: float = 0.0) -> None:
        if total_steps <= 0 or not 0 <= warmup_steps <= total_steps:
            raise ValueError("need 0 <= warmup_steps <= total_steps and total_steps > 0")
        if not 0.0 <= min_lr_ratio <= 1.0:
            raise ValueError("min_lr_ratio must be in [0, 1]")
        self.warmup_steps = warmup_steps
        self.total_steps = total_steps
        self.min_lr_ratio = min_lr_ratio
        super().__init__(optimizer)

    def factor(self, step: int) -> float:
        w, floor = self.warmup_steps, self.min_lr_ratio
        if step < w:
            return (step + 1) / w
        decay_steps = self.total_steps - w if self.total_steps > w else 1
        t = (step - w) / decay_steps
        if t > 1.0:
            t = 1.0
        return floor + (1.0 - floor) * (0.5 * (1.0 + math.cos(math.pi * t)))
