"""Learning-rate schedules, kept minimal (API of the reference's optim/lr_scheduler.py).

A schedule is a multiplier of each group's initial learning rate as a function of the
schedule's step count; stepping it writes ``initial_lr * multiplier`` into every group, which
the next optimizer kernel launch reads as a scalar argument. Nothing here touches the device.
"""

from __future__ import annotations

import math
from typing import Any

from tensorgrad_b200.optim.optimizer import Optimizer

__all__ = ["CosineWarmupLR", "LRScheduler", "StepLR"]


class LRScheduler:
    """Base schedule: subclasses define ``factor(step)``."""

    def __init__(self, optimizer: Optimizer[Any]) -> None:
        self.optimizer = optimizer
        self.last_step = 0
        self._write()

    def factor(self, step: int) -> float:
        raise NotImplementedError

    def step(self) -> None:
        self.last_step += 1
        self._write()

    def get_last_lr(self) -> list[float]:
        return [g.lr for g in self.optimizer.param_groups]

    def _write(self) -> None:
        mult = self.factor(self.last_step)
        for g in self.optimizer.param_groups:
            g.lr = g.initial_lr * mult


class StepLR(LRScheduler):
    """``gamma ** (step // step_size)``."""

    def __init__(self, optimizer: Optimizer[Any], step_size: int, gamma: float = 0.1) -> None:
        if step_size <= 0:
            raise ValueError("step_size must be positive")
        self.step_size, self.gamma = step_size, gamma
        super().__init__(optimizer)

    def factor(self, step: int) -> float:
        return float(self.gamma ** (step // self.step_size))


class CosineWarmupLR(LRScheduler):
    """Linear warm-up over ``warmup_steps`` (``(step + 1) / warmup``), then a half cosine from
    1 down to ``min_lr_ratio`` at ``total_steps`` (held there afterwards)."""

    def __init__(self, optimizer: Optimizer[Any], warmup_steps: int, total_steps: int,
                 min_lr_ratio: float = 0.0) -> None:
        if warmup_steps < 0 or total_steps <= 0 or warmup_steps > total_steps:
            raise ValueError("need 0 <= warmup_steps <= total_steps and total_steps > 0")
        if not 0.0 <= min_lr_ratio <= 1.0:
            raise ValueError("min_lr_ratio must be in [0, 1]")
        self.warmup_steps, self.total_steps, self.min_lr_ratio = (warmup_steps, total_steps,
                                                                  min_lr_ratio)
        super().__init__(optimizer)

    def factor(self, step: int) -> float:
        if step < self.warmup_steps:
            return (step + 1) / self.warmup_steps
        done = min((step - self.warmup_steps) / max(self.total_steps - self.warmup_steps, 1), 1.0)
        cosine = 0.5 * (1.0 + math.cos(math.pi * done))
        return self.min_lr_ratio + (1.0 - self.min_lr_ratio) * cosine
