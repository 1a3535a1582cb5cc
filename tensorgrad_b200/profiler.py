"""Per-op timing (the reference's ``tensorgrad.profiler`` API, profiler.py:25-152).

    with tensorgrad_b200.profiler.profile() as prof:
        loss = tg.cross_entropy(model(x), y)
        loss.backward()
    print(prof.table())

Inside the block every public op and every VJP the backward pass runs is timed, and the
device is synchronised around each timed call, so a row's time is the device work it
launched plus its host overhead. Time of ops called by an op (a composite op, a graph VJP) is
charged to those ops: every row is self time and the rows add up. The "autograd engine" row
is the backward pass's own time outside VJPs. Timing synchronises the stream, so never
profile a run whose throughput you report.
"""

from __future__ import annotations

import contextlib
import functools
import time
from collections.abc import Callable, Iterator
from dataclasses import dataclass
from typing import Any, TypeVar

__all__ = ["ENGINE", "OpStats", "Profile", "profile", "profiled"]

#: Name of the row that holds the backward engine's own time.
ENGINE = "autograd engine"
_R = TypeVar("_R")


@dataclass
class OpStats:
    """Call counts and self time (seconds) of one op."""

    forward_calls: int = 0
    forward_seconds: float = 0.0
    backward_calls: int = 0
    backward_seconds: float = 0.0

    @property
    def total_seconds(self) -> float:
        """Forward plus backward self time."""
        return self.forward_seconds + self.backward_seconds


class Profile:
    """Per-op timings collected by :func:`profile`, keyed by op name."""

    def __init__(self) -> None:
        self.ops: dict[str, OpStats] = {}
        #: Wall-clock duration of the ``with`` block.
        self.wall_seconds = 0.0
        self._nested: list[float] = []  # time of timed calls inside each call in progress

    def timed(self, name: str, backward: bool, fn: Callable[..., _R], *args: Any,
              **kwargs: Any) -> _R:
        """Run ``fn(*args, **kwargs)`` between two device synchronisations and charge its
        self time to ``name``."""
        from tensorgrad_b200.device import synchronize

        synchronize()
        self._nested.append(0.0)
        start = time.perf_counter()
        try:
            return fn(*args, **kwargs)
        finally:
            synchronize()
            elapsed = time.perf_counter() - start
            own = elapsed - self._nested.pop()
            if self._nested:
                self._nested[-1] += elapsed
            stats = self.ops.setdefault(name, OpStats())
            if backward:
                stats.backward_calls += 1
                stats.backward_seconds += own
            else:
                stats.forward_calls += 1
                stats.forward_seconds += own

    @property
    def profiled_seconds(self) -> float:
        """Time inside ops and the engine (the sum of all rows)."""
        return sum(s.total_seconds for s in self.ops.values())

    def table(self, limit: int | None = None) -> str:
        """Rows by total self time, as an aligned text table (milliseconds)."""
        rows = sorted(self.ops.items(), key=lambda kv: kv[1].total_seconds, reverse=True)
        total = self.profiled_seconds or 1.0
        width = max([2, *(len(name) for name in self.ops)])
        head = (f"{'op':<{width}}  {'fwd calls':>9}  {'fwd ms':>9}  {'bwd calls':>9}  "
                f"{'bwd ms':>9}  {'total ms':>9}  {'share':>6}")
        lines = [head, "-" * len(head)]
        for name, s in rows[:limit]:
            lines.append(f"{name:<{width}}  {s.forward_calls:>9}  {1e3 * s.forward_seconds:>9.2f}  "
                         f"{s.backward_calls:>9}  {1e3 * s.backward_seconds:>9.2f}  "
                         f"{1e3 * s.total_seconds:>9.2f}  {s.total_seconds / total:>6.1%}")
        rest = self.wall_seconds - self.profiled_seconds
        lines.append(f"ops and engine: {1e3 * self.profiled_seconds:.2f} ms of "
                     f"{1e3 * self.wall_seconds:.2f} ms wall time ({1e3 * rest:.2f} ms elsewhere: "
                     "Python code between ops, optimiser, data)")
        return "\n".join(lines)


class _Active:
    profile: Profile | None = None


def active() -> Profile | None:
    """The profile being collected, if a :func:`profile` block is open."""
    return _Active.profile


@contextlib.contextmanager
def profile() -> Iterator[Profile]:
    """Collect per-op timings for the code inside the ``with`` block (blocks do not nest)."""
    if _Active.profile is not None:
        raise RuntimeError("profile() blocks cannot be nested")
    result = Profile()
    _Active.profile = result
    start = time.perf_counter()
    try:
        yield result
    finally:
        result.wall_seconds = time.perf_counter() - start
        _Active.profile = None


def profiled(name: str) -> Callable[[Callable[..., _R]], Callable[..., _R]]:
    """Decorator for op functions: time each call under ``name`` while profiling."""

    def decorate(fn: Callable[..., _R]) -> Callable[..., _R]:
        @functools.wraps(fn)
        def wrapper(*args: Any, **kwargs: Any) -> _R:
            prof = _Active.profile
            if prof is None:
                return fn(*args, **kwargs)
            return prof.timed(name, False, fn, *args, **kwargs)

        return wrapper

    return decorate
