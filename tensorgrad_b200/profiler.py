"""Per-op timing (the reference's ``tensorgrad.profiler`` API, profiler.py:49-152).

Inside ``with profile() as prof:`` every public op and every VJP is timed; the device is
synchronised around each timed call so a row's time is the device work it launched plus its
host overhead. Self time excludes nested timed calls. ``prof.table()`` prints the summary.
Timing synchronises the stream, so never profile a run whose throughput you report.
"""

from __future__ import annotations

import contextlib
import functools
import time
from collections import defaultdict
from collections.abc import Callable, Iterator
from typing import Any, TypeVar

ENGINE = "autograd engine"
_R = TypeVar("_R")


class Profile:
    def __init__(self) -> None:
        self.total: dict[tuple[str, bool], float] = defaultdict(float)
        self.self_time: dict[tuple[str, bool], float] = defaultdict(float)
        self.calls: dict[tuple[str, bool], int] = defaultdict(int)
        self._child: list[float] = []

    def timed(self, name: str, fn: Callable[..., _R], *args: Any, backward: bool = True) -> _R:
        from tensorgrad_b200.device import synchronize

        synchronize()
        self._child.append(0.0)
        t0 = time.perf_counter()
        try:
            return fn(*args)
        finally:
            synchronize()
            dt = time.perf_counter() - t0
            child = self._child.pop()
            key = (name, backward)
            self.total[key] += dt
            self.self_time[key] += dt - child
            self.calls[key] += 1
            if self._child:
                self._child[-1] += dt

    def table(self, limit: int = 20) -> str:
        rows = sorted(self.self_time.items(), key=lambda kv: -kv[1])[:limit]
        grand = sum(self.self_time.values()) or 1.0
        lines = [f"{'op':<28}{'pass':<10}{'calls':>8}{'self ms':>12}{'share':>9}"]
        for (name, bwd), t in rows:
            lines.append(
                f"{name:<28}{'backward' if bwd else 'forward':<10}"
                f"{self.calls[(name, bwd)]:>8}{1e3 * t:>12.3f}{100 * t / grand:>8.1f}%"
            )
        return "\n".join(lines)


_active: list[Profile] = []


def active() -> Profile | None:
    return _active[-1] if _active else None


@contextlib.contextmanager
def profile() -> Iterator[Profile]:
    prof = Profile()
    _active.append(prof)
    try:
        yield prof
    finally:
        _active.pop()


def profiled(name: str) -> Callable[[Callable[..., _R]], Callable[..., _R]]:
    """Decorator: time the forward call of a public op when a profile is active."""

    def deco(fn: Callable[..., _R]) -> Callable[..., _R]:
        @functools.wraps(fn)
        def wrapper(*args: Any, **kwargs: Any) -> _R:
            prof = active()
            if prof is None:
                return fn(*args, **kwargs)
            return prof.timed(name, lambda: fn(*args, **kwargs), backward=False)

        return wrapper

    return deco
