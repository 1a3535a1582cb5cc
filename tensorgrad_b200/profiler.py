"""Per-op timing (the reference's ``tensorgrad.profiler`` API).

    with tensorgrad_b200.profiler.profile() as prof:
        loss = tg.cross_entropy(model(x), y)
        loss.backward()
    print(prof.table())

While a profile is open, each public op call and each VJP the engine runs is timed between
two device synchronisations, so a row holds the device work the call launched plus its host
overhead. Nested timed calls (the ops inside a composite op or a graph VJP) are subtracted
from their caller: rows are self times and sum to the profiled total. The backward engine's
own work outside the VJPs has a row of its own (``ENGINE``). The synchronisations change the
timing of the code they wrap: never profile a run whose throughput you report.
"""

from __future__ import annotations

import contextlib
import functools
import time
from collections.abc import Callable, Iterator
from dataclasses import dataclass
from typing import Any, TypeVar

__all__ = ["ENGINE", "OpStats", "Profile", "profile", "profiled"]

ENGINE = "autograd engine"  # the row of the backward engine's own time
_T = TypeVar("_T")


@dataclass
class OpStats:
    """One op's calls and self seconds, forward and backward apart."""

    forward_calls: int = 0
    forward_seconds: float = 0.0
    backward_calls: int = 0
    backward_seconds: float = 0.0

    @property
    def total_seconds(self) -> float:
        return self.forward_seconds + self.backward_seconds

    def add(self, backward: bool, seconds: float) -> None:
        if backward:
            self.backward_calls += 1
            self.backward_seconds += seconds
        else:
            self.forward_calls += 1
            self.forward_seconds += seconds


# Columns of ``Profile.table``: header, and the cell of a row (9 characters wide).
_COLUMNS: list[tuple[str, Callable[[OpStats], str]]] = [
    ("fwd calls", lambda s: f"{s.forward_calls:>9}"),
    ("fwd ms", lambda s: f"{1e3 * s.forward_seconds:>9.2f}"),
    ("bwd calls", lambda s: f"{s.backward_calls:>9}"),
    ("bwd ms", lambda s: f"{1e3 * s.backward_seconds:>9.2f}"),
    ("total ms", lambda s: f"{1e3 * s.total_seconds:>9.2f}"),
]


class Profile:
    """What one ``profile()`` block collected: ``ops`` maps an op name to its
    :class:`OpStats`; ``wall_seconds`` is the block's duration."""

    def __init__(self) -> None:
        self.ops: dict[str, OpStats] = {}
        self.wall_seconds = 0.0
        self._inner: list[float] = []  # seconds of timed calls nested in each open call

    def timed(self, name: str, backward: bool, fn: Callable[..., _T], *args: Any,
              **kwargs: Any) -> _T:
        """``fn(*args, **kwargs)``, its self time charged to ``name``."""
        from tensorgrad_b200.device import synchronize

        synchronize()
        self._inner.append(0.0)
        t0 = time.perf_counter()
        try:
            return fn(*args, **kwargs)
        finally:
            synchronize()
            spent = time.perf_counter() - t0
            nested = self._inner.pop()
            if self._inner:
                self._inner[-1] += spent
            self.ops.setdefault(name, OpStats()).add(backward, spent - nested)

    @property
    def profiled_seconds(self) -> float:
        """All rows together: the time inside ops and the engine."""
        return sum(stats.total_seconds for stats in self.ops.values())

    def table(self, limit: int | None = None) -> str:
        """One aligned row per op (largest total first; the first ``limit`` rows) in
        milliseconds with each op's share, then the profiled and wall totals."""
        total = self.profiled_seconds or 1.0
        width = max(len(name) for name in ["op", *self.ops])
        header = "  ".join([f"{'op':<{width}}", *(f"{h:>9}" for h, _ in _COLUMNS),
                            f"{'share':>6}"])
        out = [header, "-" * len(header)]
        ranked = sorted(self.ops.items(), key=lambda item: -item[1].total_seconds)
        for name, stats in ranked[:limit]:
            cells = [f"{name:<{width}}", *(cell(stats) for _, cell in _COLUMNS),
                     f"{stats.total_seconds / total:>6.1%}"]
            out.append("  ".join(cells))
        inside, wall = 1e3 * self.profiled_seconds, 1e3 * self.wall_seconds
        out.append(f"ops and engine: {inside:.2f} ms of {wall:.2f} ms wall time "
                   f"({wall - inside:.2f} ms elsewhere: Python code between ops, optimiser, "
                   "data)")
        return "\n".join(out)


class _Current:
    profile: Profile | None = None


def active() -> Profile | None:
    """The open profile, or ``None``."""
    return _Current.profile


@contextlib.contextmanager
def profile() -> Iterator[Profile]:
    """Time the ops run inside the ``with`` block (one block at a time, one thread)."""
    if _Current.profile is not None:
        raise RuntimeError("profile() blocks cannot be nested")
    prof = _Current.profile = Profile()
    t0 = time.perf_counter()
    try:
        yield prof
    finally:
        prof.wall_seconds = time.perf_counter() - t0
        _Current.profile = None


def profiled(name: str) -> Callable[[Callable[..., _T]], Callable[..., _T]]:
    """Mark an op function: while a profile is open its calls are timed as ``name``."""

    def wrap(fn: Callable[..., _T]) -> Callable[..., _T]:
        @functools.wraps(fn)
        def call(*args: Any, **kwargs: Any) -> _T:
            prof = _Current.profile
            if prof is not None:
                return prof.timed(name, False, fn, *args, **kwargs)
            return fn(*args, **kwargs)

        return call

    return wrap
