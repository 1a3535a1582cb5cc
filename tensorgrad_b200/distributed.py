"""Data-parallel training: one process per GPU, gradients averaged over the ranks.

The reference is single-process; this module adds the exchange step that batch sharding
needs. Every parameter's gradient lives in a flat arena (see ``optim.arena``), so the
average runs in place on contiguous buckets of those buffers, with no gather or scatter.

Buckets are consecutive parameters of an arena, about ``bucket_bytes`` each. The engine's
leaf hook (``autograd.add_leaf_hook``) fires when a parameter's gradient is final; when the
last parameter of a bucket is final, that bucket's all-reduce is launched at once and overlaps
the rest of the backward walk. ``reduce()`` (after ``backward``) launches any bucket not yet
launched, in bucket order, then waits. Every rank runs the same graph, so the hooks fire in
the same order and all ranks issue the same collectives in the same order.

The exchange goes through a :class:`Communicator`:

* :class:`NcclCommunicator` (the default on GPUs): NCCL through ``libtgb200.so``, set up
  nonblocking with a deadline, collectives on their own stream, and a host-side watch that
  aborts the communicator and raises :class:`CollectiveTimeout` / :class:`CollectiveError`
  when a collective fails or does not finish in time (a rank that died or left);
* :class:`ProcessGroupCommunicator`: ``torch.distributed`` (``gloo`` ranks on CPU in tests);
* :class:`FaultyCommunicator`: a test double around either that drops, delays or corrupts
  chosen buckets, to show that the reducer surfaces each failure.

With ``verify=True`` the reducer also compares a float64 checksum of every reduced bucket
across the ranks and raises :class:`CollectiveMismatch` when they differ (silent corruption
on one rank). ``torch.distributed`` is used only to bootstrap: to share the NCCL unique id
through its store, for barriers and for the max-over-ranks timing of the benchmark.
"""

from __future__ import annotations

import ctypes
import os
import sys
import time
from collections.abc import Callable, Sequence
from typing import Any

import numpy as np

from tensorgrad_b200.optim.arena import flatten_parameters
from tensorgrad_b200.tensor import Tensor

__all__ = ["BucketedAllReduce", "CollectiveError", "CollectiveMismatch", "CollectiveTimeout",
           "Communicator", "FaultyCommunicator", "GradientAllReduce", "NcclCommunicator",
           "ProcessGroupCommunicator", "barrier", "check_peers", "leave_job", "max_over_ranks",
           "plan_buckets", "world_size"]


class CollectiveError(RuntimeError):
    """A collective failed; the communicator that ran it is no longer usable."""


class CollectiveTimeout(CollectiveError, TimeoutError):
    """A collective did not finish before its deadline (a rank died, left or hangs)."""


class CollectiveMismatch(CollectiveError):
    """Ranks ended a reduction with different values (corruption on some rank)."""


def _dist():
    """``torch.distributed`` when the program initialised a process group, else None. Never
    imports torch itself: a process that did not load it has no process group."""
    dist = sys.modules.get("torch.distributed")
    if dist is None:
        return None
    return dist if dist.is_available() and dist.is_initialized() else None


def world_size() -> int:
    d = _dist()
    return d.get_world_size() if d is not None else int(os.environ.get("WORLD_SIZE", "1"))


def rank() -> int:
    d = _dist()
    return d.get_rank() if d is not None else int(os.environ.get("RANK", "0"))


def barrier() -> None:
    d = _dist()
    if d is not None:
        d.barrier()


def max_over_ranks(value: float) -> float:
    """The maximum of a host scalar over all ranks (timings are max over ranks)."""
    d = _dist()
    if d is None:
        return value
    import torch

    backend = d.get_backend()
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    d.all_reduce(t, op=d.ReduceOp.MAX)
    return float(t.item())


_LEFT = "tgb200/left/{}"


def leave_job() -> None:
    """Announce, through the process group's store, that this rank stops after the step it
    finished. The other ranks' reducers check before each step's first launch and raise
    :class:`CollectiveError` there instead of waiting for this rank; a step already under way
    on another rank runs into its deadline (:class:`CollectiveTimeout`). Call it between
    steps, with none of this rank's collectives in flight."""
    d = _dist()
    if d is not None:
        d.distributed_c10d._get_default_store().set(_LEFT.format(rank()), b"1")


def check_peers() -> None:
    """Raise :class:`CollectiveError` if another rank announced with :func:`leave_job`."""
    d = _dist()
    if d is None:
        return
    store = d.distributed_c10d._get_default_store()
    for r in range(d.get_world_size()):
        if r != d.get_rank() and store.check([_LEFT.format(r)]):
            raise CollectiveError(f"rank {r} left the job; no gradient exchange with it")


def plan_buckets(sizes: Sequence[int], offsets: Sequence[int], itemsize: int,
                 bucket_bytes: int) -> list[tuple[int, int, list[int]]]:
    """Group consecutive parameters (element ``sizes`` at element ``offsets`` of one flat
    buffer) into buckets of at least ``bucket_bytes`` (the last may be smaller). Returns
    ``(start, stop, member indices)`` per bucket, ``stop`` the next bucket's start (so the
    padding between slots is reduced too and the buckets tile the buffer)."""
    buckets: list[tuple[int, int, list[int]]] = []
    members: list[int] = []
    start = offsets[0] if offsets else 0
    for i, (size, off) in enumerate(zip(sizes, offsets, strict=True)):
        members.append(i)
        end = off + size
        if (end - start) * itemsize >= bucket_bytes:
            nxt = offsets[i + 1] if i + 1 < len(offsets) else end
            buckets.append((start, nxt, members))
            members, start = [], nxt
    if members:
        buckets.append((start, offsets[-1] + sizes[-1], members))
    return buckets


# ----------------------------------------------------------------------------- communicators
def _slice(buf: Any, start: int, stop: int) -> Any:
    """Elements ``[start, stop)`` of a flat buffer (a device array or a framework tensor)."""
    if hasattr(buf, "flat_view"):
        return buf.flat_view(start, stop - start)
    return buf[start:stop]


class Communicator:
    """The exchange step's interface: ``all_reduce_avg`` launches the in-place average of one
    bucket over the ranks and returns a handle; ``wait`` returns once every handle has
    completed, or raises :class:`CollectiveTimeout` / :class:`CollectiveError`;
    ``values_agree`` says whether a small host vector is identical on every rank (the same
    answer on every rank)."""

    world: int = 1

    def all_reduce_avg(self, view: Any) -> Any:
        raise NotImplementedError

    def wait(self, handles: list[Any], deadline_s: float) -> None:
        raise NotImplementedError

    def values_agree(self, values: np.ndarray, deadline_s: float) -> bool:
        raise NotImplementedError

    def close(self) -> None:
        """Release the communicator (idempotent)."""


class LocalCommunicator(Communicator):
    """One rank: nothing to exchange."""

    def all_reduce_avg(self, view: Any) -> Any:
        return None

    def wait(self, handles: list[Any], deadline_s: float) -> None:
        return None

    def values_agree(self, values: np.ndarray, deadline_s: float) -> bool:
        return True


class ProcessGroupCommunicator(Communicator):
    """``torch.distributed`` collectives on framework tensors (``gloo`` on CPU in the tests;
    it sums, then scales by 1/world)."""

    def __init__(self) -> None:
        d = _dist()
        if d is None:
            raise RuntimeError("ProcessGroupCommunicator needs an initialised process group")
        self.dist = d
        self.world = d.get_world_size()

    def all_reduce_avg(self, view: Any) -> Any:
        d = self.dist
        return view, d.all_reduce(view, op=d.ReduceOp.SUM, async_op=True)

    def wait(self, handles: list[Any], deadline_s: float) -> None:
        import datetime

        end = time.monotonic() + deadline_s
        for view, work in handles:
            left = max(end - time.monotonic(), 0.001)
            try:
                done = work.wait(timeout=datetime.timedelta(seconds=left))
            except RuntimeError as exc:
                raise CollectiveTimeout(f"gradient all-reduce did not finish in {deadline_s} s: "
                                        f"{exc}") from exc
            if done is False:
                raise CollectiveTimeout(f"gradient all-reduce did not finish in {deadline_s} s")
            view.mul_(1.0 / self.world)

    def values_agree(self, values: np.ndarray, deadline_s: float) -> bool:
        import torch

        mine = torch.tensor(values, dtype=torch.float64)
        mean = mine.clone()
        self.wait([self.all_reduce_avg(mean)], deadline_s)
        flag = torch.tensor([0.0 if torch.equal(mine, mean) else 1.0], dtype=torch.float64)
        self.wait([self.all_reduce_avg(flag)], deadline_s)
        return float(flag.item()) == 0.0


def _nccl_library() -> str | None:
    """The NCCL the process's framework ships (so one NCCL serves the whole process), if any;
    otherwise the system's ``libnccl.so.2``."""
    try:
        import nvidia.nccl  # type: ignore[import-not-found]
    except ImportError:
        return None
    for base in getattr(nvidia.nccl, "__path__", []):
        path = os.path.join(base, "lib", "libnccl.so.2")
        if os.path.exists(path):
            return path
    return None


class NcclCommunicator(Communicator):
    """NCCL through ``libtgb200.so`` (``tg_comm_*``): in-place averages of device buckets on
    the communicator's stream, overlapping the compute stream; ``wait`` watches them with a
    deadline and, on a failure or an expired deadline, the library aborts the communicator
    and this raises. Each rank's set-up waits at most ``timeout_s`` for the others."""

    _uid_seq = 0

    def __init__(self, nranks: int, rank_id: int, unique_id: bytes, timeout_s: float = 60.0) -> None:
        from tensorgrad_b200 import device
        from tensorgrad_b200._lib import check, lib

        self.world, self.rank = nranks, rank_id
        self.timeout_s = timeout_s
        device.current_device()
        check(lib.tg_comm_load((_nccl_library() or "").encode()), "load NCCL")
        handle = ctypes.c_void_p()
        uid = ctypes.create_string_buffer(unique_id, 128)
        status = lib.tg_comm_init(nranks, rank_id, uid, timeout_s, ctypes.byref(handle))
        self._raise_for(status, "NCCL communicator set-up")
        self.handle: int | None = handle.value

    @staticmethod
    def _raise_for(status: int, what: str) -> None:
        from tensorgrad_b200._lib import check, last_error

        if status == 5:
            raise CollectiveTimeout(f"{what}: {last_error()}")
        if status == 7:
            raise CollectiveError(f"{what}: {last_error()}")
        check(status, what)

    @classmethod
    def from_process_group(cls, timeout_s: float = 60.0) -> NcclCommunicator:
        """Every rank of the initialised process group: rank 0 makes the unique id, the
        others read it from the process group's store."""
        from tensorgrad_b200._lib import check, lib

        d = _dist()
        if d is None:
            raise RuntimeError("NcclCommunicator.from_process_group needs torch.distributed")
        store = d.distributed_c10d._get_default_store()
        key = f"tgb200/nccl_uid/{cls._uid_seq}"
        cls._uid_seq += 1
        if d.get_rank() == 0:
            check(lib.tg_comm_load((_nccl_library() or "").encode()), "load NCCL")
            buf = ctypes.create_string_buffer(128)
            check(lib.tg_comm_unique_id(buf, 128), "NCCL unique id")
            store.set(key, buf.raw)
        uid = bytes(store.get(key))
        return cls(d.get_world_size(), d.get_rank(), uid, timeout_s)

    def all_reduce_avg(self, view: Any) -> Any:
        from tensorgrad_b200 import device
        from tensorgrad_b200._lib import lib

        if self.handle is None:
            raise CollectiveError("the NCCL communicator was closed or aborted")
        status = lib.tg_comm_all_reduce(self.handle, view.ptr, view.size,
                                        device.dtype_code(view.dtype), 1, device.stream(),
                                        self.timeout_s)
        self._raise_for(status, "gradient all-reduce")
        return None

    def wait(self, handles: list[Any], deadline_s: float) -> None:
        from tensorgrad_b200 import device
        from tensorgrad_b200._lib import check, lib

        if self.handle is None:
            raise CollectiveError("the NCCL communicator was closed or aborted")
        status = lib.tg_comm_wait(self.handle, deadline_s)
        if status != 0:  # the library aborted the communicator: free what is left of it
            lib.tg_comm_destroy(self.handle, 1.0)
            self.handle = None
        self._raise_for(status, "gradient all-reduce")
        check(lib.tg_comm_join(self.handle, device.stream()), "join collectives")

    def values_agree(self, values: np.ndarray, deadline_s: float) -> bool:
        from tensorgrad_b200 import device

        mine = np.ascontiguousarray(values, dtype=np.float64)
        mean = device.from_numpy(mine)
        self.all_reduce_avg(mean)
        self.wait([], deadline_s)
        flag = device.from_numpy(np.array([0.0 if np.array_equal(mean.numpy(), mine) else 1.0]))
        self.all_reduce_avg(flag)
        self.wait([], deadline_s)
        return float(flag.numpy()[0]) == 0.0

    def close(self) -> None:
        from tensorgrad_b200._lib import lib

        if self.handle is not None:
            lib.tg_comm_destroy(self.handle, self.timeout_s)
            self.handle = None


class FaultyCommunicator(Communicator):
    """Test double: forwards to ``inner`` but, for the (step, bucket) pairs in ``faults``,
    ``"drop"``s the bucket (never launches it: every rank's wait then runs into the
    deadline), ``"delay"``s its launch by ``delay_s`` or ``"corrupt"``s this rank's result
    after the reduction (the reducer's ``verify`` must catch it). The reducer calls
    ``next_step()`` once per step."""

    def __init__(self, inner: Communicator, faults: dict[tuple[int, int], str],
                 delay_s: float = 0.2) -> None:
        self.inner, self.faults, self.delay_s = inner, dict(faults), delay_s
        self.world = inner.world
        self.step, self.bucket = 0, 0
        self._corrupt: list[Any] = []

    def next_step(self) -> None:
        self.step += 1
        self.bucket = 0

    def all_reduce_avg(self, view: Any) -> Any:
        fault = self.faults.get((self.step, self.bucket))
        self.bucket += 1
        if fault == "drop":
            return _Dropped()
        if fault == "delay":
            time.sleep(self.delay_s)
        if fault == "corrupt":
            self._corrupt.append(view)
        return self.inner.all_reduce_avg(view)

    def wait(self, handles: list[Any], deadline_s: float) -> None:
        if any(isinstance(h, _Dropped) for h in handles):
            time.sleep(deadline_s)
            raise CollectiveTimeout(f"gradient all-reduce did not finish in {deadline_s} s "
                                    "(a bucket was never exchanged)")
        self.inner.wait(handles, deadline_s)
        for view in self._corrupt:
            view.mul_(1.0 + 1e-3) if hasattr(view, "mul_") else None
        self._corrupt.clear()

    def values_agree(self, values: np.ndarray, deadline_s: float) -> bool:
        return self.inner.values_agree(values, deadline_s)

    def close(self) -> None:
        self.inner.close()


class _Dropped:
    """Handle of a bucket a FaultyCommunicator never launched."""


# ----------------------------------------------------------------------------- the reducer
class BucketedAllReduce:
    """Averages flat gradient buffers across ranks bucket by bucket.

    ``buffers`` lists, per flat buffer (a device array, or a framework tensor for CPU tests),
    the ids, element offsets and sizes of the parameters whose gradients live in it.
    ``ready(param_id)`` marks one parameter's gradient final; a bucket whose members are all
    final is launched at once. ``finish()`` launches the rest in bucket order and waits for
    all of them, at most ``deadline_s`` seconds; with ``verify`` it then checks that every
    rank holds the same reduced values (a float64 checksum per bucket).
    """

    def __init__(self, buffers: Sequence[tuple[Any, list[int], list[int], list[int]]],
                 bucket_bytes: int = 32 << 20, comm: Communicator | None = None,
                 deadline_s: float = 300.0, verify: bool = False) -> None:
        self.comm = comm if comm is not None else _default_process_group_comm()
        self.deadline_s, self.verify = deadline_s, verify
        self.views: list[Any] = []
        self.members: list[int] = []  # member count per bucket
        self.owner: dict[int, int] = {}
        for flat, ids, offsets, sizes in buffers:
            itemsize = flat.dtype.itemsize if hasattr(flat, "flat_view") else flat.element_size()
            for start, stop, idx in plan_buckets(sizes, offsets, itemsize, bucket_bytes):
                b = len(self.views)
                self.views.append(_slice(flat, start, stop))
                self.members.append(len(idx))
                for i in idx:
                    self.owner[ids[i]] = b
        self.pending = list(self.members)
        self.launched = [False] * len(self.views)
        self.order: list[int] = []       # launch order of the current step
        self.last_order: list[int] = []  # launch order of the last finished step
        self.handles: list[Any] = []
        #: Called before a step's first launch; raises if a peer is known to be gone.
        self.peer_check: Callable[[], None] | None = (
            check_peers if self.comm.world > 1 and _dist() is not None else None)

    def _launch(self, b: int) -> None:
        if not self.order and self.peer_check is not None:
            self.peer_check()
        self.launched[b] = True
        self.order.append(b)
        if self.comm.world > 1:
            self.handles.append(self.comm.all_reduce_avg(self.views[b]))

    def ready(self, param_id: int) -> None:
        b = self.owner.get(param_id)
        if b is None or self.launched[b]:
            return
        self.pending[b] -= 1
        if self.pending[b] == 0:
            self._launch(b)

    def finish(self) -> None:
        for b in range(len(self.views)):
            if not self.launched[b]:
                self._launch(b)
        handles, self.handles = self.handles, []
        self.pending = list(self.members)
        self.launched = [False] * len(self.views)
        self.last_order, self.order = self.order, []
        if self.comm.world > 1:
            self.comm.wait(handles, self.deadline_s)
            if self.verify:
                sums = np.array([_checksum(v) for v in self.views], dtype=np.float64)
                if not self.comm.values_agree(sums, self.deadline_s):
                    raise CollectiveMismatch("the reduced gradients differ across ranks")
        if isinstance(self.comm, FaultyCommunicator):
            self.comm.next_step()


def _checksum(view: Any) -> float:
    if hasattr(view, "flat_view"):
        return float(np.asarray(view.numpy(), dtype=np.float64).sum())
    return float(view.double().sum().item())


def _default_process_group_comm() -> Communicator:
    d = _dist()
    if d is None or d.get_world_size() == 1:
        return LocalCommunicator()
    return ProcessGroupCommunicator()


class GradientAllReduce:
    """Averages every parameter gradient across ranks, in place in the gradient arenas,
    overlapping each bucket's all-reduce with the rest of the backward walk.

    Call ``reduce()`` once after every ``backward()`` (before clipping and the optimizer). The
    exchange uses ``comm`` or, on GPUs with an initialised process group, a new
    :class:`NcclCommunicator`; a failed or late exchange raises :class:`CollectiveError` /
    :class:`CollectiveTimeout` from ``reduce()`` (at most ``deadline_s`` seconds).
    """

    def __init__(self, params: Sequence[Tensor], bucket_bytes: int = 32 << 20,
                 overlap: bool = True, comm: Communicator | None = None,
                 deadline_s: float = 300.0, verify: bool = False) -> None:
        from tensorgrad_b200 import autograd

        self.arenas = flatten_parameters(list(params))
        if comm is None:
            comm = (NcclCommunicator.from_process_group(timeout_s=min(deadline_s, 120.0))
                    if world_size() > 1 else LocalCommunicator())
        self.comm = comm
        buffers = [(arena.grad_buf, [id(p) for p in arena.params], list(arena.offsets),
                    [p.size for p in arena.params]) for arena in self.arenas]
        self.buckets = BucketedAllReduce(buffers, bucket_bytes, comm, deadline_s, verify)
        self.closed = False
        self._remove: Callable[[], None] | None = None
        if overlap and comm.world > 1:
            self._remove = autograd.add_leaf_hook(lambda t: self.buckets.ready(id(t)))

    def leave(self) -> None:
        """This rank stops after the step it finished (see :func:`leave_job`)."""
        leave_job()

    def reduce(self) -> None:
        for arena in self.arenas:
            arena.settle_clip()
        self.buckets.finish()

    def close(self, abort: bool = False) -> None:
        """Release the communicator; ``abort`` when a peer is gone (no final handshake)."""
        if self._remove is not None:
            self._remove()
            self._remove = None
        if not self.closed:
            if abort and isinstance(self.comm, NcclCommunicator) and self.comm.handle:
                from tensorgrad_b200._lib import lib

                lib.tg_comm_abort(self.comm.handle)
                lib.tg_comm_destroy(self.comm.handle, 1.0)
                self.comm.handle = None
            else:
                self.comm.close()
        self.closed = True
