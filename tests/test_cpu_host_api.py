"""Host-side parts of the API that need no GPU: the DataLoader's batch order (against the
reference's own, ``tests/golden/ops_extra.npz``), its argument checks, the graph drawings of
``viz`` (the reference's output format, on graph nodes made without device data) and the
host allocator switch."""

from __future__ import annotations

import re

import numpy as np
import pytest

from tests.conftest import load_golden


def test_data_loader_order_matches_reference():
    from tensorgrad_b200.utils import DataLoader

    gold = load_golden("ops_extra.npz")
    loader = DataLoader(np.arange(10), batch_size=4, shuffle=True, seed=5)
    assert len(loader) == 3
    for epoch in range(2):
        order = np.concatenate(list(loader.batches()))
        np.testing.assert_array_equal(order, gold[f"loader_epoch{epoch}"])
    assert len(DataLoader(np.zeros((10, 3)), batch_size=4, drop_last=True)) == 2
    assert [b.tolist() for b in DataLoader(np.zeros(5), batch_size=2).batches()] == [
        [0, 1], [2, 3], [4]]
    with pytest.raises(ValueError, match="different lengths"):
        DataLoader(np.zeros(3), np.zeros(4))
    with pytest.raises(ValueError, match="positive"):
        DataLoader(np.zeros(3), batch_size=0)
    with pytest.raises(ValueError, match="at least one"):
        DataLoader()


class _Meta:
    """Stands in for device data: the drawings read shapes only."""

    def __init__(self, shape):
        self.shape = tuple(shape)
        self.ndim = len(self.shape)
        self.dtype = np.dtype(np.float64)
        self.size = int(np.prod(self.shape))


def _leaf(shape, requires_grad):
    from tensorgrad_b200.tensor import Tensor

    t = Tensor._wrap(_Meta(shape))
    t._requires_grad = requires_grad
    return t


def _op(name, shape, *parents):
    from tensorgrad_b200.autograd import Node

    t = _leaf(shape, True)
    t._node = Node(name, parents, lambda g, need: (None,) * len(parents))
    return t


def _small_graph():
    w, x = _leaf((2, 3), True), _leaf((3,), False)
    y = _op("tanh", (2,), _op("matmul", (2,), w, x))
    return _op("sum", (), _op("mul", (2,), y, y)), {"w": w, "x": x}


def test_drawings_match_the_reference_text():
    """``viz.to_mermaid`` / ``to_dot`` of graphs of the same shape as two the reference drew,
    character for character (tests/golden/viz.npz), from graph nodes made without device
    data."""
    from tensorgrad_b200 import viz

    gold = load_golden("viz.npz")
    loss, names = _small_graph()
    assert viz.to_mermaid(loss, names=names, direction="LR") == str(gold["mermaid_lr"])
    assert viz.to_dot(loss, names=names) == str(gold["dot_tb"])
    a = _leaf((2,), True)
    hidden = _op("relu", (2,), a)
    out = _op("sum", (), hidden)
    named = {'say "a"': a, "hidden": hidden}
    assert viz.to_mermaid(out, names=named) == str(gold["mermaid_named"])
    assert viz.to_dot(out, names=named) == str(gold["dot_named"])
    dot = viz.to_dot(loss, names=names)
    declared = set(re.findall(r"^  (n\d+) \[label=", dot, re.M))
    edges = re.findall(r"^  (n\d+) -> (n\d+);", dot, re.M)
    assert declared == {f"n{i}" for i in range(6)} and len(edges) == 5  # y * y: one edge
    with pytest.raises(ValueError, match="at least one"):
        viz.to_dot()


def test_retain_freed_memory_reports_glibc():
    from tensorgrad_b200.utils import retain_freed_memory

    assert retain_freed_memory() in (True, False)


class _Group:
    def __init__(self, lr):
        self.lr = self.initial_lr = lr


class _Opt:
    def __init__(self, *lrs):
        self.param_groups = [_Group(lr) for lr in lrs]


def test_lr_schedules():
    import math

    from tensorgrad_b200.optim.lr_scheduler import CosineWarmupLR, LRScheduler, StepLR

    opt = _Opt(0.1, 1.0)
    sched = StepLR(opt, step_size=2, gamma=0.5)
    seen = [sched.get_last_lr()]
    for _ in range(4):
        sched.step()
        seen.append(sched.get_last_lr())
    assert seen == [[0.1, 1.0], [0.1, 1.0], [0.05, 0.5], [0.05, 0.5], [0.025, 0.25]]
    opt = _Opt(1.0)
    cos = CosineWarmupLR(opt, warmup_steps=2, total_steps=6, min_lr_ratio=0.1)
    got = [cos.factor(s) for s in range(8)]
    want = [0.5, 1.0] + [0.1 + 0.9 * 0.5 * (1 + math.cos(math.pi * min(t / 4, 1.0)))
                         for t in range(6)]
    assert got == want and opt.param_groups[0].lr == 0.5
    for bad in (dict(warmup_steps=3, total_steps=2), dict(warmup_steps=-1, total_steps=2),
                dict(warmup_steps=0, total_steps=0)):
        with pytest.raises(ValueError, match="warmup_steps"):
            CosineWarmupLR(_Opt(1.0), **bad)
    with pytest.raises(ValueError, match="min_lr_ratio"):
        CosineWarmupLR(_Opt(1.0), 0, 5, min_lr_ratio=2.0)
    with pytest.raises(ValueError, match="step_size"):
        StepLR(_Opt(1.0), 0)
    with pytest.raises(TypeError):
        LRScheduler(_Opt(1.0))  # abstract


def test_profile_self_times_and_table(monkeypatch):
    from tensorgrad_b200 import device, profiler

    monkeypatch.setattr(device, "synchronize", lambda: None)  # no device: host timing only

    @profiler.profiled("outer")
    def outer():
        return inner() + 1

    @profiler.profiled("inner")
    def inner():
        return 1

    with profiler.profile() as prof:
        assert outer() == 2
        prof.timed("vjp", True, lambda: None)
    assert prof.ops["outer"].forward_calls == prof.ops["inner"].forward_calls == 1
    assert prof.ops["vjp"].backward_calls == 1 and prof.ops["vjp"].forward_calls == 0
    assert prof.profiled_seconds <= prof.wall_seconds
    lines = prof.table().splitlines()
    assert lines[0].split() == ["op", "fwd", "calls", "fwd", "ms", "bwd", "calls", "bwd", "ms",
                                "total", "ms", "share"]
    assert set(lines[1]) == {"-"} and len(lines) == 6 and "wall time" in lines[-1]
    assert len(prof.table(limit=1).splitlines()) == 4
    assert profiler.active() is None
    with pytest.raises(RuntimeError, match="nested"), profiler.profile(), profiler.profile():
        pass


def test_gradient_slot_is_handed_out_once_per_pass():
    """A VJP may write a parameter's gradient straight into its arena slot only while the slot
    holds no gradient of this pass, nobody else took it, and no clip factor is pending; the
    claim ends when the engine accumulates the gradient or on zero_grad (host logic only)."""
    from tensorgrad_b200.ops._util import grad_buffer

    class _Arena:
        pending_clip = None

    slot = _Meta((2, 3))
    p = _leaf((2, 3), True)
    p._grad_slot, p._arena = slot, _Arena()
    assert p._grad_target() is slot
    assert p._grad_target() is None  # taken: a second contribution gets a buffer of its own
    p.zero_grad()
    assert p._grad_target() is slot
    p.zero_grad()
    p._arena.pending_clip = 0.5
    assert p._grad_target() is None
    p._arena.pending_clip = None
    p._grad = _leaf((2, 3), False)  # a gradient from an earlier pass: accumulate, not overwrite
    assert p._grad_target() is None
    p._grad = None
    assert grad_buffer(p, (2, 3), np.float64) is slot
    q = _leaf((2, 3), True)
    assert q._grad_target() is None  # no arena slot


def test_device_array_reads_numpy_methods_from_a_host_copy():
    """``tensor.data.argmax(1)``, ``.mean()`` and the like work as on the reference's NumPy
    arrays (read-only, from a host copy); private names are not forwarded."""
    from tensorgrad_b200.device import DeviceArray

    host = np.array([[0.5, 2.0, -1.0], [3.0, 1.0, 1.5]])

    class _Copyable(DeviceArray):
        def numpy(self, out=None):
            return host.copy()

    a = _Copyable(None, 0, host.shape, host.dtype)
    np.testing.assert_array_equal(a.argmax(1), [1, 0])
    assert a.mean() == pytest.approx(host.mean())
    assert a.max(axis=0).tolist() == [3.0, 2.0, 1.5]
    with pytest.raises(AttributeError):
        a._not_there
    assert not hasattr(a, "mul_")  # not a NumPy attribute: no host copy, no forwarding


def test_bench_readback_copies_every_result_without_blocking():
    """The end-to-end loop's read-back: one asynchronous copy per result tensor into
    alternating page-locked buffers, a wait only on the copy of two steps back, and the last
    result's value after the closing synchronisation (fakes stand in for the device)."""
    import ctypes
    import types

    import bench

    queried: list[int] = []

    class _Event:
        count = 0

        def __init__(self):
            _Event.count += 1
            self.id = _Event.count

        def record(self):
            pass

        def query(self):
            queried.append(self.id)
            return True

    copies: list[tuple[int, int]] = []

    def memcpy_d2h(dst, src, nbytes, stream):
        ctypes.memmove(dst, src, nbytes)
        copies.append((dst, nbytes))
        return 0

    fake_device = types.SimpleNamespace(pinned_empty=lambda shape, dt: np.empty(shape, dt),
                                        stream=lambda: 0, _Event=_Event)
    fake_lib = types.SimpleNamespace(tg_memcpy_d2h=memcpy_d2h)

    def result(value):
        host = np.array(value, dtype=np.float32)
        data = types.SimpleNamespace(ptr=host.ctypes.data, nbytes=host.nbytes)
        return types.SimpleNamespace(shape=host.shape, dtype=host.dtype, data=data, keep=host)

    reader = bench._AsyncReadback(fake_lib, fake_device)
    assert reader.value() is None
    losses = [result(v) for v in (4.0, 3.5, 3.25)]
    for r in losses:
        reader.issue(r)
    assert len(copies) == 3 and copies[0][0] != copies[1][0] and copies[0][0] == copies[2][0]
    assert queried == [1]  # the third step waited for the first step's copy only
    assert reader.value() == 3.25


def test_profile_table_text_matches_reference():
    """The profiler's table, character for character, against the reference's table for the
    same statistics (tests/golden/profiler_table.npz)."""
    from tensorgrad_b200 import profiler
    from tests.golden.specs import PROFILE_ROWS

    gold = load_golden("profiler_table.npz")
    prof = profiler.Profile()
    for name, fc, fs, bc, bs in PROFILE_ROWS:
        prof.ops[name] = profiler.OpStats(fc, fs, bc, bs)
    prof.wall_seconds = 0.125
    assert prof.table() == str(gold["table"])
    assert prof.table(limit=2) == str(gold["table_limit2"])
