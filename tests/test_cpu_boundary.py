"""CPU-only checks: the C-ABI library builds, loads without a GPU and exports every symbol
that include/tgb200.h declares; the ctypes binding covers the same set; the host engine's
tape walk behaves like the reference's (driven with host arrays, no kernels)."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tgb200.h")


def header_functions() -> set[str]:
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(tg_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def libpath() -> str:
    from tensorgrad_b200 import _build

    if not os.path.exists(_build.LIB):
        _build.build()
    return _build.LIB


def test_library_exports_every_declared_symbol(libpath):
    dll = ctypes.CDLL(libpath)
    names = header_functions()
    assert len(names) > 30
    missing = [n for n in sorted(names) if not hasattr(dll, n)]
    assert not missing, missing


def test_binding_declares_exactly_the_header(libpath):
    from tensorgrad_b200._lib import SIGNATURES

    assert set(SIGNATURES) == header_functions()


def test_status_strings_without_a_gpu(libpath):
    dll = ctypes.CDLL(libpath)
    dll.tg_status_string.restype = ctypes.c_char_p
    assert dll.tg_status_string(0) == b"ok"
    assert dll.tg_status_string(4) == b"index out of range"
    assert dll.tg_version() >= 100


# ---------------------------------------------------------------------- host engine logic
def leaf(values, requires_grad=True):
    from tensorgrad_b200.tensor import Tensor

    t = Tensor._wrap(np.asarray(values, dtype=np.float64))
    t._requires_grad = requires_grad
    return t


def op(parents, data, vjp, name="op"):
    from tensorgrad_b200.autograd import Node
    from tensorgrad_b200.tensor import Tensor

    out = Tensor._wrap(np.asarray(data, dtype=np.float64))
    out._requires_grad = True
    out._node = Node(name, tuple(parents), vjp)
    return out


def test_engine_sums_fan_out_and_respects_need_mask():
    from tensorgrad_b200 import autograd

    a = leaf([2.0])
    c = leaf([5.0], requires_grad=False)
    seen_need = []

    def mul_vjp(g, need):
        seen_need.append(need)
        return (g * 5.0 if need[0] else None, g * 2.0 if need[1] else None)

    b = op([a, c], [10.0], mul_vjp, "mul")
    d = op([a, b], [12.0], lambda g, need: (g, g), "add")  # d = a + b: a is used twice
    autograd._run_backward((d,), (np.ones(1),), retain_graph=False, targets=None)
    np.testing.assert_allclose(a.grad.data, [6.0])  # 1 (direct) + 5 (through b)
    assert c.grad is None
    assert seen_need == [(True, False)]


def test_engine_freed_graph_error_and_shape_check():
    from tensorgrad_b200 import autograd

    a = leaf([1.0, 2.0])
    b = op([a], [1.0, 2.0], lambda g, need: (g,), "id")
    autograd._run_backward((b,), (np.ones(2),), retain_graph=False, targets=None)
    with pytest.raises(RuntimeError, match="backward through the graph a second time"):
        autograd._run_backward((b,), (np.ones(2),), retain_graph=False, targets=None)
    c = op([a], [1.0], lambda g, need: (np.ones(3),), "bad")
    with pytest.raises(RuntimeError, match="produced a gradient of shape"):
        autograd._run_backward((c,), (np.ones(1),), retain_graph=True, targets=None)


def test_engine_targets_prune_and_leave_grad_untouched():
    from tensorgrad_b200 import autograd

    a, z = leaf([3.0]), leaf([4.0])
    calls = []

    def vjp(g, need):
        calls.append(need)
        return (g * 2.0 if need[0] else None, g if need[1] else None)

    b = op([a, z], [6.0], vjp, "f")
    got = autograd._run_backward((b,), (np.ones(1),), retain_graph=True, targets=[a])
    np.testing.assert_allclose(got[id(a)], [2.0])
    assert a.grad is None and z.grad is None
    assert calls == [(True, False)]  # z does not lead to a target


def test_leaf_hook_fires_once_per_leaf_when_final():
    from tensorgrad_b200 import autograd

    a, w = leaf([1.0]), leaf([1.0])
    b = op([a, w], [1.0], lambda g, need: (g, g), "add")
    c = op([b, w], [1.0], lambda g, need: (g, g), "add")
    fired = []
    remove = autograd.add_leaf_hook(lambda t: fired.append((id(t), float(t.grad.data[0]))))
    try:
        autograd._run_backward((c,), (np.ones(1),), retain_graph=False, targets=None)
    finally:
        remove()
    assert sorted(fired) == sorted([(id(a), 1.0), (id(w), 2.0)])


def test_leaf_is_finalised_right_after_its_last_consumer():
    # y = f(h, w2), h = g(x, w1): w2's gradient is final once f's VJP ran, so its leaf hook
    # (data-parallel bucketing) fires before g's VJP, not at the end of the walk.
    from tensorgrad_b200 import autograd

    x, w1, w2 = leaf([1.0]), leaf([2.0]), leaf([3.0])
    events = []

    def g_vjp(g, need):
        events.append("vjp g")
        return (g, g)

    def f_vjp(g, need):
        events.append("vjp f")
        return (g, g)

    h = op([x, w1], [1.0], g_vjp, "g")
    y = op([h, w2], [1.0], f_vjp, "f")
    names = {id(x): "x", id(w1): "w1", id(w2): "w2"}
    remove = autograd.add_leaf_hook(lambda t: events.append("leaf " + names[id(t)]))
    try:
        autograd._run_backward((y,), (np.ones(1),), retain_graph=False, targets=None)
    finally:
        remove()
    assert events.index("leaf w2") < events.index("vjp g")
    assert sorted(e for e in events if e.startswith("leaf")) == ["leaf w1", "leaf w2", "leaf x"]
