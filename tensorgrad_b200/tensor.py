"""The device :class:`Tensor`, dtype defaults and tensor factories (tensor.py of the reference).

Same API as the reference's ``Tensor`` (tensor.py:71-477): ``requires_grad``, ``.grad``,
``backward()``, arithmetic operators, op methods and factories. ``data`` is a
:class:`~tensorgrad_b200.device.DeviceArray` in device memory instead of a host
``ndarray``; ``numpy()`` / ``np.asarray(t)`` return host copies.
"""

from __future__ import annotations

import operator
from collections.abc import Sequence
from typing import Any, Self

import numpy as np

from tensorgrad_b200 import autograd as _autograd
from tensorgrad_b200 import device as _device
from tensorgrad_b200._random import get_rng
from tensorgrad_b200.autograd import Node
from tensorgrad_b200.device import DeviceArray

__all__ = [
    "Tensor",
    "arange",
    "full",
    "get_default_dtype",
    "ones",
    "ones_like",
    "rand",
    "randn",
    "set_default_dtype",
    "tensor",
    "zeros",
    "zeros_like",
]


class _DTypeState:
    default: Any = np.float32


def set_default_dtype(dtype: Any) -> None:
    """Set the floating dtype for tensors built from Python floats (float32; float64 is the
    float64 build mode, where every kernel runs in double precision)."""
    if not np.issubdtype(dtype, np.floating):
        raise TypeError(f"default dtype must be a floating type, got {dtype}")
    _DTypeState.default = dtype


def get_default_dtype() -> Any:
    return _DTypeState.default


def _host_array(data: object, dtype: Any) -> np.ndarray:
    if isinstance(data, np.ndarray | np.generic):
        if (isinstance(data, np.ndarray) and (dtype is None or np.dtype(dtype) == data.dtype)
                and data.flags.c_contiguous and _device.is_pinned(data)):
            # Page-locked memory (device.pinned_empty) is uploaded by an asynchronous DMA
            # straight from the caller's buffer, which must stay unchanged until the next
            # synchronisation (the contract of pinned_empty).
            return data
        return np.array(data, dtype=dtype, copy=True)
    arr = np.asarray(data, dtype=dtype)
    if dtype is None and arr.dtype == np.float64:
        arr = arr.astype(get_default_dtype())
    return arr


def _to_device(data: object, dtype: Any) -> DeviceArray:
    if isinstance(data, Tensor):
        data = data.data
    if isinstance(data, DeviceArray):
        dt = data.dtype if dtype is None else np.dtype(dtype)
        return data.astype(dt, copy=True)
    arr = _host_array(data, dtype)
    if arr.dtype == np.int32 or arr.dtype == np.uint32:
        arr = arr.astype(np.int64)
    return _device.from_numpy(arr)


class Tensor:
    """An n-dimensional device array that records the ops applied to it for autodiff."""

    __slots__ = (
        "__weakref__", "_arena", "_grad", "_grad_slot", "_node", "_requires_grad", "_retains_grad",
        "_slot_taken", "data",
    )

    __array_ufunc__ = None

    data: DeviceArray

    def __init__(self, data: object, requires_grad: bool = False, dtype: Any = None) -> None:
        self.data = _to_device(data, dtype)
        self._grad: Tensor | None = None
        self._grad_slot: DeviceArray | None = None
        self._arena: Any = None
        self._node: Node | None = None
        self._retains_grad = False
        self._requires_grad = False
        self._slot_taken = False
        self.requires_grad = requires_grad

    @classmethod
    def _wrap(cls, data: DeviceArray) -> Tensor:
        out = Tensor.__new__(Tensor)
        out.data = data
        out._grad = None
        out._grad_slot = None
        out._arena = None
        out._node = None
        out._retains_grad = False
        out._requires_grad = False
        out._slot_taken = False
        return out

    # ------------------------------------------------------------------ properties
    @property
    def requires_grad(self) -> bool:
        return self._requires_grad

    @requires_grad.setter
    def requires_grad(self, value: bool) -> None:
        if self._node is not None:
            raise RuntimeError("requires_grad can only be changed on leaf tensors")
        if value and not np.issubdtype(self.data.dtype, np.floating):
            raise TypeError(
                f"only floating-point tensors can require gradients (got {self.data.dtype})"
            )
        self._requires_grad = bool(value)

    @property
    def grad(self) -> Tensor | None:
        if self._arena is not None and self._arena.pending_clip is not None:
            self._arena.settle_clip()
        return self._grad

    @grad.setter
    def grad(self, value: Any) -> None:
        if self._arena is not None and self._arena.pending_clip is not None:
            self._arena.settle_clip()
        if value is not None:
            if isinstance(value, DeviceArray):
                value = Tensor._wrap(value)
            elif not isinstance(value, Tensor):
                value = Tensor._wrap(_device.from_numpy(np.asarray(value)))
            if value.shape != self.shape:
                raise ValueError(f"grad has shape {value.shape}, expected {self.shape}")
        self._grad = value

    @property
    def shape(self) -> tuple[int, ...]:
        return self.data.shape

    @property
    def ndim(self) -> int:
        return self.data.ndim

    @property
    def size(self) -> int:
        return self.data.size

    @property
    def dtype(self) -> np.dtype[Any]:
        return self.data.dtype

    @property
    def is_leaf(self) -> bool:
        return self._node is None

    @property
    def grad_fn(self) -> Node | None:
        return self._node

    @property
    def T(self) -> Tensor:  # noqa: N802
        return _shape.permute(self, tuple(reversed(range(self.ndim))))

    # ------------------------------------------------------------------ autograd
    def backward(
        self, grad: Any = None, retain_graph: bool | None = None, create_graph: bool = False
    ) -> None:
        """Backpropagate from this tensor, accumulating into the leaves' ``.grad``."""
        if grad is None and not create_graph and self._requires_grad and self.data.size == 1:
            seed = _device.from_numpy(np.ones(self.shape, dtype=self.dtype))
            _autograd._run_backward((self,), (seed,), retain_graph=bool(retain_graph),
                                    targets=None)
            return
        _autograd.backward(self, grad, retain_graph=retain_graph, create_graph=create_graph)

    def _grad_target(self) -> DeviceArray | None:
        """This leaf's arena slot, for a VJP to write the leaf's gradient into directly: only
        while the slot holds no gradient of this pass (``.grad`` is None), no other VJP has
        taken it, and no clip factor is pending on the arena. The VJP writes the whole slot;
        ``_accumulate_grad`` then finds the gradient in place and copies nothing."""
        slot = self._grad_slot
        if slot is None or self._grad is not None or self._slot_taken:
            return None
        if self._arena is not None and self._arena.pending_clip is not None:
            return None
        self._slot_taken = True
        return slot

    def _accumulate_grad(self, g: DeviceArray) -> None:
        self._slot_taken = False
        if g.dtype != self.dtype:
            g = g.astype(self.dtype)
        slot = self._grad_slot
        if slot is not None:
            # The gradient lives in a flat arena (optimizer / data-parallel bucket).
            if self._arena is not None and self._arena.pending_clip is not None:
                self._arena.settle_clip()
            from tensorgrad_b200.ops.elementwise import binary_array

            cur = self._grad
            if cur is None:
                if not (g._buf is slot._buf and g._off == slot._off):
                    _device.copy_into(slot, g)
            elif cur.data is slot:
                binary_array(slot, g, 0, out=slot)
            else:
                binary_array(cur.data, g, 0, out=slot)
            if cur is None or cur.data is not slot:
                self._grad = Tensor._wrap(slot)
            return
        # Copy on first write: ``g`` may alias another gradient (add's VJP returns g twice).
        total = g.copy() if self._grad is None else self._grad.data + g
        self._grad = Tensor._wrap(total)

    def retain_grad(self) -> None:
        if not self.requires_grad:
            raise RuntimeError("cannot retain_grad() on a tensor that does not require grad")
        if self._node is not None:
            self._retains_grad = True

    def zero_grad(self) -> None:
        self._grad = None
        self._slot_taken = False

    def detach(self) -> Tensor:
        return Tensor._wrap(self.data)

    def requires_grad_(self, requires_grad: bool = True) -> Self:
        self.requires_grad = requires_grad
        return self

    # ------------------------------------------------------------------ conversion
    def numpy(self, out: np.ndarray | None = None) -> np.ndarray:
        """A host copy of the data (into ``out`` when given, e.g. a page-locked buffer from
        ``device.pinned_empty``, which the copy engine fills at full bus speed)."""
        return self.data.numpy(out)

    def __array__(self, dtype: Any = None, copy: bool | None = None) -> np.ndarray:
        # Always a host copy of device data; a dtype change refused with copy=False, as the
        # reference refuses it.
        if copy is False and dtype is not None and np.dtype(dtype) != self.dtype:
            raise ValueError(f"cannot convert {self.dtype} to {np.dtype(dtype)} without a copy")
        arr = self.data.numpy()
        return arr if dtype is None else arr.astype(dtype)

    def item(self) -> Any:
        return self.data.item()

    def tolist(self) -> Any:
        return self.data.tolist()

    def astype(self, dtype: Any) -> Tensor:
        return _elementwise.astype(self, dtype)

    def __len__(self) -> int:
        if self.ndim == 0:
            raise TypeError("len() of a 0-d tensor")
        return self.shape[0]

    def __bool__(self) -> bool:
        return bool(self.numpy())

    def __float__(self) -> float:
        return float(self.item())

    def __int__(self) -> int:
        return int(self.item())

    def __repr__(self) -> str:
        body = np.array2string(self.numpy(), separator=", ", prefix="Tensor(", precision=4)
        extras = []
        if self.dtype != get_default_dtype():
            extras.append(f"dtype={self.dtype}")
        if self._node is not None:
            extras.append(f"grad_fn=<{self._node.op}>")
        elif self.requires_grad:
            extras.append("requires_grad=True")
        return f"Tensor({body}{''.join(', ' + e for e in extras)})"

    # ------------------------------------------------------------------ arithmetic
    def __add__(self, other: Any) -> Tensor:
        return _elementwise.add(self, other)

    def __radd__(self, other: Any) -> Tensor:
        return _elementwise.add(other, self)

    def __sub__(self, other: Any) -> Tensor:
        return _elementwise.sub(self, other)

    def __rsub__(self, other: Any) -> Tensor:
        return _elementwise.sub(other, self)

    def __mul__(self, other: Any) -> Tensor:
        return _elementwise.mul(self, other)

    def __rmul__(self, other: Any) -> Tensor:
        return _elementwise.mul(other, self)

    def __truediv__(self, other: Any) -> Tensor:
        return _elementwise.div(self, other)

    def __rtruediv__(self, other: Any) -> Tensor:
        return _elementwise.div(other, self)

    def __pow__(self, exponent: Any) -> Tensor:
        return _elementwise.pow(self, exponent)

    def __rpow__(self, base: Any) -> Tensor:
        return _elementwise.pow(base, self)

    def __neg__(self) -> Tensor:
        return _elementwise.neg(self)

    def __matmul__(self, other: Any) -> Tensor:
        return _linalg.matmul(self, other)

    def __rmatmul__(self, other: Any) -> Tensor:
        return _linalg.matmul(other, self)

    def __getitem__(self, index: Any) -> Tensor:
        return _shape.getitem(self, index)

    __hash__ = object.__hash__

    def _cmp(self, other: object, op: str) -> Tensor:
        """An elementwise comparison on the device, as a boolean tensor (no graph)."""
        from tensorgrad_b200.ops import compare as _compare

        return _compare.compare(self, other, op)

    def __eq__(self, other: object) -> Tensor:  # type: ignore[override]
        return self._cmp(other, "eq")

    def __ne__(self, other: object) -> Tensor:  # type: ignore[override]
        return self._cmp(other, "ne")

    def __lt__(self, other: object) -> Tensor:
        return self._cmp(other, "lt")

    def __le__(self, other: object) -> Tensor:
        return self._cmp(other, "le")

    def __gt__(self, other: object) -> Tensor:
        return self._cmp(other, "gt")

    def __ge__(self, other: object) -> Tensor:
        return self._cmp(other, "ge")

    # ------------------------------------------------------------------ op methods
    def matmul(self, other: Any) -> Tensor:
        return _linalg.matmul(self, other)

    def exp(self) -> Tensor:
        return _elementwise.exp(self)

    def log(self) -> Tensor:
        return _elementwise.log(self)

    def sqrt(self) -> Tensor:
        return _elementwise.sqrt(self)

    def tanh(self) -> Tensor:
        return _elementwise.tanh(self)

    def sigmoid(self) -> Tensor:
        return _elementwise.sigmoid(self)

    def relu(self) -> Tensor:
        return _elementwise.relu(self)

    def gelu(self) -> Tensor:
        return _elementwise.gelu(self)

    def sum(self, axis: Any = None, keepdims: bool = False) -> Tensor:
        return _reduce.sum(self, axis, keepdims)

    def mean(self, axis: Any = None, keepdims: bool = False) -> Tensor:
        return _reduce.mean(self, axis, keepdims)

    def var(self, axis: Any = None, keepdims: bool = False, correction: int = 1) -> Tensor:
        return _reduce.var(self, axis, keepdims, correction)

    def max(self, axis: Any = None, keepdims: bool = False) -> Tensor:
        """Maximum over ``axis``; tied maxima share the gradient equally."""
        return _reduce.max(self, axis, keepdims)

    def min(self, axis: Any = None, keepdims: bool = False) -> Tensor:
        """Minimum over ``axis``; tied minima share the gradient equally."""
        return _reduce.min(self, axis, keepdims)

    def all(self, axis: Any = None, keepdims: bool = False) -> Tensor:
        """Whether every element along ``axis`` is nonzero (a boolean tensor, no graph)."""
        from tensorgrad_b200.ops import compare as _compare

        return _compare.truth(self, axis, keepdims, True)

    def any(self, axis: Any = None, keepdims: bool = False) -> Tensor:
        """Whether some element along ``axis`` is nonzero (a boolean tensor, no graph)."""
        from tensorgrad_b200.ops import compare as _compare

        return _compare.truth(self, axis, keepdims, False)

    def argmax(self, axis: int | None = None, keepdims: bool = False) -> Tensor:
        """Indices of the first maxima along ``axis`` (int64, no graph)."""
        from tensorgrad_b200.ops import compare as _compare

        return _compare.argmax(self, axis, keepdims)

    def softmax(self, axis: int = -1) -> Tensor:
        """Numerically stable softmax along ``axis``."""
        from tensorgrad_b200.ops import activation as _activation

        return _activation.softmax(self, axis)

    def log_softmax(self, axis: int = -1) -> Tensor:
        """Numerically stable log-softmax along ``axis``."""
        from tensorgrad_b200.ops import activation as _activation

        return _activation.log_softmax(self, axis)

    def masked_fill(self, mask: Any, value: float) -> Tensor:
        """Replace entries where ``mask`` holds by ``value`` (no gradient flows there)."""
        return _shape.masked_fill(self, mask, value)

    def reshape(self, *shape: int | Sequence[int]) -> Tensor:
        dims: Sequence[object] = (
            shape[0] if len(shape) == 1 and isinstance(shape[0], Sequence) else shape
        )
        return _shape.reshape(self, tuple(operator.index(d) for d in dims))  # type: ignore[arg-type]

    def transpose(self, axis0: int, axis1: int) -> Tensor:
        return _shape.transpose(self, axis0, axis1)

    def permute(self, *dims: int) -> Tensor:
        return _shape.permute(self, dims)

    def flatten(self, start_axis: int = 0, end_axis: int = -1) -> Tensor:
        return _shape.flatten(self, start_axis, end_axis)

    def unsqueeze(self, axis: int) -> Tensor:
        return _shape.unsqueeze(self, axis)

    def squeeze(self, axis: int | None = None) -> Tensor:
        return _shape.squeeze(self, axis)


# ---------------------------------------------------------------------- factories
def tensor(data: object, requires_grad: bool = False, dtype: Any = None) -> Tensor:
    return Tensor(data, requires_grad=requires_grad, dtype=dtype)


def _shape_tuple(shape: Any) -> tuple[int, ...]:
    return (shape,) if isinstance(shape, int) else tuple(int(s) for s in shape)


def _float_dtype(dtype: Any) -> Any:
    return get_default_dtype() if dtype is None else dtype


def zeros(shape: Any, *, dtype: Any = None, requires_grad: bool = False) -> Tensor:
    out = Tensor._wrap(_device.zeros(_shape_tuple(shape), _float_dtype(dtype)))
    out.requires_grad = requires_grad
    return out


def ones(shape: Any, *, dtype: Any = None, requires_grad: bool = False) -> Tensor:
    return full(shape, 1.0, dtype=dtype, requires_grad=requires_grad)


def full(shape: Any, fill_value: float, *, dtype: Any = None, requires_grad: bool = False) -> Tensor:
    arr = _device.empty(_shape_tuple(shape), _float_dtype(dtype))
    arr.fill_(fill_value)
    out = Tensor._wrap(arr)
    out.requires_grad = requires_grad
    return out


def zeros_like(t: Tensor, *, requires_grad: bool = False) -> Tensor:
    return zeros(t.shape, dtype=t.dtype, requires_grad=requires_grad)


def ones_like(t: Tensor, *, requires_grad: bool = False) -> Tensor:
    return ones(t.shape, dtype=t.dtype, requires_grad=requires_grad)


def arange(start: float, stop: float | None = None, step: float = 1) -> Tensor:
    values = np.arange(start) if stop is None else np.arange(start, stop, step)
    return Tensor._wrap(_device.from_numpy(values))


def randn(shape: Any, *, dtype: Any = None, requires_grad: bool = False) -> Tensor:
    data = get_rng().standard_normal(_shape_tuple(shape)).astype(_float_dtype(dtype))
    return Tensor(data, requires_grad=requires_grad)


def rand(shape: Any, *, dtype: Any = None, requires_grad: bool = False) -> Tensor:
    data = get_rng().random(_shape_tuple(shape)).astype(_float_dtype(dtype))
    return Tensor(data, requires_grad=requires_grad)


# Op modules import ``Tensor`` from here, so they are bound after the class exists.
from tensorgrad_b200.ops import elementwise as _elementwise  # noqa: E402
from tensorgrad_b200.ops import linalg as _linalg  # noqa: E402
from tensorgrad_b200.ops import reduce as _reduce  # noqa: E402
from tensorgrad_b200.ops import shape as _shape  # noqa: E402
