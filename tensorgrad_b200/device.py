"""Device-resident storage: :class:`DeviceArray`, the ``data`` of every tensor.

Memory comes from PyTorch's CUDA caching allocator (allocation only: buffers are reused
across steps without ``cudaMalloc``); every byte that moves or changes does so through
``libtgb200.so``. A :class:`DeviceArray` is contiguous, row-major, and duck-types the parts
of ``numpy.ndarray`` that user code reads from ``tensor.data`` (``shape``, ``dtype``,
``np.asarray(a)``, ``a.item()``, indexing for inspection, whole-array assignment).
"""

from __future__ import annotations

import math
import os
from collections.abc import Sequence
from typing import Any

import numpy as np

from tensorgrad_b200._lib import ADD, DIV, F32, F64, MUL, SUB, check, int64_array, lib

try:  # torch is the allocator and the NCCL plumbing only
    import torch
except ImportError as exc:  # pragma: no cover - torch is part of the image
    raise RuntimeError("tensorgrad_b200 allocates device memory through torch") from exc

_TORCH_DTYPES = {
    np.dtype(np.float32): torch.float32,
    np.dtype(np.float64): torch.float64,
    np.dtype(np.int64): torch.int64,
    np.dtype(np.int32): torch.int32,
    np.dtype(np.bool_): torch.bool,
    np.dtype(np.uint8): torch.uint8,
}


class _State:
    device: torch.device | None = None
    stream: int = 0  # the legacy default stream, which torch also uses by default


def set_device(index: int) -> None:
    """Select the CUDA device for new tensors (one process per GPU)."""
    torch.cuda.set_device(index)
    _State.device = torch.device("cuda", index)


def current_device() -> torch.device:
    dev = _State.device
    if dev is None:
        if not torch.cuda.is_available():
            raise RuntimeError(
                "tensorgrad_b200 needs a CUDA device (B200): tensors live in device memory "
                "and there is no CPU fallback"
            )
        index = int(os.environ.get("LOCAL_RANK", torch.cuda.current_device()))
        set_device(index)
        dev = _State.device
    assert dev is not None
    return dev


def stream() -> int:
    """The CUDA stream every kernel is launched on."""
    return _State.stream


def dtype_code(dtype: np.dtype[Any]) -> int:
    if dtype == np.float32:
        return F32
    if dtype == np.float64:
        return F64
    raise TypeError(f"no device kernels for dtype {dtype}")


def synchronize() -> None:
    """Wait for the stream; then raise any error that the device recorded: a bounded wait of
    a tensor-core kernel that ran out (its outputs are then incomplete), or an index that
    device-side validation rejected."""
    check(lib.tg_stream_synchronize(_State.stream), "synchronize")
    _raise_kernel_timeouts()
    if _Async.pending:
        _raise_async_errors()


def _raise_kernel_timeouts() -> None:
    """The tensor-core GEMM and the fused attention kernels give up a pipeline wait after a
    cycle budget (about two seconds) instead of hanging; they then record TG_ERR_TIMEOUT in
    a device status word, drain and return without finishing their outputs. Both words are
    read (and cleared) at every host synchronisation, so such a step raises here."""
    failed = [name for name, fn in (("tensor-core GEMM", lib.tg_gemm_tc_status),
                                    ("fused attention", lib.tg_attention_tc_status))
              if fn(1) != 0]
    if failed:
        raise RuntimeError(f"{' and '.join(failed)}: a bounded device-side wait ran out "
                           "(TG_ERR_TIMEOUT); the outputs of the kernels since the last "
                           "synchronisation are incomplete")


# Device-side validation. Ops that take device-resident indices (embedding ids, class
# targets) cannot check them on the host without a synchronisation per call, so their
# kernels check them and set a flag word instead; the flags are read back at the next host
# synchronisation, which raises the error the op raises for host inputs.
ASYNC_EMBEDDING_ID = 0
ASYNC_CLASS_TARGET = 1
_ASYNC_MESSAGES = {
    ASYNC_EMBEDDING_ID: "embedding ids out of range (device-resident ids, checked on the device)",
    ASYNC_CLASS_TARGET: "cross_entropy target out of range (device-resident targets, checked on "
                        "the device)",
}


class _Async:
    words: DeviceArray | None = None
    pending = False


def async_error_word(kind: int) -> int:
    """Device address of the int32 flag word of ``kind`` (ASYNC_*); marks a check pending."""
    if _Async.words is None or _Async.words._t.device != current_device():
        _Async.words = zeros((len(_ASYNC_MESSAGES),), np.int32)
    _Async.pending = True
    return _Async.words.ptr + 4 * kind


def _raise_async_errors() -> None:
    _Async.pending = False
    words = _Async.words
    if words is None:
        return
    host = np.zeros(words.shape, np.int32)
    check(lib.tg_memcpy_d2h(host.ctypes.data, words.ptr, host.nbytes, _State.stream), "d2h")
    check(lib.tg_stream_synchronize(_State.stream), "synchronize")
    if host.any():
        check(lib.tg_memset_zero(words.ptr, words.nbytes, _State.stream), "zeros")
        kind = int(np.flatnonzero(host)[0])
        raise IndexError(_ASYNC_MESSAGES[kind])


class DeviceArray:
    """A contiguous device buffer with a shape and a NumPy dtype."""

    __slots__ = ("_t", "dtype", "shape")

    __array_ufunc__ = None  # ``ndarray op DeviceArray`` defers to our operators

    def __init__(self, t: torch.Tensor, shape: tuple[int, ...], dtype: np.dtype[Any]) -> None:
        self._t = t
        self.shape = shape
        self.dtype = dtype

    # ------------------------------------------------------------- properties
    @property
    def ptr(self) -> int:
        return self._t.data_ptr()

    @property
    def size(self) -> int:
        return math.prod(self.shape)

    @property
    def ndim(self) -> int:
        return len(self.shape)

    @property
    def itemsize(self) -> int:
        return self.dtype.itemsize

    @property
    def nbytes(self) -> int:
        return self.size * self.dtype.itemsize

    @property
    def T(self) -> DeviceArray:  # noqa: N802
        from tensorgrad_b200.ops import shape as _shape_ops

        return _shape_ops.permute_array(self, tuple(reversed(range(self.ndim))))

    # ------------------------------------------------------------- host transfer
    def numpy(self, out: np.ndarray | None = None) -> np.ndarray:
        """A host copy (synchronises the stream), into ``out`` when given (a C-contiguous
        array of this shape and dtype; page-locked memory is copied at full bus speed)."""
        if out is None:
            out = np.empty(self.shape, dtype=self.dtype)
        elif (out.shape != tuple(self.shape) or out.dtype != self.dtype
              or not out.flags.c_contiguous):
            raise ValueError(f"numpy(out=...) needs a C-contiguous {self.dtype} array of shape "
                             f"{tuple(self.shape)}, got {out.dtype} {out.shape}")
        if out.nbytes:
            check(lib.tg_memcpy_d2h(out.ctypes.data, self.ptr, out.nbytes, _State.stream), "d2h")
            synchronize()
        return out

    def __array__(self, dtype: Any = None, copy: bool | None = None) -> np.ndarray:
        arr = self.numpy()
        return arr if dtype is None else arr.astype(dtype)

    def item(self) -> Any:
        if self.size != 1:
            raise ValueError("can only convert an array of size 1 to a Python scalar")
        return self.numpy().item()

    def tolist(self) -> Any:
        return self.numpy().tolist()

    def __float__(self) -> float:
        return float(self.item())

    def __len__(self) -> int:
        if not self.shape:
            raise TypeError("len() of a 0-d array")
        return self.shape[0]

    def __repr__(self) -> str:
        return f"DeviceArray({self.numpy()!r}, device={self._t.device})"

    def __getitem__(self, index: Any) -> Any:
        return self.numpy()[index]

    def __setitem__(self, index: Any, value: Any) -> None:
        if index is not Ellipsis and index != slice(None):
            raise NotImplementedError("only whole-array assignment (a[...] = v) is supported")
        if isinstance(value, DeviceArray):
            if value.shape != self.shape and value.size != 1:
                value_np = np.broadcast_to(value.numpy(), self.shape)
                upload_into(self, np.ascontiguousarray(value_np, dtype=self.dtype))
                return
            if value.size == self.size and value.dtype == self.dtype:
                copy_into(self, value)
                return
            value = value.numpy()
        arr = np.broadcast_to(np.asarray(value, dtype=self.dtype), self.shape)
        upload_into(self, np.ascontiguousarray(arr))

    # ------------------------------------------------------------- views and copies
    def reshape(self, *shape: int | Sequence[int]) -> DeviceArray:
        dims = shape[0] if len(shape) == 1 and isinstance(shape[0], Sequence) else shape
        new = _resolve_shape(tuple(int(d) for d in dims), self.size)  # type: ignore[union-attr]
        return DeviceArray(self._t, new, self.dtype)

    def flat_view(self, offset: int, count: int, shape: tuple[int, ...] | None = None) -> DeviceArray:
        """A view of ``count`` elements starting at element ``offset`` of this buffer."""
        t = self._t.view(-1)[offset:offset + count]
        return DeviceArray(t, shape if shape is not None else (count,), self.dtype)

    def copy(self) -> DeviceArray:
        out = empty(self.shape, self.dtype)
        copy_into(out, self)
        return out

    def astype(self, dtype: Any, copy: bool = True) -> DeviceArray:
        dt = np.dtype(dtype)
        if dt == self.dtype:
            return self.copy() if copy else self
        from tensorgrad_b200.ops.elementwise import cast_array

        return cast_array(self, dt)

    # ------------------------------------------------------------- arithmetic (engine sums)
    def _binary(self, other: Any, op: int, reverse: bool = False) -> DeviceArray:
        from tensorgrad_b200.ops.elementwise import binary_array

        o = other if isinstance(other, DeviceArray) else scalar_like(other, self.dtype)
        return binary_array(o, self, op) if reverse else binary_array(self, o, op)

    def __add__(self, other: Any) -> DeviceArray:
        return self._binary(other, ADD)

    def __radd__(self, other: Any) -> DeviceArray:
        return self._binary(other, ADD, True)

    def __sub__(self, other: Any) -> DeviceArray:
        return self._binary(other, SUB)

    def __rsub__(self, other: Any) -> DeviceArray:
        return self._binary(other, SUB, True)

    def __mul__(self, other: Any) -> DeviceArray:
        return self._binary(other, MUL)

    def __rmul__(self, other: Any) -> DeviceArray:
        return self._binary(other, MUL, True)

    def __truediv__(self, other: Any) -> DeviceArray:
        return self._binary(other, DIV)

    def __neg__(self) -> DeviceArray:
        return self._binary(-1.0, MUL)

    def __iadd__(self, other: Any) -> DeviceArray:
        from tensorgrad_b200.ops.elementwise import binary_array

        o = other if isinstance(other, DeviceArray) else scalar_like(other, self.dtype)
        binary_array(self, o, ADD, out=self)
        return self

    def __imul__(self, other: Any) -> DeviceArray:
        from tensorgrad_b200.ops.elementwise import binary_array

        o = other if isinstance(other, DeviceArray) else scalar_like(other, self.dtype)
        binary_array(self, o, MUL, out=self)
        return self

    def __isub__(self, other: Any) -> DeviceArray:
        from tensorgrad_b200.ops.elementwise import binary_array

        o = other if isinstance(other, DeviceArray) else scalar_like(other, self.dtype)
        binary_array(self, o, SUB, out=self)
        return self

    def fill_(self, value: float) -> DeviceArray:
        if value == 0:
            check(lib.tg_memset_zero(self.ptr, self.nbytes, _State.stream), "fill")
        else:
            upload_into(self, np.full(self.shape, value, dtype=self.dtype))
        return self


# ---------------------------------------------------------------------- factories
def _resolve_shape(shape: tuple[int, ...], size: int) -> tuple[int, ...]:
    if shape.count(-1) > 1:
        raise ValueError("can only specify one unknown dimension")
    if -1 in shape:
        known = math.prod(d for d in shape if d != -1)
        if known == 0 or size % known:
            raise ValueError(f"cannot reshape array of size {size} into shape {shape}")
        shape = tuple(size // known if d == -1 else d for d in shape)
    if math.prod(shape) != size:
        raise ValueError(f"cannot reshape array of size {size} into shape {shape}")
    return shape


def empty(shape: Sequence[int], dtype: Any) -> DeviceArray:
    dt = np.dtype(dtype)
    shp = tuple(int(s) for s in shape)
    t = torch.empty(max(math.prod(shp), 1), dtype=_TORCH_DTYPES[dt], device=current_device())
    return DeviceArray(t, shp, dt)


def zeros(shape: Sequence[int], dtype: Any) -> DeviceArray:
    out = empty(shape, dtype)
    if out.nbytes:
        check(lib.tg_memset_zero(out.ptr, out.nbytes, _State.stream), "zeros")
    return out


class _Staging:
    """Page-locked staging blocks for small uploads from pageable host arrays.

    A block is reused only after the CUDA event recorded behind its copy has completed, so
    an upload never waits for the device queue (no stream synchronisation on the hot path).
    """

    LIMIT = 4 << 20  # larger uploads (model initialisation) copy synchronously

    def __init__(self) -> None:
        self.blocks: list[list[Any]] = []  # [pinned tensor, capacity, event or None]

    def upload(self, dst: DeviceArray, arr: np.ndarray) -> None:
        block = None
        for b in self.blocks:
            if b[1] >= arr.nbytes and (b[2] is None or b[2].query()):
                block = b
                break
        if block is None:
            cap = max(1 << 16, 1 << (arr.nbytes - 1).bit_length())
            block = [torch.empty(cap, dtype=torch.uint8, pin_memory=True), cap, None]
            self.blocks.append(block)
        host = block[0].numpy()[: arr.nbytes]
        host[:] = arr.reshape(-1).view(np.uint8)
        check(lib.tg_memcpy_h2d(dst.ptr, host.ctypes.data, arr.nbytes, _State.stream), "h2d")
        ev = block[2] or torch.cuda.Event()
        ev.record(torch.cuda.current_stream(dst._t.device))
        block[2] = ev


_STAGING = _Staging()


def upload_into(dst: DeviceArray, arr: np.ndarray) -> None:
    arr = np.ascontiguousarray(arr, dtype=dst.dtype)
    if not arr.nbytes:
        return
    if _is_pinned(arr):
        check(lib.tg_memcpy_h2d(dst.ptr, arr.ctypes.data, arr.nbytes, _State.stream), "h2d")
    elif arr.nbytes <= _Staging.LIMIT:
        _STAGING.upload(dst, arr)
    else:
        check(lib.tg_memcpy_h2d(dst.ptr, arr.ctypes.data, arr.nbytes, _State.stream), "h2d")
        synchronize()  # keep ``arr`` alive until the driver has read it


_PINNED: list[tuple[int, int, Any]] = []


def pinned_empty(shape: Sequence[int], dtype: Any) -> np.ndarray:
    """A host array in page-locked memory: uploads from it (``from_numpy``, ``Tensor(...)``)
    are asynchronous DMA copies that read it after the call returns, so it must not be
    changed before the next synchronisation."""
    dt = np.dtype(dtype)
    t = torch.empty(max(math.prod(shape), 1), dtype=_TORCH_DTYPES[dt], pin_memory=True)
    arr = t.numpy()[: math.prod(shape)].reshape(shape)
    _PINNED.append((arr.ctypes.data, arr.nbytes, t))
    return arr


def _is_pinned(arr: np.ndarray) -> bool:
    p = arr.ctypes.data
    return any(base <= p and p + arr.nbytes <= base + n for base, n, _ in _PINNED)


def is_pinned(arr: np.ndarray) -> bool:
    """Whether ``arr`` lies in page-locked memory from ``pinned_empty``."""
    return _is_pinned(arr)


def from_numpy(arr: np.ndarray, dtype: Any = None) -> DeviceArray:
    a = np.ascontiguousarray(arr, dtype=dtype)
    out = empty(a.shape, a.dtype)
    upload_into(out, a)
    return out


def copy_into(dst: DeviceArray, src: DeviceArray) -> None:
    if dst.nbytes != src.nbytes:
        raise ValueError(f"copy of {src.nbytes} bytes into {dst.nbytes}")
    if src.nbytes:
        check(lib.tg_memcpy_d2d(dst.ptr, src.ptr, src.nbytes, _State.stream), "d2d")


def numpy_many(arrays: Sequence[DeviceArray]) -> list[np.ndarray]:
    """Host copies of several device arrays with one synchronisation: every copy is queued
    into one page-locked staging block (16-byte aligned slots), then the stream is waited on
    once and the slots are unpacked into ordinary arrays."""
    offsets, total = [], 0
    for a in arrays:
        offsets.append(total)
        total += -(-a.nbytes // 16) * 16
    if not arrays:
        return []
    staging = torch.empty(max(total, 16), dtype=torch.uint8, pin_memory=True).numpy()
    base = staging.ctypes.data
    for a, off in zip(arrays, offsets, strict=True):
        if a.nbytes:
            check(lib.tg_memcpy_d2h(base + off, a.ptr, a.nbytes, _State.stream), "d2h")
    synchronize()
    return [staging[off:off + a.nbytes].view(a.dtype).reshape(a.shape).copy()
            for a, off in zip(arrays, offsets, strict=True)]


def scalar_like(value: Any, dtype: np.dtype[Any]) -> DeviceArray:
    return from_numpy(np.asarray(value, dtype=dtype))


def scratch(nbytes: int) -> DeviceArray:
    """A temporary byte buffer (at least 16 bytes, 256-byte aligned by the allocator)."""
    return empty((max(int(nbytes), 16),), np.uint8)


def contiguous_strides(shape: Sequence[int]) -> list[int]:
    strides = [1] * len(shape)
    for i in range(len(shape) - 2, -1, -1):
        strides[i] = strides[i + 1] * shape[i + 1]
    return strides


def shape_args(shape: Sequence[int]):  # noqa: ANN201
    return int64_array(shape)
