"""Device-resident storage: :class:`DeviceArray`, the ``data`` of every tensor.

Memory comes from ``libtgb200.so``'s stream-ordered allocator (``tg_malloc`` / ``tg_free``:
each device's pool keeps freed blocks, so a step's buffers are reused without ``cudaMalloc``)
and page-locked host memory from ``tg_host_alloc``; every byte that moves or changes does so
through the library. No framework is imported. A :class:`DeviceArray` is a contiguous,
row-major view of a :class:`_Block` (several arrays may share one block, e.g. the slots of a
flat parameter arena), and duck-types the parts of ``numpy.ndarray`` that user code reads from
``tensor.data`` (``shape``, ``dtype``, ``np.asarray(a)``, ``a.item()``, indexing for
inspection, assignment to the whole array or to an indexed part).
"""

from __future__ import annotations

import ctypes
import math
import os
from collections.abc import Sequence
from typing import Any

import numpy as np

from tensorgrad_b200._lib import ADD, DIV, F32, F64, MUL, SUB, check, int64_array, lib


class _State:
    device: int | None = None
    stream: int = 0  # the legacy default stream (what other CUDA libraries use by default)


def set_device(index: int) -> None:
    """Select the CUDA device for new tensors (one process per GPU)."""
    check(lib.tg_set_device(int(index)), "set_device")
    _State.device = int(index)


def device_count() -> int:
    n = ctypes.c_int(0)
    lib.tg_device_count(ctypes.byref(n))
    return n.value


def current_device() -> int:
    """Index of the device new tensors go to (``LOCAL_RANK`` by default, else 0)."""
    dev = _State.device
    if dev is None:
        if device_count() == 0:
            raise RuntimeError(
                "tensorgrad_b200 needs a CUDA device (B200): tensors live in device memory "
                "and there is no CPU fallback"
            )
        set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dev = _State.device
    assert dev is not None
    return dev


class _Block:
    """One device allocation; freed (stream-ordered) when the last array viewing it goes."""

    __slots__ = ("__weakref__", "device", "nbytes", "ptr")

    def __init__(self, nbytes: int) -> None:
        self.device = current_device()
        self.nbytes = nbytes
        p = ctypes.c_void_p()
        check(lib.tg_malloc(ctypes.byref(p), nbytes, _State.stream), "device allocation")
        self.ptr = int(p.value or 0)

    def __del__(self) -> None:
        if self.ptr:
            try:
                lib.tg_free(self.ptr, _State.stream)
            except Exception:  # noqa: BLE001 - interpreter shutdown: the process frees all
                pass
            self.ptr = 0


def stream() -> int:
    """The CUDA stream every kernel is launched on."""
    return _State.stream


def memory_stats(reset_peak: bool = False) -> dict[str, int]:
    """Bytes of the current device's memory pool: ``reserved`` (held by the pool), ``used``
    (in live buffers) and ``peak`` (the most in use at once since the last reset; with
    ``reset_peak`` the mark starts again from now). Frees are stream-ordered, so synchronize
    first for figures that include everything already released."""
    dev = current_device()
    reserved, used, peak = ctypes.c_uint64(0), ctypes.c_uint64(0), ctypes.c_uint64(0)
    check(lib.tg_pool_stats(dev, ctypes.byref(reserved), ctypes.byref(used)), "memory_stats")
    check(lib.tg_pool_peak(dev, int(reset_peak), ctypes.byref(peak)), "memory_stats")
    return {"reserved": reserved.value, "used": used.value, "peak": peak.value}


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
    if _Async.words is None or _Async.words._buf.device != current_device():
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
    """A contiguous device array: ``shape`` elements of ``dtype`` at byte ``_off`` of a
    device allocation."""

    __slots__ = ("_buf", "_off", "dtype", "shape")

    __array_ufunc__ = None  # ``ndarray op DeviceArray`` defers to our operators

    def __init__(self, buf: _Block, off: int, shape: tuple[int, ...],
                 dtype: np.dtype[Any]) -> None:
        self._buf = buf
        self._off = off
        self.shape = shape
        self.dtype = dtype

    # ------------------------------------------------------------- properties
    @property
    def ptr(self) -> int:
        return self._buf.ptr + self._off

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

    def __getattr__(self, name: str) -> Any:
        """NumPy's other array methods and attributes (``mean``, ``argmax``, ``std``,
        ``astype(...).sum()`` ...) for code that inspects ``tensor.data`` as the reference's
        NumPy arrays allow: taken from a host copy, so they read the values and never change
        the device array (and cost a device-to-host copy per use)."""
        if name.startswith("_") or not hasattr(np.ndarray, name):
            raise AttributeError(f"'DeviceArray' object has no attribute '{name}'")
        return getattr(self.numpy(), name)

    def __float__(self) -> float:
        return float(self.item())

    def __len__(self) -> int:
        if not self.shape:
            raise TypeError("len() of a 0-d array")
        return self.shape[0]

    def __repr__(self) -> str:
        return f"DeviceArray({self.numpy()!r}, device=cuda:{self._buf.device})"

    def __getitem__(self, index: Any) -> Any:
        return self.numpy()[index]

    def __setitem__(self, index: Any, value: Any) -> None:
        whole = index is Ellipsis or (isinstance(index, slice) and index == slice(None))
        if not whole:
            self._assign_part(index, value)
            return
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

    def _assign_part(self, index: Any, value: Any) -> None:
        """``a[index] = value``. Basic indexing (ints, slices, ``...``, ``None``) writes the
        selected strided view on the device with one strided copy of ``value`` broadcast to
        it; integer or boolean array indices go through a host copy of the array (an
        interactive edit, not a training-step path)."""
        from tensorgrad_b200.ops.shape import _basic_view, broadcast_array, strided_copy

        try:
            offset, shape, strides = _basic_view(self.shape, self.itemsize, index)
        except NotImplementedError:
            host = self.numpy()
            host[index] = value.numpy() if isinstance(value, DeviceArray) else value
            upload_into(self, host)
            return
        if isinstance(value, DeviceArray):
            src = value if value.dtype == self.dtype else value.astype(self.dtype)
            if src.shape != shape:
                if np.broadcast_shapes(src.shape, shape) != tuple(shape):
                    raise ValueError(f"could not broadcast input array from shape {src.shape} "
                                     f"into shape {tuple(shape)}")
                src = broadcast_array(src, tuple(shape))
        else:
            src = from_numpy(np.ascontiguousarray(
                np.broadcast_to(np.asarray(value, dtype=self.dtype), shape)))
        if math.prod(shape):
            strided_copy(src.ptr, contiguous_strides(shape), self.ptr + offset * self.itemsize,
                         strides, shape, self.itemsize)

    # ------------------------------------------------------------- views and copies
    def reshape(self, *shape: int | Sequence[int]) -> DeviceArray:
        dims = shape[0] if len(shape) == 1 and isinstance(shape[0], Sequence) else shape
        new = _resolve_shape(tuple(int(d) for d in dims), self.size)  # type: ignore[union-attr]
        return DeviceArray(self._buf, self._off, new, self.dtype)

    def flat_view(self, offset: int, count: int, shape: tuple[int, ...] | None = None) -> DeviceArray:
        """A view of ``count`` elements starting at element ``offset`` of this buffer."""
        if offset < 0 or count < 0 or offset + count > max(self.size, 1):
            raise ValueError(f"flat_view [{offset}, {offset + count}) of {self.size} elements")
        return DeviceArray(self._buf, self._off + offset * self.dtype.itemsize,
                           shape if shape is not None else (count,), self.dtype)

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
    return DeviceArray(_Block(max(math.prod(shp), 1) * dt.itemsize), 0, shp, dt)


def zeros(shape: Sequence[int], dtype: Any) -> DeviceArray:
    out = empty(shape, dtype)
    if out.nbytes:
        check(lib.tg_memset_zero(out.ptr, out.nbytes, _State.stream), "zeros")
    return out


def _host_bytes(nbytes: int) -> np.ndarray:
    """A page-locked host byte array that lives as long as the process (they are few and
    reused: staging blocks and the pinned input arrays of a training loop)."""
    p = ctypes.c_void_p()
    check(lib.tg_host_alloc(ctypes.byref(p), max(nbytes, 1)), "pinned allocation")
    raw = (ctypes.c_ubyte * max(nbytes, 1)).from_address(int(p.value or 0))
    arr = np.frombuffer(raw, dtype=np.uint8)[:nbytes]
    _PINNED.append((arr.ctypes.data, nbytes, raw))
    return arr


class _Event:
    """A timing-free CUDA event recorded behind a copy (to know when its source is free)."""

    __slots__ = ("handle",)

    def __init__(self) -> None:
        h = ctypes.c_void_p()
        check(lib.tg_event_create(ctypes.byref(h)), "event")
        self.handle = h.value

    def record(self) -> None:
        check(lib.tg_event_record(self.handle, _State.stream), "event record")

    def query(self) -> bool:
        r = lib.tg_event_query(self.handle)
        if r < 0:
            check(-r, "event query")
        return r == 1

    def __del__(self) -> None:
        if self.handle:
            try:
                lib.tg_event_destroy(self.handle)
            except Exception:  # noqa: BLE001 - interpreter shutdown
                pass


class _Staging:
    """Page-locked staging blocks for small uploads from pageable host arrays.

    A block is reused only after the CUDA event recorded behind its copy has completed, so
    an upload never waits for the device queue (no stream synchronisation on the hot path).
    """

    LIMIT = 4 << 20  # larger uploads (model initialisation) copy synchronously

    def __init__(self) -> None:
        self.blocks: list[list[Any]] = []  # [pinned bytes, capacity, event or None]

    def upload(self, dst: DeviceArray, arr: np.ndarray) -> None:
        block = None
        for b in self.blocks:
            if b[1] >= arr.nbytes and (b[2] is None or b[2].query()):
                block = b
                break
        if block is None:
            cap = max(1 << 16, 1 << (arr.nbytes - 1).bit_length())
            block = [_host_bytes(cap), cap, None]
            self.blocks.append(block)
        host = block[0][: arr.nbytes]
        host[:] = arr.reshape(-1).view(np.uint8)
        check(lib.tg_memcpy_h2d(dst.ptr, host.ctypes.data, arr.nbytes, _State.stream), "h2d")
        ev = block[2] or _Event()
        ev.record()
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
    n = math.prod(shape)
    return _host_bytes(max(n, 1) * dt.itemsize)[: n * dt.itemsize].view(dt).reshape(shape)


def _is_pinned(arr: np.ndarray) -> bool:
    p = arr.ctypes.data
    return any(base <= p and p + arr.nbytes <= base + n for base, n, _ in _PINNED)


def is_pinned(arr: np.ndarray) -> bool:
    """Whether ``arr`` lies in page-locked memory from ``pinned_empty``."""
    return _is_pinned(arr)


def from_numpy(arr: np.ndarray, dtype: Any = None) -> DeviceArray:
    # ascontiguousarray gives 0-d input a shape of (1,): keep the caller's shape.
    a = np.ascontiguousarray(arr, dtype=dtype).reshape(np.shape(arr))
    out = empty(a.shape, a.dtype)
    upload_into(out, a)
    return out


def copy_into(dst: DeviceArray, src: DeviceArray) -> None:
    if dst.nbytes != src.nbytes:
        raise ValueError(f"copy of {src.nbytes} bytes into {dst.nbytes}")
    if src.nbytes:
        check(lib.tg_memcpy_d2d(dst.ptr, src.ptr, src.nbytes, _State.stream), "d2d")


_READBACK: list[np.ndarray] = []


def _staging_for_readback(nbytes: int) -> np.ndarray:
    """One reusable page-locked block for bulk device-to-host copies (grown on demand)."""
    if not _READBACK or _READBACK[0].nbytes < nbytes:
        _READBACK[:] = [_host_bytes(max(nbytes, 1 << 20))]
    return _READBACK[0][:nbytes]


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
    staging = _staging_for_readback(max(total, 16))
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
