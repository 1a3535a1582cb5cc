"""Host allocator tuning (the reference's utils/memory.py): keep memory freed by NumPy in the
process instead of returning it to the kernel. The device side needs none of it (the
library's stream-ordered pool keeps freed device blocks); host-heavy loops around the device
step (data preparation, checkpoint writing) still profit from it."""

from __future__ import annotations

import ctypes
import ctypes.util
import sys

__all__ = ["retain_freed_memory"]

_M_TRIM_THRESHOLD, _M_MMAP_THRESHOLD = -1, -3  # mallopt(3) parameters of glibc's malloc.h


def retain_freed_memory(mmap_threshold: int = 64 << 20, trim_threshold: int = 1 << 30) -> bool:
    """Serve requests up to ``mmap_threshold`` bytes from the heap and return free heap
    memory to the kernel only beyond ``trim_threshold`` bytes (both set together: raising
    only the trim threshold freezes glibc's adaptive mmap threshold). Returns whether glibc
    took both settings; ``False`` elsewhere, where nothing changes."""
    if not sys.platform.startswith("linux"):
        return False
    try:
        libc = ctypes.CDLL(ctypes.util.find_library("c") or "libc.so.6")
    except OSError:
        return False
    mallopt = getattr(libc, "mallopt", None)
    if mallopt is None:
        return False
    mallopt.argtypes = [ctypes.c_int, ctypes.c_int]
    mallopt.restype = ctypes.c_int
    ok_mmap = bool(mallopt(_M_MMAP_THRESHOLD, int(mmap_threshold)))
    ok_trim = bool(mallopt(_M_TRIM_THRESHOLD, int(trim_threshold)))
    return ok_mmap and ok_trim
