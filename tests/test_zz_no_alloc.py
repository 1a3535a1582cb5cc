"""The allocation-free LayerNorm VJP against the allocating one.

``tg_layer_norm_backward_noalloc`` serves callers that cannot allocate device memory (a C or
FFI host without a CUDA allocator of its own, or a latency-critical path where cudaMalloc's
possible device synchronisation is not acceptable): its partial sums live in a static 4 MiB
device array instead of caller-provided scratch. It must give the same gradients as
``tg_layer_norm_backward`` on two calls in a row (the array keeps the previous call's
contents), and refuse sizes whose partials would not fit. This file is collected last.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ops as O
from tests.conftest import assert_parity

pytestmark = pytest.mark.gpu


def _run(entry: str, dtype, x, w, g):
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import check, lib

    code = device.dtype_code(np.dtype(dtype))
    rows, cols = x.shape
    dx, dw, dg = (device.from_numpy(a.astype(dtype)) for a in (x, w, g))
    y = device.empty((rows, cols), dtype)
    mean, rstd = device.empty((rows,), dtype), device.empty((rows,), dtype)
    check(lib.tg_layer_norm_forward(code, dx.ptr, dw.ptr, None, y.ptr, mean.ptr, rstd.ptr,
                                    rows, cols, 1e-5, device.stream()))
    gx, gw, gb = (device.empty(s, dtype) for s in ((rows, cols), (cols,), (cols,)))
    if entry == "noalloc":
        check(lib.tg_layer_norm_backward_noalloc(code, dg.ptr, dx.ptr, dw.ptr, mean.ptr,
                                                 rstd.ptr, gx.ptr, gw.ptr, gb.ptr, rows, cols,
                                                 7, device.stream()))
    else:
        scratch = device.scratch(lib.tg_layer_norm_scratch_bytes(code, rows, cols))
        check(lib.tg_layer_norm_backward(code, dg.ptr, dx.ptr, dw.ptr, mean.ptr, rstd.ptr,
                                         gx.ptr, gw.ptr, gb.ptr, rows, cols, 7, scratch.ptr,
                                         device.stream()))
    return gx.numpy(), gw.numpy(), gb.numpy()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_noalloc_matches_allocating_entry_point_twice(dtype):
    rng = np.random.default_rng(11)
    # Two calls in a row with different shapes: the second reuses the static array.
    for rows, cols in ((8192, 768), (333, 100)):
        x = rng.standard_normal((rows, cols)) * 2 + 0.5
        w = 1 + 0.1 * rng.standard_normal(cols)
        g = rng.standard_normal((rows, cols))
        ours = _run("noalloc", dtype, x, w, g)
        theirs = _run("alloc", dtype, x, w, g)
        for a, b, name in zip(ours, theirs, ("gx", "gw", "gb"), strict=True):
            # Same kernels, same launch shape: the results agree exactly.
            np.testing.assert_array_equal(a, b, err_msg=f"{name} {rows}x{cols}")
        _, xhat, rstd = O.layer_norm_forward(x, w, None)
        ref = O.layer_norm_backward(g, xhat, rstd, w)
        for a, r, name in zip(ours, ref, ("gx", "gw", "gb"), strict=True):
            assert_parity(a, r, 1e-4 if dtype == np.float32 else 1e-10, f"{name} vs oracle")


def test_noalloc_rejects_partials_beyond_the_static_array():
    from tensorgrad_b200._lib import last_error, lib

    # 296 blocks x 2 x 1024 columns x 8 bytes = 4.6 MiB > 4 MiB: refused before any launch.
    status = lib.tg_layer_norm_backward_noalloc(1, None, None, None, None, None, None, None,
                                                None, 100000, 1024, 7, None)
    assert status == 1
    assert "static scratch" in last_error()
