"""The bounded waits of the fused attention kernels, made to run out on purpose.

The test shortens the wait budget of the fused kernels to about a millisecond and tells the
forward's producer to issue no load: the first wait on a load then has nothing to wait for
(a flag that nothing sets), gives up, records TG_ERR_TIMEOUT and the kernel drains and frees
its tensor memory with nothing in flight. The host reads the status through the C ABI and
the next synchronisation raises; with the defaults restored, the same call matches the
oracle again, so the context is still usable. No fault, trap or unbounded wait is involved.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import ops as O
from tests.conftest import assert_parity

pytestmark = pytest.mark.gpu

TG_ERR_TIMEOUT = 5


def _forward(q, k, v, causal):
    """One fused forward through the C ABI: (B, H, T, D) contiguous fp32 inputs."""
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F32, AttnShape, check, lib

    b, h, t, d = q.shape
    s = AttnShape(batch=b, heads=h, tq=t, tk=k.shape[2], head_dim=d,
                  q_sb=h * t * d, q_sh=t * d, q_st=d,
                  k_sb=h * k.shape[2] * d, k_sh=k.shape[2] * d, k_st=d,
                  v_sb=h * k.shape[2] * d, v_sh=k.shape[2] * d, v_st=d,
                  o_sb=h * t * d, o_sh=t * d, o_st=d, causal=int(causal))
    dq, dk, dv = (device.from_numpy(a.astype(np.float32)) for a in (q, k, v))
    o = device.zeros(q.shape, np.float32)
    lse = device.zeros((b, h, t), np.float32)
    scratch = device.scratch(lib.tg_attention_forward_scratch_bytes(F32, s))
    check(lib.tg_attention_forward(F32, s, dq.ptr, dk.ptr, dv.ptr, o.ptr, lse.ptr, scratch.ptr,
                                   device.stream()), "attention forward")
    return o, (dq, dk, dv, lse, scratch)


def test_fused_forward_wait_runs_out_reports_timeout_and_recovers():
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import check, lib

    rng = np.random.default_rng(77)
    q, k, v = (rng.standard_normal((1, 2, 256, 64)) for _ in range(3))
    device.synchronize()
    assert lib.tg_attention_tc_status(1) == 0
    check(lib.tg_attention_set_wait_test(2_000_000, 1))  # ~1 ms, no loads issued
    try:
        _, keep = _forward(q, k, v, causal=True)
        check(lib.tg_stream_synchronize(device.stream()), "synchronize")
        assert lib.tg_attention_tc_status(0) == TG_ERR_TIMEOUT
        with pytest.raises(RuntimeError, match="bounded device-side wait ran out"):
            device.synchronize()  # reads and clears the status word
        assert lib.tg_attention_tc_status(0) == 0
        del keep
    finally:
        check(lib.tg_attention_set_wait_test(0, 0))
    o, _ = _forward(q, k, v, causal=True)
    got = o.numpy()
    assert lib.tg_attention_tc_status(1) == 0
    assert_parity(got, O.attention_forward(q, k, v, True)[0], 1e-4, "out after recovery")
