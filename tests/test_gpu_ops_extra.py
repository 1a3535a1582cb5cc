"""The remaining ops of the reference's API on the device, against the reference's own results
(``tests/golden/ops_extra.npz``, float64; the program is shared with the fixture generator,
``specs.ops_extra_program``): softmax / log_softmax / logsumexp (also with ``-inf`` entries),
max / min with tied extrema, where and masked_fill, concat, binary cross entropy with logits
(every reduction, logits 0 and +-40), the Elman RNN (tanh and relu), matmul with vectors,
comparisons and all / any / argmax, attention with a boolean mask (also with the causal mask
and dropout) and with values wider than the keys. float64 at 1e-10, fp32 at 1e-4; boolean
and index results exactly.
"""

from __future__ import annotations

import types

import numpy as np
import pytest

from tests.conftest import assert_parity, load_golden
from tests.golden.specs import ops_extra_inputs, ops_extra_program

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,rel", [(np.float64, 1e-10), (np.float32, 1e-4)],
                         ids=["fp64", "fp32"])
def test_extra_ops_match_reference(dtype, rel):
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import ops

    gold = load_golden("ops_extra.npz")
    d = {k: (v.astype(dtype) if v.dtype.kind == "f" else v) for k, v in ops_extra_inputs().items()}
    tg.set_default_dtype(dtype)
    try:
        O = types.SimpleNamespace(rnn=ops.rnn, sdpa=ops.scaled_dot_product_attention)
        ours = ops_extra_program(tg, O, lambda t: t.numpy(), d)
    finally:
        tg.set_default_dtype(np.float32)
    assert set(ours) == {k for k in gold if not k.startswith("loader_")}
    for k, v in ours.items():
        ref = gold[k]
        assert np.shape(v) == ref.shape, (k, np.shape(v), ref.shape)
        if ref.dtype.kind in "iub":
            np.testing.assert_array_equal(v, ref, err_msg=k)
        else:
            assert_parity(v, ref, rel, k)


def test_profiler_rows_add_up():
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import profiler

    x = tg.Tensor(np.random.default_rng(0).standard_normal((64, 32)), requires_grad=True)
    w = tg.Tensor(np.random.default_rng(1).standard_normal((16, 32)), requires_grad=True)
    with profiler.profile() as prof:
        loss = tg.softmax(tg.linear(x, w), -1).sum()
        loss.backward()
    assert prof.ops["linear"].forward_calls == 1 and prof.ops["linear"].backward_calls == 1
    assert prof.ops["softmax"].forward_calls == 1
    assert profiler.ENGINE in prof.ops
    assert 0 < prof.profiled_seconds <= prof.wall_seconds
    table = prof.table()
    assert table.splitlines()[0].startswith("op") and "wall time" in table.splitlines()[-1]
    with pytest.raises(RuntimeError, match="nested"), profiler.profile(), profiler.profile():
        pass


def test_gradcheck_and_gradgradcheck_on_the_device():
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import GradcheckError, gradcheck, gradgradcheck

    rng = np.random.default_rng(4)
    x = tg.Tensor(rng.standard_normal((3, 4)), requires_grad=True)
    w = tg.Tensor(rng.standard_normal((4, 2)), requires_grad=True)
    assert gradcheck(lambda a, b: tg.tanh(a @ b), [x, w])
    assert gradgradcheck(lambda a, b: tg.softmax(a @ b, -1), [x, w])
    with pytest.raises(TypeError, match="float64"):
        gradcheck(lambda a: a * 2.0, [tg.Tensor(np.ones(3, np.float32), requires_grad=True)])
    # A wrong VJP is caught (a user op whose backward forgets the factor 2).
    from tensorgrad_b200.ops._util import make_result

    def doubled(a):
        return make_result((a * 2.0).data, (a,), lambda g, need: (g,), "bad_double")

    with pytest.raises(GradcheckError, match="input 0"):
        gradcheck(doubled, [x])
    assert not gradcheck(doubled, [x], raise_exception=False)


def test_data_loader_batches_upload_in_order():
    import tensorgrad_b200 as tg
    from tensorgrad_b200.utils import DataLoader

    xs = np.arange(30, dtype=np.float64).reshape(10, 3)
    ys = np.arange(10)
    loader = DataLoader(xs, ys, batch_size=4, shuffle=True, seed=5)
    for epoch in range(2):
        order = []
        for xb, yb in loader:
            assert isinstance(xb, tg.Tensor) and xb.dtype == np.float64 and yb.dtype == np.int64
            np.testing.assert_array_equal(xb.numpy(), xs[yb.numpy()])
            order.extend(yb.numpy().tolist())
        np.testing.assert_array_equal(order, load_golden("ops_extra.npz")[f"loader_epoch{epoch}"])


def test_device_array_assignment():
    """``tensor.data[index] = value`` as NumPy assigns: whole array, basic-index views (with
    broadcasting, from host values and from device arrays) and integer / boolean arrays."""
    import tensorgrad_b200 as tg
    from tensorgrad_b200 import device

    ref = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    t = tg.Tensor(ref.copy())
    cases = [
        (Ellipsis, 7.0), ((0, 1), np.array([1, 2, 3, 4], np.float32)), ((slice(None), 2), -1.0),
        ((1, slice(0, 3, 2), slice(1, None)), np.ones((2, 3), np.float32) * 5),
        ((Ellipsis, 0), np.arange(3, dtype=np.float32)), (np.array([1, 0]), 9.0),
        (ref > 20, 0.5),
    ]
    for index, value in cases:
        ref[index] = value
        t.data[index] = value
        np.testing.assert_array_equal(t.numpy(), ref, err_msg=str(index))
    src = device.from_numpy(np.full((4,), 3.0, np.float32))
    ref[1, :, :] = 3.0
    t.data[1] = src  # a device row broadcast over the view
    np.testing.assert_array_equal(t.numpy(), ref)
    with pytest.raises(ValueError, match="broadcast"):
        t.data[0] = device.from_numpy(np.ones(5, np.float32))


def test_argument_errors_match_reference_messages():
    import tensorgrad_b200 as tg

    x = tg.Tensor(np.ones((2, 3, 4), np.float32))
    with pytest.raises(ValueError, match="start_axis must not come after end_axis"):
        tg.flatten(x, 2, 1)
    assert tg.flatten(x, 1, 2).shape == (2, 12)
    with pytest.raises(ValueError, match="0-d tensors; use mul instead"):
        tg.matmul(tg.Tensor(np.float32(2.0)), x)
    with pytest.raises(ValueError, match="without a copy"):
        x.__array__(np.float64, copy=False)
    assert np.asarray(x, dtype=np.float64).dtype == np.float64
