"""The CNN path on the device: conv2d, batch norm, max pooling and whole training steps.

* op level: the reference's own outputs (``conv_pool.npz``), the reference's known-answer
  rules (naive convolution loops, numpy.argmax pooling with ties and NaNs), the oracle;
* model level: two steps of the small CNN against the reference fixture (fp32 at 1e-4,
  float64 at 1e-10), and one step of the CNN configuration's layer stack against the
  float64 oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cnn as ocnn
from oracle import ops as O
from tests.conftest import (
    assert_parity, assert_update_parity, assert_zero_gradient, ill_conditioned, load_golden,
)
from tests.golden.specs import (
    CNN_SMALL, CNN_ZERO_GRAD, CONV_CASES, POOL_CASES, conv_inputs, pool_input,
)
from tests.test_oracle_golden import argmax_pool, naive_conv2d

pytestmark = pytest.mark.gpu

REL = {np.float32: 1e-4, np.float64: 1e-10}


def tensors(dtype, *arrays, grad=True):
    import tensorgrad_b200 as tg

    return [tg.Tensor(np.asarray(a, dtype=dtype), requires_grad=grad) for a in arrays]


# ---------------------------------------------------------------------------- ops
@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["fp32", "fp64"])
@pytest.mark.parametrize("case", range(len(CONV_CASES)))
def test_conv2d_matches_reference_fixture(case, dtype):
    import tensorgrad_b200 as tg

    gold = load_golden("conv_pool.npz")
    x_shape, wspec, stride, padding, seed = CONV_CASES[case]
    x, w, b, rng = conv_inputs(x_shape, wspec, seed)
    tx, tw, tb = tensors(dtype, x, w, b)
    y = tg.conv2d(tx, tw, tb, stride=stride, padding=padding)
    g = rng.standard_normal(y.shape)
    gx, gw, gb = tg.autograd.grad(y, [tx, tw, tb], grad_outputs=g.astype(dtype))
    rel = REL[dtype]
    for name, ours in (("y", y), ("gx", gx), ("gw", gw), ("gb", gb)):
        assert_parity(ours.numpy(), gold[f"conv{case}/{name}"], rel, f"conv{case} {name}")


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["fp32", "fp64"])
@pytest.mark.parametrize("case", range(len(POOL_CASES)))
def test_max_pool2d_matches_reference_fixture(case, dtype):
    import tensorgrad_b200 as tg

    gold = load_golden("conv_pool.npz")
    x_shape, kernel, stride, padding, seed = POOL_CASES[case]
    x, rng = pool_input(x_shape, seed)
    (tx,) = tensors(dtype, x)
    y = tg.max_pool2d(tx, kernel, stride, padding)
    g = rng.standard_normal(y.shape)
    (gx,) = tg.autograd.grad(y, [tx], grad_outputs=g.astype(dtype))
    # Selection is exact (the values are on a half-integer grid, exact in fp32 too); where
    # windows overlap, an input cell sums several window gradients, in another order.
    np.testing.assert_array_equal(y.numpy(), gold[f"pool{case}/y"].astype(dtype))
    assert_parity(gx.numpy(), gold[f"pool{case}/gx"], REL[dtype], f"pool{case} gx")


@pytest.mark.parametrize(("stride", "pad"), [(1, 0), (1, 1), (2, 1), (3, 0)])
def test_conv2d_matches_naive_loops(rng, stride, pad):
    import tensorgrad_b200 as tg

    x = rng.standard_normal((2, 3, 7, 6))
    w = rng.standard_normal((4, 3, 3, 3))
    b = rng.standard_normal(4)
    y = tg.conv2d(*tensors(np.float32, x, w, b, grad=False), stride=stride, padding=pad)
    assert_parity(y.numpy(), naive_conv2d(x, w, b, stride, pad), 1e-4, "conv vs loops")


# (8, 12) and (16, 8) with 2 x 2 windows at stride 2 take the vectorised 2 x 2 kernels.
@pytest.mark.parametrize(("k", "stride", "pad", "hw"),
                         [(2, 2, 0, (7, 6)), (3, 1, 1, (7, 6)), (3, 2, 1, (7, 6)),
                          (2, 1, 0, (7, 6)), (2, 2, 0, (8, 12)), (2, 2, 0, (16, 8))])
def test_max_pool2d_ties_and_nans_follow_argmax(k, stride, pad, hw):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(k * 10 + stride + hw[1])
    x = np.round(rng.standard_normal((2, 3, *hw)))
    x.reshape(-1)[::13] = np.nan
    (t,) = tensors(np.float32, x)
    out = tg.max_pool2d(t, k, stride, pad)
    g = rng.standard_normal(out.shape).astype(np.float32)
    out.backward(g)
    ey, egx = argmax_pool(x, g.astype(np.float64), k, stride, pad)
    np.testing.assert_array_equal(out.numpy(), ey.astype(np.float32))
    assert_parity(t.grad.numpy(), egx, 1e-6, "pool gradient")


def test_max_pool2d_padding_never_wins():
    import tensorgrad_b200 as tg

    out = tg.max_pool2d(tg.Tensor(-np.ones((1, 1, 2, 2), dtype=np.float32)), 2, stride=1,
                        padding=1)
    assert np.all(out.numpy() == -1.0)


@pytest.mark.parametrize("shape", [(256, 3, 64, 64, 32), (64, 32, 32, 32, 64), (3, 5, 9, 11, 7)],
                         ids=["conv1", "conv2", "odd"])
def test_conv2d_backward_matches_oracle_at_config_shapes(shape):
    # conv1 (K = 27: padded patch rows, no input gradient needed in the model but checked
    # here), conv2 (K = 288, tensor-core weight gradient with split-K over 1024-pixel
    # images), and an odd shape whose pixel count is not a multiple of 16 (other GEMM path).
    import tensorgrad_b200 as tg

    n, c, h, c_out = shape[0], shape[1], shape[2], shape[4]
    wd = shape[3]
    rng = np.random.default_rng(sum(shape))
    x = rng.standard_normal((n, c, h, wd))
    w = rng.standard_normal((c_out, c, 3, 3)) / np.sqrt(9 * c)
    b = rng.standard_normal(c_out)
    tx, tw, tb = tensors(np.float32, x, w, b)
    y = tg.conv2d(tx, tw, tb, padding=1)
    g = rng.standard_normal(y.shape)
    gx, gw, gb = tg.autograd.grad(y, [tx, tw, tb], grad_outputs=g.astype(np.float32))
    ey, cols = ocnn.conv2d_forward(x, w, b, (1, 1), (1, 1))
    egx, egw, egb = ocnn.conv2d_backward(g, x.shape, w, cols, (1, 1), (1, 1))
    for name, ours, ref in (("y", y, ey), ("gx", gx, egx), ("gw", gw, egw), ("gb", gb, egb)):
        assert_parity(ours.numpy(), ref, 1e-4, f"{shape} {name}")


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["fp32", "fp64"])
@pytest.mark.parametrize("shape", [(16, 32, 64, 64), (8, 6, 5, 7), (4, 3)], ids=["2d", "odd", "1d"])
def test_batch_norm_train_matches_oracle(shape, dtype):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(len(shape) * 7 + shape[0])
    c = shape[1]
    x = rng.standard_normal(shape) * 3 + 1.5
    w = 1 + 0.1 * rng.standard_normal(c)
    b = 0.1 * rng.standard_normal(c)
    g = rng.standard_normal(shape)
    tx, tw, tb = tensors(dtype, x, w, b)
    from tensorgrad_b200 import device

    rm = device.from_numpy(np.full(c, 0.2, dtype=dtype))
    rv = device.from_numpy(np.full(c, 0.7, dtype=dtype))
    y = tg.ops.batch_norm(tx, rm, rv, tw, tb, training=True, momentum=0.1, eps=1e-5)
    gx, gw, gb = tg.autograd.grad(y, [tx, tw, tb], grad_outputs=g.astype(dtype))
    erm, erv = np.full(c, 0.2), np.full(c, 0.7)
    ey, cache = ocnn.batch_norm_forward(x, w, b, erm, erv)
    egx, egw, egb = ocnn.batch_norm_backward(g, cache, w)
    rel = REL[dtype]
    for name, ours, ref in (("y", y.numpy(), ey), ("gx", gx.numpy(), egx), ("gw", gw.numpy(), egw),
                            ("gb", gb.numpy(), egb), ("running_mean", rm.numpy(), erm),
                            ("running_var", rv.numpy(), erv)):
        assert_parity(ours, ref, rel, f"{shape} {name}")


# ---------------------------------------------------------------------------- model steps
def cnn_model(cfg: ocnn.Config):
    import tensorgrad_b200 as tg

    nn = tg.nn
    return nn.Sequential(
        nn.Conv2d(cfg.in_channels, cfg.c1, 3, padding=1), nn.BatchNorm2d(cfg.c1), nn.ReLU(),
        nn.MaxPool2d(2), nn.Conv2d(cfg.c1, cfg.c2, 3, padding=1), nn.BatchNorm2d(cfg.c2),
        nn.ReLU(), nn.MaxPool2d(2), nn.Flatten(),
        nn.Linear(cfg.c2 * (cfg.size // 4) ** 2, cfg.classes),
    )


def run_cnn_steps(cfg, batch, seed, steps, dtype, record_acts=False):
    import tensorgrad_b200 as tg

    tg.set_default_dtype(dtype)
    try:
        tg.manual_seed(0)
        model = cnn_model(cfg)
        model.load_state_dict(ocnn.init_params(cfg, seed) | ocnn.init_buffers(cfg))
        names = [n for n, _ in model.named_parameters()]
        assert names == [n for n, _ in ocnn.param_shapes(cfg)]
        params = list(model.parameters())
        opt = tg.optim.AdamW(params, lr=3e-4, betas=(0.9, 0.999), eps=1e-8, weight_decay=1e-4)
        recs = []
        for step in range(1, steps + 1):
            x, labels = ocnn.synthetic_batch(cfg, batch, seed + step)
            h, outs = tg.Tensor(x.astype(dtype)), []
            for layer in model:  # what Sequential.forward does, keeping the activations
                h = layer(h)
                outs.append(h)
            loss = tg.cross_entropy(h, labels)
            opt.zero_grad()
            loss.backward()
            rec = {"loss": float(loss.item()),
                   "grads": {n: p.grad.numpy() for n, p in zip(names, params, strict=True)},
                   "before": {n: p.numpy() for n, p in zip(names, params, strict=True)}}
            opt.step()
            rec["params"] = {n: p.numpy() for n, p in zip(names, params, strict=True)}
            rec["buffers"] = {n: b.numpy() for n, b in model.named_buffers()}
            if record_acts:
                rec["acts"] = {"b1": outs[1].numpy(), "r1": outs[2].numpy(),
                               "b2": outs[5].numpy(), "r2": outs[6].numpy()}
            recs.append(rec)
        return recs
    finally:
        tg.set_default_dtype(np.float32)


def check_cnn(recs, refs, rel):
    """Loss and gradients with the parity metric (the zero-gradient conv biases absolutely);
    running statistics (the mean relative to the running standard deviation, the scale at
    which batch norm uses it); post-AdamW parameters over the entries whose gradients are
    determined at the tolerance, the zero-gradient biases excluded there and checked instead
    through AdamW applied to our own gradients."""
    ill: dict[str, np.ndarray] = {}
    for step, (rec, ref) in enumerate(zip(recs, refs, strict=True), start=1):
        assert rec["loss"] == pytest.approx(ref["loss"], rel=rel)
        for n, g in rec["grads"].items():
            if n in CNN_ZERO_GRAD:
                scale = float(np.abs(ref["grads"][CNN_ZERO_GRAD[n]]).max())
                assert_zero_gradient(g, scale, rel, f"step{step} grad {n}")
                continue
            assert_parity(g, ref["grads"][n], rel, f"step{step} grad {n}")
            mask = ill_conditioned(ref["grads"][n], rel)
            ill[n] = mask if n not in ill else (ill[n] | mask)
        for n, b in rec["buffers"].items():
            scale = 1.0
            if n.endswith("running_mean"):
                scale = float(np.sqrt(np.abs(ref["buffers"][n.replace("mean", "var")]).max()))
            err = float(np.abs(b - ref["buffers"][n]).max())
            assert err <= rel * max(float(np.abs(ref["buffers"][n]).max()), scale), (
                f"step{step} {n}: {err:.3e}")
        for n, p in rec["params"].items():
            if n in CNN_ZERO_GRAD:
                continue
            assert_update_parity(p, ref["params"][n], ill[n], rel, f"step{step} param {n}")
        if step == 1:
            for n, p in rec["params"].items():
                mine, _, _ = O.adamw_update(rec["before"][n].astype(np.float64),
                                            rec["grads"][n].astype(np.float64),
                                            np.zeros(p.shape), np.zeros(p.shape), 1, 3e-4,
                                            (0.9, 0.999), 1e-8, 1e-4)
                assert_parity(p, mine, max(rel, 1e-6), f"AdamW kernel on our grads {n}")


@pytest.mark.parametrize("dtype", [np.float32, np.float64], ids=["fp32", "fp64"])
def test_cnn_small_two_steps_match_reference_fixture(dtype):
    gold = load_golden("cnn_small.npz")
    s = CNN_SMALL
    recs = run_cnn_steps(s["cfg"], s["batch"], s["seed"], s["steps"], dtype)
    names = list(recs[0]["grads"])
    refs = [{"loss": float(gold[f"step{k}/loss"]),
             "grads": {n: gold[f"step{k}/grad/{n}"] for n in names},
             "params": {n: gold[f"step{k}/param/{n}"] for n in names},
             "buffers": {n: gold[f"step{k}/buffer/{n}"] for n in recs[0]["buffers"]}}
            for k in range(1, s["steps"] + 1)]
    check_cnn(recs, refs, REL[dtype])


def decisions_of(acts):
    """The discrete choices of a run: ReLU masks and the pooling winners of its values."""
    return {"relu1": acts["b1"] > 0, "relu2": acts["b2"] > 0,
            "win1": ocnn.max_pool2d_forward(acts["r1"].astype(np.float64), (2, 2), (2, 2))[1],
            "win2": ocnn.max_pool2d_forward(acts["r2"].astype(np.float64), (2, 2), (2, 2))[1]}


def assert_near_ties_only(ours, ref_acts, rel):
    """Every ReLU decision or pooling winner of the float32 run that differs from the float64
    oracle's own is a near-tie for it: a pre-activation within ``rel`` of zero, or two window
    cells within ``rel`` of each other (relative to the largest activation)."""
    theirs = decisions_of(ref_acts)
    for k in ("1", "2"):
        b = ref_acts["b" + k]
        scale = float(np.abs(b).max())
        flip = ours["relu" + k] != theirs["relu" + k]
        assert np.all(np.abs(b[flip]) <= rel * scale), f"relu{k}: decisive flips"
        r = ref_acts["r" + k]
        diff = ours["win" + k] != theirs["win" + k]
        if diff.any():
            n, c, oh, ow = diff.shape
            cells = r.reshape(n, c, oh, 2, ow, 2).transpose(0, 1, 2, 4, 3, 5).reshape(n, c, oh, ow, 4)
            a = np.take_along_axis(cells, ours["win" + k][..., None], -1)[..., 0]
            t = np.take_along_axis(cells, theirs["win" + k][..., None], -1)[..., 0]
            assert np.all(np.abs(a - t)[diff] <= rel * scale), f"pool{k}: decisive flips"


def test_cnn_config_layer_stack_matches_oracle():
    # The CNN configuration's layers (3->32->64 channels, 64x64 images, 4 classes) on a
    # 32-image batch, one step against the float64 oracle. Among ~4M ReLU inputs a few sit
    # within float32 rounding of zero (or of a pooling tie), where float32 and float64 may
    # choose differently and route a whole gradient element elsewhere. So the oracle runs
    # with this run's discrete choices, and every choice that differs from the oracle's own
    # must be such a near-tie.
    cfg = ocnn.Config()
    seed, batch = 3, 32
    recs = run_cnn_steps(cfg, batch, seed, 1, np.float32, record_acts=True)
    x, labels = ocnn.synthetic_batch(cfg, batch, seed + 1)
    own: dict = {}
    ocnn.forward_backward(ocnn.init_params(cfg, seed), ocnn.init_buffers(cfg), x, labels,
                          acts=own)
    assert_near_ties_only(decisions_of(recs[0]["acts"]), own, 1e-5)
    ref = ocnn.train_step(ocnn.init_params(cfg, seed), ocnn.init_buffers(cfg), x, labels,
                          decisions=decisions_of(recs[0]["acts"]))
    check_cnn(recs, [ref], 1e-4)
