"""Per-op parity of the CUDA path (through the C ABI) against the float64 oracle."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import ops as O
from tests.conftest import assert_parity, assert_zero_gradient, load_golden
from tests.golden.specs import ATTN_CASES, attention_inputs

pytestmark = pytest.mark.gpu

REL32 = 1e-4   # fp32 kernels vs the float64 reference
REL64 = 1e-10  # float64 build mode


@pytest.fixture(params=[np.float32, np.float64], ids=["fp32", "fp64"])
def dtype(request):
    import tensorgrad_b200 as tg

    tg.set_default_dtype(request.param)
    yield request.param
    tg.set_default_dtype(np.float32)


def rel(dtype) -> float:
    return REL32 if dtype == np.float32 else REL64


def tensor(a, dtype, requires_grad=True):
    import tensorgrad_b200 as tg

    return tg.Tensor(np.asarray(a, dtype=dtype), requires_grad=requires_grad)


# ------------------------------------------------------------------------------- GEMM
# The last two are large enough for CTA pairs (256-row tiles, cta_group::2) when those are
# enabled: 128- and 256-wide tiles with ragged rows (the odd CTA of the last pair has none)
# and ragged columns (see test_gemm_cta_pairs_match_float64).
# (Reductions of at most 8 take the small-k kernel: test_gemm_small_k.)
GEMM_SHAPES = [(1, 1, 9), (7, 5, 12), (128, 128, 32), (130, 257, 100), (300, 64, 768),
               (64, 300, 36), (1000, 333, 68), (8192 // 16, 3072 // 4, 768), (2100, 1000, 100),
               (4096, 2000, 300), (160, 96, 200)]
# (160, 96, 200): MN extents that are multiples of 32 but not of the tile, so the chunked
# 5-D maps of MN-major operands load boxes that reach past the last chunk (zero fill).


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
def test_gemm_tensor_core_matches_float64(m, n, k, ta, tb):
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F32, check, lib

    rng = np.random.default_rng(m * 7 + n * 3 + k + 10 * ta + tb)
    a = rng.standard_normal((k, m) if ta else (m, k))
    b = rng.standard_normal((n, k) if tb else (k, n))
    c0 = rng.standard_normal((m, n))
    bias = rng.standard_normal(n)
    ref = 0.5 * ((a.T if ta else a) @ (b.T if tb else b)) + 0.25 * c0 + bias
    da = device.from_numpy(a.astype(np.float32))
    db = device.from_numpy(b.astype(np.float32))
    dc = device.from_numpy(c0.astype(np.float32))
    dbias = device.from_numpy(bias.astype(np.float32))
    lda, ldb = a.shape[1], b.shape[1]
    check(lib.tg_gemm(F32, ta, tb, m, n, k, 0.5, da.ptr, lda, db.ptr, ldb, 0.25, dc.ptr, n,
                      dbias.ptr, device.stream()))
    out = dc.numpy()
    assert lib.tg_gemm_tc_status(1) == 0
    # 3xTF32 reaches near-fp32 accuracy (~1e-5 of max|C|): far inside the 1e-4 tolerance.
    assert_parity(out, ref, 2e-5, f"gemm {m}x{n}x{k} ta={ta} tb={tb}")


@pytest.mark.parametrize("m,n,k,tb", [(4096, 1280, 2048, 1), (8192, 768, 3072, 1),
                                      (8192, 768, 3072, 0)])
def test_gemm_stream_k_tail_matches_float64(m, n, k, tb):
    """Products whose tiles fill the SMs' last round only partly and whose reduction is long
    (64 k-blocks or more per tile) run with the stream-K tail: tiles cut between CTAs sum
    their partials in piece order. Bias included; run twice to check the arrival counters
    are left at zero for the next launch."""
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F32, check, lib

    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k))
    b = rng.standard_normal((n, k) if tb else (k, n))
    bias = rng.standard_normal(n)
    ref = (a @ (b.T if tb else b)) + bias
    da, db = device.from_numpy(a.astype(np.float32)), device.from_numpy(b.astype(np.float32))
    dbias = device.from_numpy(bias.astype(np.float32))
    for _ in range(2):
        dc = device.empty((m, n), np.float32)
        check(lib.tg_gemm(F32, 0, tb, m, n, k, 1.0, da.ptr, k, db.ptr, b.shape[1], 0.0, dc.ptr,
                          n, dbias.ptr, device.stream()))
        # 1e-4, the fp32 parity bar: with k = 2048-3072 the fp32 accumulator in tensor memory
        # takes ~1000 additions of partial sums of a few hundred (2e-5 of max|C| measured
        # 2.3e-5 at k = 3072, with or without the stream-K tail's two-piece sum).
        assert_parity(dc.numpy(), ref, 1e-4, f"stream-K gemm {m}x{n}x{k} tb={tb}")
    assert lib.tg_gemm_tc_status(1) == 0


def test_gemm_cta_pairs_match_float64():
    # The opt-in CTA-pair kernel (TG_GEMM_PAIR=1 is read once per process): the GEMM tests
    # above, on the pair-sized shapes, in a child process with pairs enabled.
    import os
    import subprocess
    import sys

    env = dict(os.environ, TG_GEMM_PAIR="1")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider",
                          os.path.join(root, "tests", "test_gpu_kernels.py"), "-k",
                          "gemm_tensor_core and (2100-1000-100 or 4096-2000-300)"],
                         env=env, cwd=root, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]
    assert "8 passed" in res.stdout, res.stdout[-2000:]


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (7, 5, 3), (51200 // 16, 2048, 2), (333, 130, 8)])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("dt", ["f32", "f64"])
def test_gemm_small_k(m, n, k, ta, tb, dt):
    """Reductions of at most 8 (the LSTM/GRU input projection from 2 inputs) run on the
    CUDA-core small-k kernel: plain FMAs, so fp32 and fp64 both land within rounding."""
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F32, F64, check, lib

    np_dt, code, rel = (np.float32, F32, 1e-6) if dt == "f32" else (np.float64, F64, 1e-14)
    rng = np.random.default_rng(m + n + k + 10 * ta + tb)
    a = rng.standard_normal((k, m) if ta else (m, k))
    b = rng.standard_normal((n, k) if tb else (k, n))
    c0 = rng.standard_normal((m, n))
    bias = rng.standard_normal(n)
    ref = 0.5 * ((a.T if ta else a) @ (b.T if tb else b)) + 0.25 * c0 + bias
    da, db = device.from_numpy(a.astype(np_dt)), device.from_numpy(b.astype(np_dt))
    dc, dbias = device.from_numpy(c0.astype(np_dt)), device.from_numpy(bias.astype(np_dt))
    before = lib.tg_gemm_fallback_count()
    check(lib.tg_gemm(code, ta, tb, m, n, k, 0.5, da.ptr, a.shape[1], db.ptr, b.shape[1], 0.25,
                      dc.ptr, n, dbias.ptr, device.stream()))
    assert_parity(dc.numpy(), ref, rel, f"small-k gemm {m}x{n}x{k} ta={ta} tb={tb}")
    assert lib.tg_gemm_fallback_count() == before


def test_gemm_fallback_is_counted():
    """An fp32 product the tensor-core kernel cannot take (a leading dimension that is not a
    multiple of 4 floats) runs on the CUDA-core kernel, correctly, and is counted."""
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F32, check, lib

    rng = np.random.default_rng(3)
    a, b = rng.standard_normal((64, 30)), rng.standard_normal((30, 50))
    da = device.from_numpy(a.astype(np.float32))
    db = device.from_numpy(b.astype(np.float32))
    dc = device.empty((64, 50), np.float32)
    before = lib.tg_gemm_fallback_count()
    check(lib.tg_gemm(F32, 0, 0, 64, 50, 30, 1.0, da.ptr, 30, db.ptr, 50, 0.0, dc.ptr, 50, None,
                      device.stream()))
    assert_parity(dc.numpy(), a @ b, 1e-5, "fallback gemm")
    assert lib.tg_gemm_fallback_count() == before + 1


def test_gemm_simt_fp64():
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F64, check, lib

    rng = np.random.default_rng(0)
    a, b = rng.standard_normal((77, 45)), rng.standard_normal((45, 93))
    da, db = device.from_numpy(a), device.from_numpy(b)
    dc = device.empty((77, 93), np.float64)
    check(lib.tg_gemm(F64, 0, 0, 77, 93, 45, 1.0, da.ptr, 45, db.ptr, 93, 0.0, dc.ptr, 93, None,
                      device.stream()))
    assert_parity(dc.numpy(), a @ b, 1e-13, "gemm fp64")


# ------------------------------------------------------------------------------- layers
# (batch dims, in, out): plain; out not a multiple of 4 (the VJP re-lays the gradient with
# 16-byte rows for the tensor maps); a wide input with few output tiles (split-K forward).
@pytest.mark.parametrize("lead,fin,fout", [((4, 9), 24, 40), ((33, 7), 48, 65),
                                           ((256,), 4096, 4)])
def test_linear(dtype, lead, fin, fout):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(fin + fout)
    x, w, b, g = (rng.standard_normal(s) for s in ((*lead, fin), (fout, fin), (fout,),
                                                    (*lead, fout)))
    tx, tw, tb = tensor(x, dtype), tensor(w, dtype), tensor(b, dtype)
    y = tg.linear(tx, tw, tb)
    y.backward(g.astype(dtype))
    assert_parity(y.numpy(), O.linear_forward(x, w, b), rel(dtype), "y")
    gx, gw, gb = O.linear_backward(g, x, w, True)
    assert_parity(tx.grad.numpy(), gx, rel(dtype), "gx")
    assert_parity(tw.grad.numpy(), gw, rel(dtype), "gw")
    assert_parity(tb.grad.numpy(), gb, rel(dtype), "gb")


@pytest.mark.parametrize("cols", [16, 128, 768, 1000])
def test_layer_norm(dtype, cols):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(cols)
    x = rng.standard_normal((3, 37, cols)) * 3 + 1
    w, b = 1 + 0.1 * rng.standard_normal(cols), 0.1 * rng.standard_normal(cols)
    g = rng.standard_normal(x.shape)
    tx, tw, tb = tensor(x, dtype), tensor(w, dtype), tensor(b, dtype)
    y = tg.layer_norm(tx, tw, tb)
    y.backward(g.astype(dtype))
    ref, xhat, rstd = O.layer_norm_forward(x, w, b)
    gx, gw, gb = O.layer_norm_backward(g, xhat, rstd, w)
    assert_parity(y.numpy(), ref, rel(dtype), "y")
    assert_parity(tx.grad.numpy(), gx, rel(dtype), "gx")
    assert_parity(tw.grad.numpy(), gw, rel(dtype), "gw")
    assert_parity(tb.grad.numpy(), gb, rel(dtype), "gb")


def test_gelu_and_relu(dtype):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(2)
    x = rng.standard_normal((5, 203)) * 3
    g = rng.standard_normal(x.shape)
    tx = tensor(x, dtype)
    y = tg.gelu(tx)
    y.backward(g.astype(dtype))
    ref, t = O.gelu_forward(x)
    assert_parity(y.numpy(), ref, rel(dtype), "gelu")
    assert_parity(tx.grad.numpy(), O.gelu_backward(g, x, t), rel(dtype), "gelu grad")
    assert float(tg.gelu(tg.Tensor(np.array(1.0))).item()) == pytest.approx(0.841192, abs=1e-6)
    tr = tensor(x, dtype)
    yr = tg.relu(tr)
    yr.backward(g.astype(dtype))
    assert_parity(yr.numpy(), O.relu_forward(x), rel(dtype), "relu")
    assert_parity(tr.grad.numpy(), O.relu_backward(g, x), rel(dtype), "relu grad")


@pytest.mark.parametrize("vocab", [1, 5, 300])
def test_embedding_scatter_add(dtype, vocab):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(vocab)
    ids = rng.integers(0, vocab, size=(7, 11))
    w = rng.standard_normal((vocab, 3))
    g = rng.standard_normal((7, 11, 3))
    tw = tensor(w, dtype)
    out = tg.embedding(ids, tw)
    out.backward(g.astype(dtype))
    assert_parity(out.numpy(), w[ids], rel(dtype), "gather")
    assert_parity(tw.grad.numpy(), O.embedding_backward(ids, g, vocab), rel(dtype), "scatter")


@pytest.mark.parametrize("vocab,shape", [(5, (7, 11)), (65, (32, 128)), (50304, (3, 1000))])
def test_embedding_device_ids(dtype, vocab, shape):
    """Device-resident ids: gather checked on the device, the VJP's stable order sorted on the
    device; the gradient equals the oracle's (same order of summation per row) and the result
    of the host-id path bit for bit."""
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(vocab + shape[1])
    ids = rng.integers(0, vocab, size=shape)
    ids[0, :5] = ids[0, 0]  # a run of equal ids
    dim = 8
    w = rng.standard_normal((vocab, dim))
    g = rng.standard_normal((*shape, dim))
    tw = tensor(w, dtype)
    out = tg.embedding(tg.Tensor(ids), tw)
    out.backward(g.astype(dtype))
    assert np.array_equal(out.numpy(), w.astype(dtype)[ids])
    assert_parity(tw.grad.numpy(), O.embedding_backward(ids, g, vocab), rel(dtype), "scatter")
    tw_host = tensor(w, dtype)
    tg.embedding(ids, tw_host).backward(g.astype(dtype))
    assert np.array_equal(tw.grad.numpy(), tw_host.grad.numpy())


def test_device_ids_and_targets_out_of_range_raise_at_sync():
    import tensorgrad_b200 as tg

    w = tg.Tensor(np.arange(12.0).reshape(4, 3))
    out = tg.embedding(tg.Tensor(np.array([1, 4])), w)  # id 4 is out of range: a zero row
    with pytest.raises(IndexError, match="embedding ids"):
        out.numpy()
    assert np.array_equal(tg.embedding(tg.Tensor(np.array([1, 2])), w).numpy(),
                          np.arange(12.0).reshape(4, 3)[[1, 2]])
    loss = tg.cross_entropy(tg.Tensor(np.zeros((2, 3))), tg.Tensor(np.array([0, 3])))
    with pytest.raises(IndexError, match="target out of range"):
        loss.item()
    ok = tg.cross_entropy(tg.Tensor(np.zeros((2, 3))), tg.Tensor(np.array([0, 2])))
    assert ok.item() == pytest.approx(np.log(3.0))


def test_embedding_rejects_bad_ids():
    import tensorgrad_b200 as tg

    w = tg.Tensor(np.arange(12.0).reshape(4, 3))
    for bad in (-1, 4):
        with pytest.raises(IndexError, match="embedding ids"):
            tg.embedding(np.array([bad]), w)
    with pytest.raises(TypeError, match="integers"):
        tg.embedding(np.array([0.5]), w)


@pytest.mark.parametrize("classes", [4, 65, 50304])
def test_cross_entropy(dtype, classes):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(classes)
    rows = 37 if classes > 1000 else 300
    logits = rng.standard_normal((rows, classes)) * 2
    target = rng.integers(0, classes, size=rows)
    target[::7] = -100
    tl = tensor(logits, dtype)
    loss = tg.cross_entropy(tl, target)
    loss.backward()
    ref, logp = O.cross_entropy_forward(logits, target)
    assert float(loss.item()) == pytest.approx(float(ref), rel=rel(dtype))
    assert_parity(tl.grad.numpy(), O.cross_entropy_backward(1.0, logp, target, logits.shape),
                  rel(dtype), "ce grad")
    for red in ("sum", "none"):
        out = tg.cross_entropy(tensor(logits, dtype, False), target, reduction=red)
        refr, _ = O.cross_entropy_forward(logits, target, reduction=red)
        assert_parity(out.numpy(), refr, rel(dtype), f"ce {red}")


def test_cross_entropy_all_ignored_and_bad_target():
    import tensorgrad_b200 as tg

    out = tg.cross_entropy(tg.Tensor(np.zeros((2, 3))), np.array([7, 7]), ignore_index=7)
    assert out.item() == 0.0
    with pytest.raises(IndexError, match="target out of range"):
        tg.cross_entropy(tg.Tensor(np.zeros((2, 3))), np.array([0, 3]))


def test_cross_entropy_device_targets(dtype):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(5)
    logits = rng.standard_normal((300, 65)) * 2
    target = rng.integers(0, 65, size=300)
    target[::7] = -100
    tl = tensor(logits, dtype)
    loss = tg.cross_entropy(tl, tg.Tensor(target))
    loss.backward()
    ref, logp = O.cross_entropy_forward(logits, target)
    assert float(loss.item()) == pytest.approx(float(ref), rel=rel(dtype))
    assert_parity(tl.grad.numpy(), O.cross_entropy_backward(1.0, logp, target, logits.shape),
                  rel(dtype), "ce grad")


def test_embedding_backward_from_host_segments():
    """``tg_embedding_backward`` (the scatter-add in the order of a host-side stable argsort,
    for FFI hosts that sort themselves) against NumPy's ``add.at``; the package's own VJP sorts
    on the device and is covered by the GPT parity tests."""
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F32, F64, check, lib

    rng = np.random.default_rng(21)
    ids = rng.integers(0, 7, size=40)
    for np_dt, code, tol in ((np.float32, F32, 1e-6), (np.float64, F64, 1e-14)):
        g = rng.standard_normal((40, 5)).astype(np_dt)
        order = np.argsort(ids, kind="stable")
        sorted_ids = ids[order]
        starts = np.flatnonzero(np.concatenate(([True], sorted_ids[1:] != sorted_ids[:-1])))
        seg_start = np.append(starts, ids.size).astype(np.int64)
        seg_id = sorted_ids[starts].astype(np.int64)
        dg, d_order = device.from_numpy(g), device.from_numpy(order.astype(np.int64))
        d_start, d_id = device.from_numpy(seg_start), device.from_numpy(seg_id)
        gw = device.empty((7, 5), np_dt)
        check(lib.tg_embedding_backward(code, dg.ptr, d_order.ptr, d_start.ptr, d_id.ptr,
                                        seg_id.size, gw.ptr, 7, 5, 0, device.stream()))
        ref = np.zeros((7, 5))
        np.add.at(ref, ids, g.astype(np.float64))
        assert_parity(gw.numpy(), ref, tol, f"segment scatter-add {np.dtype(np_dt).name}")


# ------------------------------------------------------------------------------- attention
@pytest.mark.parametrize("shape,causal,seed", ATTN_CASES)
def test_attention_matches_reference_fixture(dtype, shape, causal, seed):
    import tensorgrad_b200 as tg

    gold = load_golden("attention.npz")
    key = "x".join(map(str, shape)) + ("_causal" if causal else "")
    q, k, v, do = attention_inputs(shape, seed)
    tq, tk, tv = (tensor(a, dtype) for a in (q, k, v))
    o = tg.nn.functional.scaled_dot_product_attention(tq, tk, tv, causal=causal)
    dq, dk, dv = tg.autograd.grad(o, [tq, tk, tv], grad_outputs=do.astype(dtype))
    for name, ours in (("out", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        assert_parity(ours.numpy(), gold[f"{key}/{name}"], rel(dtype), f"{key} {name}")


def test_attention_causal_with_longer_keys(dtype):
    # Causal with tk > tq (query i sees keys j <= i + tk - tq): the CUDA-core path.
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(9)
    q, k, v = (rng.standard_normal(s) for s in ((1, 2, 5, 16), (1, 2, 9, 16), (1, 2, 9, 16)))
    do = rng.standard_normal((1, 2, 5, 16))
    tq, tk, tv = (tensor(a, dtype) for a in (q, k, v))
    o = tg.nn.functional.scaled_dot_product_attention(tq, tk, tv, causal=True)
    dq, dk, dv = tg.autograd.grad(o, [tq, tk, tv], grad_outputs=do.astype(dtype))
    ref_o, p = O.attention_forward(q, k, v, True)
    for ours, ref, name in zip((o, dq, dk, dv), (ref_o, *O.attention_backward(do, q, k, v, p)),
                               ("out", "dq", "dk", "dv"), strict=True):
        assert_parity(ours.numpy(), ref, rel(dtype), name)


# Heads of 32 and 64 features take the fused forward (scores only in tensor memory): ragged
# lengths, more keys than queries, both masks, against the float64 oracle.
@pytest.mark.parametrize("qshape,tk,causal", [((2, 3, 150, 64), 150, False),
                                              ((1, 2, 70, 64), 130, False),
                                              ((1, 2, 97, 32), 97, False),
                                              ((2, 2, 1, 64), 1, True),
                                              ((1, 3, 257, 64), 257, True)])
def test_fused_attention_forward_shapes(dtype, qshape, tk, causal):
    import tensorgrad_b200 as tg
    from tensorgrad_b200._lib import lib

    rng = np.random.default_rng(qshape[2] + tk)
    b, h, tq, d = qshape
    q, k, v = (rng.standard_normal(s) for s in (qshape, (b, h, tk, d), (b, h, tk, d)))
    do = rng.standard_normal(qshape)
    tq_, tk_, tv_ = (tensor(a, dtype) for a in (q, k, v))
    o = tg.nn.functional.scaled_dot_product_attention(tq_, tk_, tv_, causal=causal)
    dq, dk, dv = tg.autograd.grad(o, [tq_, tk_, tv_], grad_outputs=do.astype(dtype))
    ref_o, p = O.attention_forward(q, k, v, causal)
    refs = (ref_o, *O.attention_backward(do, q, k, v, p))
    assert lib.tg_attention_tc_status(1) == 0  # no bounded wait of the fused kernels expired
    for ours, ref, name in zip((o, dq, dk, dv), refs, ("out", "dq", "dk", "dv"), strict=True):
        if np.max(np.abs(ref)) == 0.0:
            # A single visible key: softmax is 1 whatever the scores, dq = dk = 0 exactly;
            # both sides hold only rounding noise of dP - delta, checked against the scale
            # of the value gradient.
            assert_zero_gradient(ours.numpy(), float(np.max(np.abs(refs[3]))), rel(dtype), name)
        else:
            assert_parity(ours.numpy(), ref, rel(dtype), name)


# Head sizes without kernels of their own take the next wider CUDA-core kernel over
# zero-padded copies (fp32 heads of a multiple of 4 features with tq == tk stay on the
# tensor-core path).
@pytest.mark.parametrize("qshape,tk,causal", [((1, 2, 7, 6), 7, True),
                                              ((2, 1, 9, 12), 11, False),
                                              ((1, 2, 5, 4), 8, True),
                                              ((1, 1, 13, 100), 13, True),
                                              ((2, 2, 6, 3), 6, False),
                                              ((1, 1, 5, 200), 7, True),
                                              ((1, 2, 9, 256), 9, False)])
def test_attention_other_head_sizes(dtype, qshape, tk, causal):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(qshape[3] + tk)
    b, h, tq, d = qshape
    q, k, v = (rng.standard_normal(s) for s in (qshape, (b, h, tk, d), (b, h, tk, d)))
    do = rng.standard_normal(qshape)
    tq_, tk_, tv_ = (tensor(a, dtype) for a in (q, k, v))
    o = tg.nn.functional.scaled_dot_product_attention(tq_, tk_, tv_, causal=causal)
    dq, dk, dv = tg.autograd.grad(o, [tq_, tk_, tv_], grad_outputs=do.astype(dtype))
    ref_o, p = O.attention_forward(q, k, v, causal)
    for ours, ref, name in zip((o, dq, dk, dv), (ref_o, *O.attention_backward(do, q, k, v, p)),
                               ("out", "dq", "dk", "dv"), strict=True):
        assert_parity(ours.numpy(), ref, rel(dtype), name)


@pytest.mark.parametrize("b,t,h,hd", [(2, 64, 4, 32), (1, 129, 2, 64), (2, 40, 3, 16),
                                      (1, 70, 1, 128), (2, 300, 2, 64), (2, 9, 3, 6)])
def test_packed_self_attention(dtype, b, t, h, hd):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(t + h)
    qkv = rng.standard_normal((b, t, 3 * h * hd))
    g = rng.standard_normal((b, t, h * hd))
    tq = tensor(qkv, dtype)
    y = tg.nn.functional.packed_self_attention(tq, h)
    y.backward(g.astype(dtype))
    ref, p = O.packed_self_attention_forward(qkv, h)
    assert_parity(y.numpy(), ref, rel(dtype), "y")
    assert_parity(tq.grad.numpy(), O.packed_self_attention_backward(g, qkv, p, h), rel(dtype),
                  "dqkv")


# ------------------------------------------------------------------------------- optimiser
def test_clip_and_adamw_match_reference(dtype):
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(3)
    shapes = [(17, 5), (64,), (3, 3, 3), (1000,)]
    ps = [rng.standard_normal(s) for s in shapes]
    gs = [rng.standard_normal(s) * 0.3 for s in shapes]
    params = [tg.nn.Parameter(p.astype(dtype)) for p in ps]
    opt = tg.optim.AdamW(params, lr=1e-2, weight_decay=0.1)
    ref_p, ref_m, ref_v = list(ps), [np.zeros_like(p) for p in ps], [np.zeros_like(p) for p in ps]
    for step in (1, 2, 3):
        for p, g in zip(params, gs, strict=True):
            p.grad = g.astype(dtype) * step
        total = tg.optim.clip_grad_norm_(params, 1.5)
        ref_total, clipped = O.clip_grad_norm([g * step for g in gs], 1.5)
        assert total == pytest.approx(ref_total, rel=rel(dtype))
        for p, c in zip(params, clipped, strict=True):
            assert_parity(p.grad.numpy(), c, rel(dtype), "clipped grad")
        opt.step()
        for i in range(len(ps)):
            ref_p[i], ref_m[i], ref_v[i] = O.adamw_update(ref_p[i], clipped[i], ref_m[i],
                                                          ref_v[i], step, 1e-2, (0.9, 0.999),
                                                          1e-8, 0.1)
        for p, r in zip(params, ref_p, strict=True):
            assert_parity(p.numpy(), r, rel(dtype), f"param step {step}")


def test_fused_clip_and_adamw_equal_the_separate_passes(dtype):
    # clip_grad_norm_ on a flat arena leaves its rescale pending and AdamW applies it inside
    # its update pass; reading the gradients before the step writes the rescale first. Both
    # orders must give the same parameters, moments and gradients bit for bit, and match the
    # float64 reference.
    import tensorgrad_b200 as tg

    rng = np.random.default_rng(31)
    shapes = [(33, 7), (128,), (5, 4, 3)]
    ps = [rng.standard_normal(s) for s in shapes]
    gs = [rng.standard_normal(s) for s in shapes]
    runs = []
    for read_grads_first in (True, False):
        params = [tg.nn.Parameter(p.astype(dtype)) for p in ps]
        opt = tg.optim.AdamW(params, lr=1e-2, weight_decay=0.1)
        for step in (1, 2):
            opt.zero_grad()
            for p, g in zip(params, gs, strict=True):
                # Accumulate through the engine, as a backward pass does.
                p._accumulate_grad(tg.Tensor(g.astype(dtype) * step).data)
            total = tg.optim.clip_grad_norm_(params, 0.5)
            grads = [p.grad.numpy() for p in params] if read_grads_first else None
            opt.step()
            if not read_grads_first:
                grads = [p.grad.numpy() for p in params]
        runs.append((total, grads, [p.numpy() for p in params]))
    (t1, g1, p1), (t2, g2, p2) = runs
    assert t1 == t2
    for a, b in zip(g1 + p1, g2 + p2, strict=True):
        np.testing.assert_array_equal(a, b)
    ref_p = list(ps)
    ref_m, ref_v = [np.zeros_like(p) for p in ps], [np.zeros_like(p) for p in ps]
    for step in (1, 2):
        _, clipped = O.clip_grad_norm([g * step for g in gs], 0.5)
        for i in range(len(ps)):
            ref_p[i], ref_m[i], ref_v[i] = O.adamw_update(ref_p[i], clipped[i], ref_m[i],
                                                          ref_v[i], step, 1e-2, (0.9, 0.999),
                                                          1e-8, 0.1)
    for got, ref in zip(p2, ref_p, strict=True):
        assert_parity(got, ref, rel(dtype), "params after fused clip + AdamW")
    for got, ref in zip(g2, clipped, strict=True):
        assert_parity(got, ref, rel(dtype), "clipped gradients read after the step")


def test_adam_state_is_per_parameter():
    import tensorgrad_b200 as tg

    a, b = tg.nn.Parameter(np.ones(1)), tg.nn.Parameter(np.ones(1))
    opt = tg.optim.Adam([a, b], lr=0.1)
    a.grad = np.array([1.0], dtype=np.float32)
    opt.step()
    assert b.numpy()[0] == 1.0
    assert len(opt.state) == 1
    np.testing.assert_allclose(a.numpy(), [0.9], rtol=1e-6)


def test_library_status_codes_raise_reference_exceptions():
    from tensorgrad_b200._lib import check, lib

    buf = ctypes.create_string_buffer(64)
    assert lib.tg_last_error(buf, 64) == 0
    with pytest.raises(ValueError):
        check(lib.tg_layer_norm_forward(0, None, None, None, None, None, None, 4, 0, 1e-5, None))


def test_tensor_core_tf32_input_conversion_and_plain_tf32_mode():
    """Plain TF32 mode (tg_set_matmul_precision(1)) and how the tensor core converts fp32
    inputs to TF32. The default 3xTF32 split clears hi's low 13 bits itself, so it does not
    depend on the conversion; this records it."""
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import F32, check, lib

    ulp = 2.0**-10
    xs = np.array([1 + 0.75 * ulp, 1 + 0.5 * ulp, 1 + 1.5 * ulp, -(1 + 0.75 * ulp)] * 32)
    m, k, n = xs.size, 16, 128  # k > 8: the tensor-core kernel, not the small-k one
    a = np.zeros((m, k), np.float32)
    a[:, 0] = xs
    b = np.zeros((k, n), np.float32)
    b[0, :] = 1.0
    da, db, dc = device.from_numpy(a), device.from_numpy(b), device.empty((m, n), np.float32)
    check(lib.tg_set_matmul_precision(1))
    try:
        check(lib.tg_gemm(F32, 0, 0, m, n, k, 1.0, da.ptr, k, db.ptr, n, 0.0, dc.ptr, n, None,
                          device.stream()))
        got = dc.numpy()[:, 0].astype(np.float64)
    finally:
        check(lib.tg_set_matmul_precision(0))
    x32 = xs.astype(np.float32)
    trunc = (x32.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32).astype(np.float64)
    rne = np.array([np.float64(np.float32(v)) for v in xs])  # placeholder, replaced below
    q = np.abs(xs) / ulp
    rne = np.sign(xs) * ulp * np.where(np.abs(q - np.floor(q) - 0.5) < 1e-12,
                                       np.where(np.floor(q) % 2 == 0, np.floor(q), np.ceil(q)),
                                       np.round(q))
    rna = np.sign(xs) * ulp * np.floor(q + 0.5)
    modes = {"truncate": trunc, "nearest-even": rne, "nearest-away": rna}
    matched = [name for name, v in modes.items() if np.array_equal(got, v)]
    print("tensor-core fp32->tf32 conversion:", matched)
    assert matched, f"TF32 conversion matches no known rounding: {got[:4]}"


def test_fma_pipe_exponential_error_bound():
    """The exponential the fused attention kernels compute on the FMA pipe for part of their
    softmax numerators: within 3e-7 relative of exp in float64 over [-87, 8] (the reduction
    x - n ln2 is exact, the fitted polynomial ~8e-8), NaN stays NaN, and exactly 0 below
    -87.3 (e^x < 2^-126) and for -inf."""
    from tensorgrad_b200 import device
    from tensorgrad_b200._lib import check, lib

    x = np.concatenate([np.linspace(-87.0, 8.0, 400001), [0.0, -0.0, 1e-30, -1e-30]])
    x32 = x.astype(np.float32)
    dx, dy = device.from_numpy(x32), device.empty(x32.shape, np.float32)
    check(lib.tg_test_exp_fma(x32.size, dx.ptr, dy.ptr, device.stream()))
    got = dy.numpy().astype(np.float64)
    rel = np.abs(got / np.exp(x32.astype(np.float64)) - 1.0)
    assert rel.max() <= 3e-7, f"max relative error {rel.max()} at {x32[np.argmax(rel)]}"
    tail = np.array([-np.inf, -87.31, -88.5, -100.0, -1e30, np.nan], dtype=np.float32)
    dt, dz = device.from_numpy(tail), device.empty(tail.shape, np.float32)
    check(lib.tg_test_exp_fma(tail.size, dt.ptr, dz.ptr, device.stream()))
    z = dz.numpy()
    assert np.all(z[:5] == 0.0) and np.isnan(z[5])
