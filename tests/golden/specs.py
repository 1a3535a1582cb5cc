"""Seeds and shapes of the golden fixtures, shared by ``make_golden.py`` and the tests."""

from __future__ import annotations

import numpy as np

from oracle import cnn as ocnn
from oracle import gpt as ogpt

#: Small GPT used for the committed fixture (all code paths of the char-GPT config). Its
#: ``max_norm`` sits below the gradient norm so that clipping is exercised.
GPT_SMALL = dict(cfg=ogpt.Config(vocab_size=65, block_size=16, n_layer=2, n_head=2, n_embd=16),
                 batch=4, seq=16, seed=0, max_norm=0.5, steps=2)
#: The same GPT trained with dropout 0.1 everywhere the reference applies it (embeddings,
#: attention weights, the attention projection and the MLP output), the global generator
#: re-seeded right after the weights are loaded so the masks start from a known state.
GPT_DROPOUT = dict(GPT_SMALL, dropout=0.1, reseed=4321)
#: (shape, p, seed) of the keep-mask fixtures: odd sizes (a partial last 64-bit draw), a
#: common rate, and a rate that rounds to "drop everything" (no draw at all).
DROPOUT_CASES = [((7, 13), 0.1, 1), ((3, 5, 4), 0.5, 2), ((10,), 0.99999999, 3)]
#: ((B, H, T, d), causal, seed) of the attention fixtures.
ATTN_CASES = [((2, 2, 24, 8), True, 1), ((1, 3, 17, 16), False, 2), ((2, 1, 33, 32), True, 3)]


def attention_inputs(shape: tuple[int, int, int, int], seed: int) -> list[np.ndarray]:
    """``q, k, v, dO`` ~ N(0, 1) from ``seed`` (the MHA-alone config's distribution)."""
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(shape) for _ in range(4)]


#: Small CNN (the CNN config's layer stack at 8x8 inputs) for the committed fixture.
CNN_SMALL = dict(cfg=ocnn.Config(in_channels=3, size=8, c1=4, c2=6, classes=4), batch=4, seed=5,
                 steps=2)

#: Op-level conv / pool cases: (x shape, (c_out, kh, kw), stride, padding, seed) and
#: (x shape, kernel, stride, padding, seed). The pool cases include overlapping windows and
#: -inf padding; ties and a NaN are planted by ``pool_input``.
CONV_CASES = [((2, 3, 9, 7), (4, 3, 2), (2, 1), (1, 0), 11), ((1, 2, 5, 5), (3, 1, 1), (1, 1), (0, 0), 12),
              ((2, 5, 6, 6), (2, 3, 3), (1, 1), (1, 1), 13)]
POOL_CASES = [((2, 3, 8, 8), (2, 2), (2, 2), (0, 0), 21), ((1, 2, 7, 9), (3, 3), (2, 2), (1, 1), 22),
              ((2, 1, 6, 5), (3, 2), (1, 1), (1, 1), 23)]


def conv_inputs(x_shape, wspec, seed):
    """``x, w, b`` ~ N(0, 1) for a conv case, and the generator that then draws the output
    gradient."""
    rng = np.random.default_rng(seed)
    c_out, kh, kw = wspec
    x = rng.standard_normal(x_shape)
    w = rng.standard_normal((c_out, x_shape[1], kh, kw))
    b = rng.standard_normal(c_out)
    return x, w, b, rng


def pool_input(x_shape, seed):
    """Values on a coarse grid (so windows hold ties) with one NaN."""
    rng = np.random.default_rng(seed)
    x = np.round(rng.standard_normal(x_shape) * 2) / 2
    x.reshape(-1)[x.size // 3] = np.nan
    return x, rng


#: Parameters of the CNN whose gradient is exactly zero: the convolution biases, each followed
#: by a batch norm.
CNN_ZERO_GRAD = {"0.bias": "0.weight", "4.bias": "4.weight"}


#: Op-level recurrent cases: (cell, T, B, I, H, seed).
RNN_CASES = [("lstm", 7, 3, 2, 5, 31), ("gru", 7, 3, 2, 5, 32), ("lstm", 4, 2, 3, 8, 33),
             ("gru", 5, 4, 6, 4, 34)]
#: The adding-problem regressors (LSTM and GRU, hidden 8, T = 12, batch 6), two AdamW steps.
RNN_SMALL = dict(hidden=8, seq=12, batch=6, seed=41, steps=2)


def rnn_inputs(cell, steps, batch, inputs, hidden, seed):
    """``x, h0, c0, w_ih, w_hh, b_ih, b_hh`` ~ N(0, 0.5) and the generator that then draws the
    output gradient (``c0`` is None for the GRU)."""
    rng = np.random.default_rng(seed)
    gates = 4 if cell == "lstm" else 3
    x = rng.standard_normal((steps, batch, inputs))
    h0 = 0.5 * rng.standard_normal((batch, hidden))
    c0 = 0.5 * rng.standard_normal((batch, hidden)) if cell == "lstm" else None
    w_ih = 0.5 * rng.standard_normal((gates * hidden, inputs))
    w_hh = 0.5 * rng.standard_normal((gates * hidden, hidden))
    b_ih = 0.5 * rng.standard_normal(gates * hidden)
    b_hh = 0.5 * rng.standard_normal(gates * hidden)
    return x, h0, c0, w_ih, w_hh, b_ih, b_hh, rng


def higher_order_inputs() -> dict[str, np.ndarray]:
    """Seeded float64 inputs of the differentiable-gradient fixture (higher_order.npz)."""
    rng = np.random.default_rng(61)
    return {
        "x": rng.standard_normal((3, 4)), "w": rng.standard_normal((4, 2)),
        "v": rng.standard_normal((3, 4)), "vw": rng.standard_normal((4, 2)),
        "c": rng.standard_normal((3, 4)),
        "xin": rng.standard_normal((5, 6)), "labels": rng.integers(0, 3, size=5),
        "w1": 0.5 * rng.standard_normal((7, 6)), "b1": 0.1 * rng.standard_normal(7),
        "w2": 0.5 * rng.standard_normal((3, 7)), "b2": 0.1 * rng.standard_normal(3),
    }


#: The GPT of GPT_DROPOUT trained one step on ``loss + penalty * sum(grad^2)``: a gradient
#: penalty that differentiates every op of the model twice (embedding, dropout, layer norm,
#: packed attention with dropout, GELU, the head and cross entropy).
GPT_PENALTY = dict(GPT_DROPOUT, penalty=0.01)


def higher_order_layer_inputs() -> dict[str, np.ndarray]:
    """Seeded float64 inputs of the second-order fixture of the fused layers
    (higher_order_layers.npz)."""
    rng = np.random.default_rng(83)
    n = rng.standard_normal
    return {
        "ln_x": n((4, 6)), "ln_w": 1.0 + 0.1 * n(6), "ln_b": 0.1 * n(6), "ln_c": n((4, 6)),
        "ln_vx": n((4, 6)), "ln_vw": n(6), "var_x": n((3, 5)),
        "q": n((2, 2, 5, 4)), "k": n((2, 2, 5, 4)), "v": n((2, 2, 5, 4)),
        "attn_c": n((2, 2, 5, 4)), "vq": n((2, 2, 5, 4)), "vk": n((2, 2, 5, 4)),
        "vv": n((2, 2, 5, 4)),
        "qkv": n((2, 5, 24)), "qkv_c": n((2, 5, 8)), "qkv_v": n((2, 5, 24)),
        "cx": n((2, 3, 7, 7)), "cw": 0.3 * n((4, 3, 3, 3)), "cb": 0.1 * n(4),
        "bn_w": 1.0 + 0.1 * n(4), "bn_b": 0.1 * n(4), "cc": n((2, 4, 4, 4)),
        "cx2": n((2, 3, 8, 8)), "cc2": n((2, 4, 2, 2)),
        "ids": rng.integers(0, 10, size=(3, 5)), "targets": rng.integers(0, 4, size=(3, 5)),
        "emb": n((10, 6)), "head": 0.5 * n((4, 6)), "v_emb": n((10, 6)), "v_head": n((4, 6)),
        "rx": n((4, 2, 3)), "rh0": 0.5 * n((2, 5)), "rc0": 0.5 * n((2, 5)),
        "r_vx": n((4, 2, 3)),
        "l_wih": 0.4 * n((20, 3)), "l_whh": 0.4 * n((20, 5)), "l_bih": 0.1 * n(20),
        "l_bhh": 0.1 * n(20), "l_c": n((4, 2, 2, 5)), "l_vw": n((20, 5)),
        "g_wih": 0.4 * n((15, 3)), "g_whh": 0.4 * n((15, 5)), "g_bih": 0.1 * n(15),
        "g_bhh": 0.1 * n(15), "g_c": n((4, 2, 5)), "g_vw": n((15, 5)),
        "d_x": n((6, 7)), "d_c": n((6, 7)), "d_v": n((6, 7)),
    }


def higher_order_layer_program(tg, O, func, host, d: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Second derivatives through each fused layer, written once for both implementations:
    ``tg`` is the package, ``O`` a namespace of its ops (tanh, relu, layer_norm, var, sdpa,
    packed, conv2d, batch_norm, max_pool2d, embedding, linear, cross_entropy, lstm, gru,
    dropout), ``func`` its function transforms and ``host(t)`` a tensor's values as an array.
    Hessian-vector products of scalar functions of each layer, and gradient penalties
    (``loss + sum(d loss / dx ** 2)`` differentiated to the parameters) through the CNN layers."""
    T = tg.Tensor
    out: dict[str, np.ndarray] = {}

    def hvp(name: str, f, primals, tangents, keys) -> None:
        _, hs = func.hvp(f, [T(d[p]) for p in primals], [T(d[t]) for t in tangents])
        for k, h in zip(keys, hs, strict=True):
            out[f"{name}_hvp_{k}"] = host(h)

    hvp("ln", lambda x, w: (O.tanh(O.layer_norm(x, w, T(d["ln_b"]))) * T(d["ln_c"])).sum(),
        ("ln_x", "ln_w"), ("ln_vx", "ln_vw"), ("x", "w"))
    out["var_hess"] = host(func.hessian(lambda x: (O.var(x, axis=1) ** 2).sum())(T(d["var_x"])))

    def attention(p: float, causal: bool):
        def f(q, k, v):
            rng = np.random.default_rng(71) if p else None
            y = O.sdpa(q, k, v, causal=causal, dropout_p=p, training=p > 0, rng=rng)
            return (O.tanh(y) * T(d["attn_c"])).sum()
        return f

    for name, p, causal in (("attn", 0.0, True), ("attn_full", 0.0, False),
                            ("attn_drop", 0.25, True)):
        hvp(name, attention(p, causal), ("q", "k", "v"), ("vq", "vk", "vv"), ("q", "k", "v"))

    def packed(qkv):
        y = O.packed(qkv, 2, causal=True, dropout_p=0.25, training=True,
                     rng=np.random.default_rng(72))
        return (O.tanh(y) * T(d["qkv_c"])).sum()

    hvp("packed", packed, ("qkv",), ("qkv_v",), ("qkv",))

    def cnn_penalty(name: str, x: str, c: str, conv: tuple[int, int], pool: tuple[int, ...]):
        ts = [T(d[k], requires_grad=True) for k in (x, "cw", "cb", "bn_w", "bn_b")]
        xs, w, b, bw, bb = ts
        h = O.conv2d(xs, w, b, stride=conv[0], padding=conv[1])
        h = O.batch_norm(h, None, None, bw, bb, training=True)
        h = O.max_pool2d(O.relu(h), pool[0], pool[1], pool[2])
        loss = (O.tanh(h) * T(d[c])).sum()
        (gx,) = tg.autograd.grad(loss, [xs], create_graph=True)
        total = loss + (gx * gx).sum()
        total.backward()
        out[f"{name}_total"] = np.asarray(host(total))
        for k, t in zip(("x", "w", "b", "bn_w", "bn_b"), ts, strict=True):
            out[f"{name}_grad_{k}"] = host(t.grad)

    cnn_penalty("cnn", "cx", "cc", (1, 1), (3, 2, 1))
    cnn_penalty("cnn2", "cx2", "cc2", (2, 1), (2, 2, 0))

    def lm(e, w):
        logits = O.linear(O.layer_norm(O.embedding(d["ids"], e)), w)
        return O.cross_entropy(logits, d["targets"])

    hvp("emb", lm, ("emb", "head"), ("v_emb", "v_head"), ("emb", "head"))

    def lstm(x, w_hh):
        y = O.lstm(x, T(d["rh0"]), T(d["rc0"]), T(d["l_wih"]), w_hh, T(d["l_bih"]),
                   T(d["l_bhh"]))
        return (O.tanh(y) * T(d["l_c"])).sum()

    def gru(x, w_hh):
        y = O.gru(x, T(d["rh0"]), T(d["g_wih"]), w_hh, T(d["g_bih"]), T(d["g_bhh"]))
        return (O.tanh(y) * T(d["g_c"])).sum()

    hvp("lstm", lstm, ("rx", "l_whh"), ("r_vx", "l_vw"), ("x", "w_hh"))
    hvp("gru", gru, ("rx", "g_whh"), ("r_vx", "g_vw"), ("x", "w_hh"))

    def dropped(x):
        y = O.dropout(x, 0.3, True, np.random.default_rng(9))
        return (O.tanh(y) * T(d["d_c"])).sum()

    hvp("dropout", dropped, ("d_x",), ("d_v",), ("x",))
    return out


def gpt_penalty_program(tg, nn, host, spec: dict) -> dict[str, np.ndarray]:
    """One GPT_PENALTY step: ``loss + penalty * sum over parameters of sum(grad ** 2)``,
    differentiated to every parameter (the gradients built with ``create_graph``)."""
    cfg = spec["cfg"]
    model = nn.GPT(nn.GPTConfig(vocab_size=cfg.vocab_size, block_size=cfg.block_size,
                                n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd,
                                dropout=spec["dropout"]))
    init = ogpt.init_params(cfg, spec["seed"])
    model.load_state_dict({**init, "head.weight": init["tok_emb.weight"]})
    tg.manual_seed(spec["reseed"])
    names = [n for n, _ in model.named_parameters()]
    params = list(model.parameters())
    ids, targets = ogpt.synthetic_batch(cfg, spec["batch"], spec["seq"], spec["seed"] + 1)
    loss = tg.cross_entropy(model(ids), targets)
    grads = tg.autograd.grad(loss, params, create_graph=True)
    penalty = (grads[0] * grads[0]).sum()
    for g in grads[1:]:
        penalty = penalty + (g * g).sum()
    total = loss + penalty * spec["penalty"]
    total.backward()
    out = {"gpt_loss": np.asarray(host(loss)), "gpt_total": np.asarray(host(total))}
    for n, p in zip(names, params, strict=True):
        out[f"gpt_grad/{n}"] = host(p.grad)
    return out


def ops_extra_inputs() -> dict[str, np.ndarray]:
    """Seeded float64 inputs of the fixture of the remaining ops (ops_extra.npz): the softmax
    family, max / min with ties, where / masked_fill, concat, binary cross entropy, the
    Elman RNN, matmul with vectors, comparisons and all / any / argmax."""
    rng = np.random.default_rng(97)
    n = rng.standard_normal
    masked = n((2, 6))
    masked[0, [1, 4]] = -np.inf
    masked[1, 5] = -np.inf
    z = 3.0 * n(9)
    z[:3] = (0.0, 40.0, -40.0)
    return {
        "s_x": n((3, 5, 4)), "s_g": n((3, 5, 4)), "s_g1": n((3, 4)), "masked": masked,
        "masked_g": n((2, 6)),
        "m_x": rng.integers(0, 3, size=(4, 6)).astype(np.float64), "m_g1": n(4),
        "w_c": rng.random((4, 6)) > 0.5, "w_a": n((4, 6)), "w_b": n(6), "w_g": n((4, 6)),
        "c_a": n((2, 3)), "c_b": n((2, 5)), "c_c": n((2, 1)), "c_g": n((2, 9)),
        "b_z": z, "b_y": rng.random(9), "b_g": n(9),
        "rx": n((5, 2, 3)), "rh0": 0.5 * n((2, 4)), "r_wih": 0.5 * n((4, 3)),
        "r_whh": 0.5 * n((4, 4)), "r_bih": 0.1 * n(4), "r_bhh": 0.1 * n(4), "r_g": n((5, 2, 4)),
        "v1": n(4), "v2": n(4), "mm": n((3, 4)), "bm": n((2, 4, 5)), "mm_g": n(3),
        "bm_g": n((2, 5)),
        "ix": n((5, 4, 3)), "ix_rows": np.array([3, 0, 3, 1]), "ix_mask": rng.random((5, 4)) > 0.4,
        "ix_cols": np.array([2, 0, 2]), "ix_t": rng.integers(0, 4, size=5),
        "aq": n((2, 2, 4, 3)), "ak": n((2, 2, 5, 3)), "av6": n((2, 2, 5, 6)),
        "av3": n((2, 2, 5, 3)), "ag6": n((2, 2, 4, 6)), "ag3": n((2, 2, 4, 3)),
        "amask": np.concatenate([np.zeros((4, 1), bool), rng.random((4, 4)) > 0.7], axis=1),
    }


def ops_extra_program(tg, O, host, d: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Values and VJPs of the remaining ops, written once for both implementations: ``O``
    holds ``rnn`` and ``sdpa`` (scaled_dot_product_attention), everything else is the
    package's top level and Tensor methods; ``host(t)`` a tensor's values as an array."""
    T = tg.Tensor
    out: dict[str, np.ndarray] = {}

    def vjp(name: str, y, xs, g) -> None:
        out[f"{name}/y"] = host(y)
        grads = tg.autograd.grad(y, xs, grad_outputs=T(g) if g is not None else None,
                                 allow_unused=True)
        for i, gr in enumerate(grads):
            out[f"{name}/g{i}"] = np.zeros(xs[i].shape) if gr is None else host(gr)

    x = T(d["s_x"], requires_grad=True)
    vjp("softmax", tg.softmax(x, -1), [x], d["s_g"])
    vjp("softmax_ax1", x.softmax(1), [x], d["s_g"])
    vjp("log_softmax", tg.log_softmax(x, -1), [x], d["s_g"])
    vjp("logsumexp", tg.logsumexp(x, 1), [x], d["s_g1"])
    vjp("logsumexp_keep", tg.logsumexp(x, -1, keepdims=True), [x], d["s_g"][..., :1])
    xm = T(d["masked"], requires_grad=True)
    vjp("softmax_masked", tg.softmax(xm), [xm], d["masked_g"])
    vjp("logsumexp_masked", tg.logsumexp(xm), [xm], d["masked_g"][:, 0])
    m = T(d["m_x"], requires_grad=True)
    vjp("max_ax1", tg.max(m, axis=1), [m], d["m_g1"])
    vjp("min_ax1", m.min(axis=1), [m], d["m_g1"])
    vjp("max_all", m.max(), [m], None)
    vjp("min_all_keep", tg.min(m, keepdims=True), [m], np.ones((1, 1)))
    a, b = T(d["w_a"], requires_grad=True), T(d["w_b"], requires_grad=True)
    vjp("where", tg.where(d["w_c"], a, b), [a, b], d["w_g"])
    vjp("masked_fill", tg.masked_fill(a, d["w_c"], -1.5), [a], d["w_g"])
    vjp("masked_fill_method", a.masked_fill(T(d["w_c"]), 2.0), [a], d["w_g"])
    ca, cb, cc = (T(d[k], requires_grad=True) for k in ("c_a", "c_b", "c_c"))
    vjp("concat", tg.concat([ca, cb, cc], axis=1), [ca, cb, cc], d["c_g"])
    z, y = T(d["b_z"], requires_grad=True), T(d["b_y"], requires_grad=True)
    for red in ("mean", "sum", "none"):
        loss = tg.binary_cross_entropy_with_logits(z, y, reduction=red)
        vjp(f"bce_{red}", loss, [z, y], d["b_g"] if red == "none" else None)
    rnn_in = [T(d[k], requires_grad=True)
              for k in ("rx", "rh0", "r_wih", "r_whh", "r_bih", "r_bhh")]
    for act in ("tanh", "relu"):
        vjp(f"rnn_{act}", O.rnn(*rnn_in, nonlinearity=act), rnn_in, d["r_g"])
    v1, v2 = T(d["v1"], requires_grad=True), T(d["v2"], requires_grad=True)
    mm, bm = T(d["mm"], requires_grad=True), T(d["bm"], requires_grad=True)
    vjp("dot", v1 @ v2, [v1, v2], None)
    vjp("matvec", mm @ v1, [mm, v1], d["mm_g"])
    vjp("vecmat_batched", v1 @ bm, [v1, bm], d["bm_g"])
    ix = T(d["ix"], requires_grad=True)
    rng_g = np.random.default_rng(5)
    for name, index in (("rows", d["ix_rows"]), ("mask", d["ix_mask"]),
                        ("cols_repeat", (slice(None), d["ix_cols"])),
                        ("pairs", (np.arange(5), d["ix_t"])),
                        ("mixed", (d["ix_rows"], slice(1, 3), 0)),
                        ("tensor_rows", T(d["ix_rows"]))):
        y_ix = ix[index]
        vjp(f"index_{name}", y_ix, [ix], rng_g.standard_normal(y_ix.shape))
    aq, ak = T(d["aq"], requires_grad=True), T(d["ak"], requires_grad=True)
    av6, av3 = T(d["av6"], requires_grad=True), T(d["av3"], requires_grad=True)
    vjp("attn_wide_values", O.sdpa(aq, ak, av6), [aq, ak, av6], d["ag6"])
    vjp("attn_mask", O.sdpa(aq, ak, av3, mask=d["amask"]), [aq, ak, av3], d["ag3"])
    vjp("attn_mask_causal", O.sdpa(aq, ak, av3, causal=True, mask=d["amask"]), [aq, ak, av3],
        d["ag3"])
    vjp("attn_mask_dropout", O.sdpa(aq, ak, av3, mask=d["amask"], dropout_p=0.25,
                                    training=True, rng=np.random.default_rng(11)),
        [aq, ak, av3], d["ag3"])
    pa, pb = T(d["w_a"]), T(d["w_b"])
    for op, fn in (("gt", lambda p, q: p > q), ("le", lambda p, q: p <= q),
                   ("eq", lambda p, q: p == q), ("ne_scalar", lambda p, q: p != 0.5)):
        out[f"cmp_{op}"] = host(fn(pa, pb)).astype(np.uint8)
    c = T(d["w_c"])
    out["all_ax0"] = host(c.all(axis=0)).astype(np.uint8)
    out["any_ax1"] = host(c.any(axis=1)).astype(np.uint8)
    out["all"] = np.asarray(host(c.all())).astype(np.uint8)
    out["argmax_ax1"] = host(T(d["m_x"]).argmax(axis=1))
    out["argmax_all"] = np.asarray(host(T(d["m_x"]).argmax()))
    out["argmax_keep"] = host(T(d["w_a"]).argmax(axis=0, keepdims=True))
    return out


#: (op, forward calls, forward seconds, backward calls, backward seconds) of the profiler
#: table fixture (profiler_table.npz).
PROFILE_ROWS = [("matmul", 3, 0.0042, 3, 0.0081), ("autograd engine", 0, 0.0, 1, 0.0011),
                ("softmax", 1, 0.00052, 1, 0.0007), ("cross_entropy", 1, 0.0009, 1, 0.0002)]
