"""Parity of every kernel of the C ABI (include/templit_cuda.h) with the CPU
oracle (oracle/ops.py) and with the reference's known answers, on seeded
inputs, including ragged sizes and the edge cases the reference tests
(empty inputs, out-of-range targets and ids, extreme logits).

Tolerances: fp32 kernels vs the float64 oracle within rtol 1e-5 (the
reference suite's eps 1e-5 / 1e-4 where it states them); integer and index
results bit-exact."""
import ctypes

import numpy as np
import pytest

from oracle import ops
from templit_b200 import capi
from tests.helpers import Dev, known_answers
from tests.test_oracle_golden import compare

pytestmark = pytest.mark.gpu

RTOL = 1e-5


@pytest.fixture(scope="module")
def dev():
    return Dev()


def rng(seed=0):
    return np.random.default_rng(seed)


def close(got, want, rtol=RTOL, atol=None, scale=None):
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64).reshape(want.shape)
    if atol is None:
        atol = rtol * (scale if scale is not None else max(1.0, np.abs(want).max(initial=0)))
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)


# ------------------------------------------------------------ known answers
KERNEL_OPS = {"binary", "scalar", "unary", "rms", "rmsnorm", "matmul", "sum_to_shape",
              "max_to_shape", "transpose", "softmax", "cross_entropy",
              "cross_entropy_derivative", "argmax", "embedding_lookup", "scatter", "adamw",
              "clip"}
CASES = [c for c in known_answers() if c["op"] in KERNEL_OPS]


def kernel_eval(dev, case):
    op, i = case["op"], case["inputs"]
    if op == "binary":
        return dev.binary(i["kind"], np.reshape(i["a"], i["a_shape"]),
                          np.reshape(i["b"], i["b_shape"]), i["out_shape"])
    if op == "scalar":
        return dev.scalar(i["kind"], i["x"], i["s"])
    if op == "unary":
        return dev.unary(i["kind"], i["x"])
    if op in ("rms", "rmsnorm", "softmax"):
        return dev.rows(op, np.reshape(i["x"], i["shape"]))
    if op == "matmul":
        return dev.gemm(np.reshape(i["a"], i["a_shape"]), np.reshape(i["b"], i["b_shape"]))
    if op == "sum_to_shape":
        return dev.reduce("sum", np.reshape(i["x"], i["shape"]), i["out_shape"])
    if op == "max_to_shape":
        return dev.reduce("max", np.reshape(i["x"], i["shape"]), i["out_shape"])
    if op == "transpose":
        return dev.transpose(np.reshape(i["x"], i["shape"]), *i["dims"])
    if op == "cross_entropy":
        z = np.reshape(i["logits"], i["shape"])
        return dev.xent(z, np.reshape(i["targets"], z.shape[:-1]))
    if op == "cross_entropy_derivative":
        z = np.reshape(i["logits"], i["shape"])
        return dev.xent(z, np.reshape(i["targets"], z.shape[:-1]), backward=True)
    if op == "argmax":
        return [dev.argmax(i["x"])]
    if op == "embedding_lookup":
        return dev.gather(np.reshape(i["weights"], i["w_shape"]), i["ids"])
    if op == "scatter":
        base = None if i["base"] is None else np.reshape(i["base"], (i["n_rows"], i["dim"]))
        return dev.scatter(np.reshape(i["values"], (-1, i["dim"])), i["ids"], i["n_rows"], base)
    if op == "clip":
        import ctypes
        grads = [dev.t(g) for g in i["grads"]]
        sq = dev.t([0.0])
        for g in grads:
            nb = dev.lib.tl_grad_sqnorm_workspace_size(g.numel())
            ws = dev.ws(nb)
            dev.call("tl_grad_sqnorm_accumulate", dev.p(g), g.numel(), dev.p(sq), dev.p(ws), nb,
                     dev.stream)
        for g in grads:
            dev.call("tl_clip_gradient", dev.p(g), dev.p(sq), ctypes.c_float(i["max_norm"]),
                     dev.p(g), g.numel(), dev.stream)
        return {"sqnorm": float(dev.host(sq)[0]), "clipped": [dev.host(g) for g in grads]}
    if op == "adamw":
        return adamw_steps(dev, i, 2)
    raise KeyError(op)


def adamw_steps(dev, i, steps):
    import ctypes
    p, g = dev.t(i["param"]), dev.t(i["grad"])
    m1, m2 = dev.t(np.zeros(p.numel())), dev.t(np.zeros(p.numel()))
    lr, wd = i["lr"], i["weight_decay"]
    b1, b2 = dev.t([i["beta1"]]), dev.t([i["beta2"]])
    decay, lrt = dev.t([np.float32(1) - np.float32(lr) * np.float32(wd)]), dev.t([lr])
    out = []
    for step in range(1, steps + 1):
        dev.call("tl_adamw", dev.p(p), dev.p(g), dev.p(p), dev.p(m1), dev.p(m2), dev.p(b1),
                 dev.p(b2), dev.p(decay), dev.p(lrt), ctypes.c_float(i["eps"]), step, p.numel(),
                 dev.stream)
        out.append(dev.host(p).copy())
    return out


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_kernels_match_reference_known_answers(dev, case):
    compare(kernel_eval(dev, case), case)


# ------------------------------------------------------ seeded oracle parity
@pytest.mark.parametrize("shape,bshape", [
    ((64, 192, 384), (64, 192, 384)),   # residual add
    ((64, 192, 384), (1, 384)),         # bias row
    ((64, 6, 192, 192), (1, 1, 192, 192)),  # attention mask
    ((64, 6, 192, 192), (1, 1)),        # score scaling
    ((64, 192, 384), (64, 192, 1)),     # per-row scalar (RMSNorm)
    ((7, 5, 3), (5, 1)),                # ragged, unaligned
    ((3,), (1,)),
])
@pytest.mark.parametrize("kind", ["add", "sub", "mul", "div"])
def test_binary_broadcast(dev, shape, bshape, kind):
    r = rng(1)
    a = r.standard_normal(shape).astype(np.float32)
    b = r.standard_normal(bshape).astype(np.float32)
    if kind == "div":
        b = np.where(np.abs(b) < 0.1, 0.5, b).astype(np.float32)
    got = dev.binary(kind, a, b, shape)
    close(got, ops.broadcast_binary(kind, a, b, shape))
    # the operand may also be the broadcast one on the left
    if kind == "sub":
        got = dev.binary(kind, b, a, shape)
        close(got, ops.broadcast_binary(kind, b, a, shape))


@pytest.mark.parametrize("n", [1, 3, 4, 1023, 1 << 20, (1 << 20) + 5])
def test_unary_scalar(dev, n):
    r = rng(2)
    x = r.standard_normal(n).astype(np.float32)
    for kind, ref in (("sigmoid", ops.sigmoid), ("exp", np.exp), ("gelu", ops.gelu),
                      ("gelu_derivative", ops.gelu_derivative)):
        close(dev.unary(kind, x), ref(x.astype(np.float64)), rtol=2e-6, atol=2e-6)
    close(dev.unary("sqrt", np.abs(x)), np.sqrt(np.abs(x).astype(np.float64)), rtol=1e-6)
    close(dev.scalar("add", x, 1e-6), ops.scalar_op("add", x, np.float32(1e-6)), rtol=1e-6)
    close(dev.scalar("div", x, 384.0), ops.scalar_op("div", x, 384.0), rtol=1e-6)
    close(dev.scalar("pow", np.abs(x), 3.0), ops.scalar_op("pow", np.abs(x), 3.0), rtol=2e-6)
    g = r.standard_normal(n).astype(np.float32)
    close(dev.gelu_backward(x, g), ops.gelu_backward(x, g), rtol=2e-6, atol=2e-6)


def test_gelu_accuracy_sweep(dev):
    """GELU and GELU' (k_elementwise, and through tl_common.cuh every GEMM
    epilogue) over a dense grid and extreme inputs against the float64
    formula in its stable form (x / (1 + e^{-2u}): the tanh form cancels
    for very negative x): GELU within 2e-6 relative plus 1e-9 absolute
    (below x of about -3 the value is under 1e-4 and its exponent's float
    rounding, 2^-24 of |2u| ~ 100, gives up to 1e-5 relative: 1e-13
    absolute, where the reference's float tanh form 0.5 x (1 + tanh u)
    has no significant digit left; below x = -9.5 the kernels return about
    1e-37 where the exact value underflows), GELU' within 5e-7 absolute plus
    2e-6 relative."""
    x = np.concatenate([np.linspace(-12, 12, (1 << 20) + 1),
                        [-1e4, -100.0, -30.0, 0.0, 1e-30, -1e-30, 30.0, 100.0, 1e4]])
    x = x.astype(np.float32)
    xd = x.astype(np.float64)
    u = np.sqrt(2 / 3.14159265) * (xd + 0.044715 * xd ** 3)
    with np.errstate(over="ignore"):
        e = np.exp(-2 * u)
    s = 1 / (1 + e)
    want_g = xd * s
    with np.errstate(invalid="ignore"):
        es = np.where(np.isinf(e), 1.0, e * s)
    want_d = s * (1 + 2 * np.sqrt(2 / 3.14159265) * xd * es * (1 + 3 * 0.044715 * xd ** 2))
    got_g = dev.unary("gelu", x).astype(np.float64)
    got_d = dev.unary("gelu_derivative", x).astype(np.float64)
    assert np.all(np.abs(got_g - want_g) <= 2e-6 * np.abs(want_g) + 1e-9)
    assert np.all(np.abs(got_d - want_d) <= 5e-7 + 2e-6 * np.abs(want_d))
    # the float64 oracle (tanh form) on ordinary inputs
    close(got_g[np.abs(x) < 5], ops.gelu(xd[np.abs(x) < 5]), rtol=2e-6, atol=2e-7)


@pytest.mark.parametrize("shape,out", [
    ((12288, 384), (12288, 1)),       # RMS row sums
    ((73728, 192), (73728, 1)),       # softmax-backward row sums
    ((64, 192, 384), (1, 384)),       # bias gradient
    ((64, 192, 1536), (1536,)),       # bias gradient, lower rank
    ((64, 384, 384), (384, 384)),     # weight-gradient batch reduction
    ((3000, 100), (1, 100)),          # ragged 128-column block
    ((1029, 36), (36,)),              # rows not a multiple of the split
    ((2, 3, 4), (1, 3, 1)),           # non-adjacent
    ((5, 7, 3), (5, 1, 3)),           # middle
    ((3, 1, 5), (1, 1, 1)),
    ((8_000_000,), (1,)),             # full reduction, split + second pass
    ((6, 5, 4, 3), (6, 1, 4, 1)),     # generic interleaving
])
def test_reduce_sum(dev, shape, out):
    r = rng(3)
    x = r.standard_normal(shape).astype(np.float32)
    got = dev.reduce("sum", x, out)
    want = ops.sum_to_shape(x, out)
    # fp32 accumulation of n terms: bound by sum |x| (not by the result)
    scale = ops.sum_to_shape(np.abs(x), out).max()
    close(got, want, rtol=0, atol=1e-6 * scale + 1e-6)


@pytest.mark.parametrize("shape,out,groups,op", [
    ((64, 192, 384), (1, 384), 3, capi.TL_REDUCE_SUM),    # the q / k / v bias gradients
    ((64, 192, 1536), (1536,), 4, capi.TL_REDUCE_SUM),
    ((3000, 100), (1, 100), 2, capi.TL_REDUCE_MAX),       # ragged column block
    ((1029, 36), (36,), 2, capi.TL_REDUCE_SUM),           # one launch per group
    ((5, 7, 3), (5, 1, 3), 3, capi.TL_REDUCE_SUM),        # not a column reduction
])
def test_reduce_group_matches_single(dev, shape, out, groups, op):
    """tl_reduce_group: each group's result bit-identical to tl_reduce of
    that tensor alone (same plan, same fold order), on two calls in a row."""
    r = rng(6)
    xs = [r.standard_normal(shape).astype(np.float32) for _ in range(groups)]
    kind = "sum" if op == capi.TL_REDUCE_SUM else "max"
    want = [dev.reduce(kind, x, out) for x in xs]
    sa, oa = capi.shape_arr(shape), capi.shape_arr(out)
    nbytes = dev.lib.tl_reduce_group_workspace_size(groups, sa, len(shape), oa, len(out))
    assert nbytes == groups * dev.lib.tl_reduce_workspace_size(sa, len(shape), oa, len(out))
    ws = dev.ws(nbytes)
    txs = [dev.t(x) for x in xs]
    for _ in range(2):
        outs = [dev.empty(out) for _ in range(groups)]
        xp = (ctypes.c_void_p * groups)(*[t.data_ptr() for t in txs])
        op_ = (ctypes.c_void_p * groups)(*[o.data_ptr() for o in outs])
        dev.call("tl_reduce_group", op, groups, xp, sa, len(shape), op_, oa, len(out),
                 dev.p(ws), nbytes, dev.stream)
        for o, w in zip(outs, want):
            np.testing.assert_array_equal(dev.host(o), w)
    bad = (ctypes.c_void_p * 5)(*([txs[0].data_ptr()] * 5))
    assert dev.lib.tl_reduce_group(op, 5, bad, sa, len(shape), bad, oa, len(out), dev.p(ws),
                                   nbytes, dev.stream) == capi.TL_ERR_INVALID
    assert dev.lib.tl_reduce_group(op, 0, bad, sa, len(shape), bad, oa, len(out), dev.p(ws),
                                   nbytes, dev.stream) == capi.TL_ERR_INVALID


@pytest.mark.parametrize("shape,out", [((2, 3), (2, 1)), ((64, 6, 192, 192), (64, 6, 192, 1)),
                                        ((9, 33), (1, 33)), ((4, 5, 6), (4, 1, 6)),
                                        ((5000, 68), (1, 68))])
def test_reduce_max(dev, shape, out):
    x = rng(4).standard_normal(shape).astype(np.float32)
    np.testing.assert_array_equal(dev.reduce("max", x, out),
                                  ops.max_to_shape(x, out).astype(np.float32))


@pytest.mark.parametrize("n,pos", [(1, 0), (5000, 4097), (1 << 22, 3_000_001), (777, 776)])
def test_argmax_bit_exact(dev, n, pos):
    x = rng(5).standard_normal(n).astype(np.float32)
    x[pos] = 50.0
    assert dev.argmax(x) == ops.argmax(x) == pos
    # ties take the lowest index; NaN and -inf never win
    y = np.full(n + 3, -np.inf, np.float32)
    y[1] = np.nan
    y[-1] = 2.0
    y[-2] = 2.0
    assert dev.argmax(y) == ops.argmax(y) == n + 1
    assert dev.argmax(np.full(4, -np.inf, np.float32)) == 0


@pytest.mark.parametrize("shape,dims", [
    ((64, 192, 384), (-2, -1)), ((384, 2048), (-2, -1)), ((64, 192, 6, 64), (1, 2)),
    ((64, 6, 192, 64), (1, 2)), ((64, 6, 192, 64), (-2, -1)), ((3, 5, 7, 9), (0, 2)),
    ((33, 65), (0, 1)), ((2, 1, 3), (0, 1)), ((2, 8, 3, 12), (1, 3)), ((3, 4, 5, 8), (0, 2)),
    ((70, 130), (0, 1)),
])
def test_transpose_bit_exact(dev, shape, dims):
    x = rng(6).standard_normal(shape).astype(np.float32)
    np.testing.assert_array_equal(dev.transpose(x, *dims), np.swapaxes(x, *dims))


@pytest.mark.parametrize("rows,cols", [(73728, 192), (12288, 2048), (3, 1), (5, 37), (2, 5000)])
def test_softmax_and_backward(dev, rows, cols):
    r = rng(7)
    x = (r.standard_normal((rows, cols)) * 4).astype(np.float32)
    close(dev.rows("softmax", x), ops.softmax_rows(x), rtol=1e-5, atol=1e-7)
    y = ops.softmax_rows(x).astype(np.float32)
    g = r.standard_normal((rows, cols)).astype(np.float32)
    close(dev.rows("softmax_bwd", g, y), ops.softmax_backward(g, y), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("rows,cols", [(73728, 192), (40, 37), (6, 5000)])
def test_softmax_scaled_masked_is_the_op_chain(dev, rows, cols):
    """Fused divide + mask add + softmax equals the three separate kernels
    bit for bit (same per-element arithmetic, same reduction order)."""
    r = rng(17)
    x = (r.standard_normal((rows, cols)) * 6).astype(np.float32)
    t = 192 if rows % 192 == 0 and cols == 192 else 4
    mask = np.triu(np.full((t, cols), -np.inf, np.float32), 1) if rows % t == 0 else None
    d = np.float32(8.0)
    fused = dev.softmax_scaled_masked(x, d, mask)
    s1 = dev.binary("div", x, np.full((1, 1), d, np.float32), x.shape)
    if mask is not None:
        s1 = dev.binary("add", s1.reshape(rows // t, t, cols), mask.reshape(1, t, cols),
                        (rows // t, t, cols)).reshape(rows, cols)
    chain = dev.rows("softmax", s1)
    np.testing.assert_array_equal(fused, chain)
    want = ops.softmax_rows(x.astype(np.float64) / 8.0 + (np.tile(mask, (rows // t, 1)) if mask is not None else 0))
    close(fused, want, rtol=1e-5, atol=1e-7)


def test_softmax_backward_divisor_and_rmsnorm_backward_addend(dev):
    r = rng(18)
    x = (r.standard_normal((384, 192)) * 3).astype(np.float32)
    y = ops.softmax_rows(x).astype(np.float32)
    g = r.standard_normal((384, 192)).astype(np.float32)
    plain = dev.rows("softmax_bwd", g, y)
    np.testing.assert_array_equal(dev.softmax_bwd_div(g, y, 8.0),
                                  dev.binary("div", plain, np.full((1, 1), 8.0, np.float32),
                                             plain.shape))
    x = r.standard_normal((96, 384)).astype(np.float32)
    yn = ops.rmsnorm(x).astype(np.float32)
    g = r.standard_normal((96, 384)).astype(np.float32)
    a = r.standard_normal((96, 384)).astype(np.float32)
    plain = dev.rows("rmsnorm_bwd", g, x, yn)
    want = dev.binary("add", a, plain, a.shape)
    np.testing.assert_array_equal(dev.rmsnorm_bwd_add(g, x, yn, a), want)
    np.testing.assert_array_equal(dev.rmsnorm_bwd_add(g, x, yn, a, in_place=True), want)


def test_softmax_masked_rows(dev):
    x = np.array([[0.0, -np.inf, -np.inf], [1000, 1001, -np.inf]], np.float32)
    close(dev.rows("softmax", x), ops.softmax_rows(x), atol=1e-7)


@pytest.mark.parametrize("rows,cols", [(12288, 384), (12288, 1536), (7, 5), (1, 768)])
def test_rms_family(dev, rows, cols):
    r = rng(8)
    x = r.standard_normal((rows, cols)).astype(np.float32)
    close(dev.rows("rms", x), ops.rms(x), rtol=1e-5)
    close(dev.rows("rmsnorm", x), ops.rmsnorm(x), rtol=1e-5, atol=1e-6)
    y = ops.rmsnorm(x).astype(np.float32)
    g = r.standard_normal((rows, cols)).astype(np.float32)
    close(dev.rows("rmsnorm_bwd", g, x, y), ops.rmsnorm_backward(g, x, y), rtol=1e-5, atol=2e-6)


@pytest.mark.parametrize("rows,vocab", [(12288, 2048), (4, 3), (9, 1001), (100, 512), (64, 1000),
                                        (33, 4100)])
def test_cross_entropy(dev, rows, vocab):
    r = rng(9)
    z = (r.standard_normal((rows, vocab)) * 3).astype(np.float32)
    t = r.integers(0, vocab, rows).astype(np.uint32)
    t[0] = vocab + 5  # out of range -> +inf row
    close(dev.xent(z, t)[1:], ops.cross_entropy(z, t)[1:], rtol=1e-5)
    assert np.isposinf(dev.xent(z, t)[0, 0])
    scale = r.uniform(0.1, 2.0, rows).astype(np.float32)
    got = dev.xent(z, t, backward=True, row_scale=scale)
    want = ops.cross_entropy_derivative(z, t, row_scale=scale)
    assert np.all(np.isposinf(got[0]))
    close(got[1:], want[1:], rtol=1e-5, atol=1e-7)
    close(dev.xent(z, t, backward=True)[1:], ops.cross_entropy_derivative(z, t)[1:],
          rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("n_rows,dim,n_ids", [(2048, 384, 12288), (192, 384, 12288), (4, 3, 4),
                                               (50, 7, 100),
                                               (3000, 1100, 5000),    # two column slices
                                               (100000, 8, 12288)])  # no slot table: searches
def test_embedding_gather_scatter(dev, n_rows, dim, n_ids):
    r = rng(10)
    w = r.standard_normal((n_rows, dim)).astype(np.float32)
    p = 1.0 / np.arange(1, n_rows + 1) ** 1.1
    ids = r.choice(n_rows, n_ids, p=p / p.sum()).astype(np.uint32)  # Zipf-like hot rows
    np.testing.assert_array_equal(dev.gather(w, ids), w[ids])
    v = r.standard_normal((n_ids, dim)).astype(np.float32)
    want = ops.scatter_add(v, ids, n_rows)
    scale = ops.scatter_add(np.abs(v), ids, n_rows).max()
    close(dev.scatter(v, ids, n_rows), want, rtol=0, atol=2e-6 * scale)
    base = r.standard_normal((n_rows, dim)).astype(np.float32)
    close(dev.scatter(v, ids, n_rows, base), ops.scatter_add(v, ids, n_rows, base), rtol=0,
          atol=2e-6 * (scale + 4))
    # deterministic: same bits every run
    np.testing.assert_array_equal(dev.scatter(v, ids, n_rows), dev.scatter(v, ids, n_rows))


def test_embedding_ids_out_of_range_flag(dev):
    from templit_b200 import capi
    dev.status()  # clear
    w = np.ones((4, 8), np.float32)
    out = dev.gather(w, np.array([1, 9, 2], np.uint32))
    assert np.all(out[1] == 0) and np.all(out[0] == 1)
    assert dev.status() & capi.TL_FLAG_INDEX_RANGE
    dev.scatter(np.ones((2, 8), np.float32), np.array([0, 7], np.uint32), 4)
    assert dev.status() & capi.TL_FLAG_INDEX_RANGE
    assert dev.status() == 0


def test_multi_grad_flat_round_trip(dev):
    """tl_multi_grad_flat: every gradient lands at chunk0 * TL_OPT_CHUNK of
    the flat buffer, padding untouched, and unpacking writes the buffer back
    (the packed all-reduce of the data-parallel step); one gradient starts
    4 bytes past an aligned address (the element-wise path)."""
    r = rng(12)
    sizes = [384 * 384, 384, 1, 8191, 8193, 5, 3 * 8192]
    base = dev.t(np.zeros(sum(sizes) + 64 * (len(sizes) + 1), np.float32))
    grads, off = [], 0
    for i, s in enumerate(sizes):
        if i == 5:
            off += 1  # unaligned
        grads.append(base[off:off + s])
        off = (off + s + 63) // 64 * 64
    vals = [r.standard_normal(s).astype(np.float32) for s in sizes]
    for g, v in zip(grads, vals):
        g.copy_(dev.t(v))
    slots = (capi.TlParamSlot * len(sizes))()
    chunk = 0
    for i, s in enumerate(sizes):
        slots[i].grad = grads[i].data_ptr()
        slots[i].count = s
        slots[i].chunk0 = chunk
        chunk += (s + capi.TL_OPT_CHUNK - 1) // capi.TL_OPT_CHUNK
    dslots = dev.t(np.frombuffer(bytes(slots), np.uint8), dtype=np.uint8)
    flat = dev.t(np.full(chunk * capi.TL_OPT_CHUNK, 7.0, np.float32))
    dev.call("tl_multi_grad_flat", dev.p(dslots), len(sizes), chunk, dev.p(flat), 0, dev.stream)
    f = dev.host(flat)
    for i, s in enumerate(sizes):
        o = slots[i].chunk0 * capi.TL_OPT_CHUNK
        np.testing.assert_array_equal(f[o:o + s], vals[i])
        nxt = slots[i + 1].chunk0 * capi.TL_OPT_CHUNK if i + 1 < len(sizes) else f.size
        assert np.all(f[o + s:nxt] == 7.0)
    flat.mul_(2.0)
    dev.call("tl_multi_grad_flat", dev.p(dslots), len(sizes), chunk, dev.p(flat), 1, dev.stream)
    for g, v in zip(grads, vals):
        np.testing.assert_array_equal(dev.host(g), 2.0 * v)


def test_multi_tensor_clip_adamw_matches_per_tensor(dev):
    """tl_multi_clip_adamw == norm + clip + AdamW per tensor (compile.h:236-258)."""
    import ctypes
    from templit_b200 import capi
    r = rng(11)
    sizes = [384 * 384, 384, 1, 8191, 8193, 2048 * 384, 5]
    lr, b1v, b2v, eps, wd, clip = 3e-4, 0.9, 0.95, 1e-8, 0.1, 1.0
    ps = [r.standard_normal(s).astype(np.float32) * 0.02 for s in sizes]
    gs = [r.standard_normal(s).astype(np.float32) * 0.05 for s in sizes]
    m1s = [r.standard_normal(s).astype(np.float32) * 1e-3 for s in sizes]
    m2s = [np.abs(r.standard_normal(s)).astype(np.float32) * 1e-4 for s in sizes]
    steps = [3] * len(sizes)
    n2 = ops.grad_sqnorm(gs)
    want = [ops.adamw(p, ops.clip(g, n2, clip), m1, m2, lr, b1v, b2v, eps, wd, st)
            for p, g, m1, m2, st in zip(ps, gs, m1s, m2s, steps)]
    tp = [dev.t(x) for x in ps]
    tg = [dev.t(x) for x in gs]
    t1 = [dev.t(x) for x in m1s]
    t2 = [dev.t(x) for x in m2s]
    slots = (capi.TlParamSlot * len(sizes))()
    chunk = 0
    for i, s in enumerate(sizes):
        slots[i].param = tp[i].data_ptr()
        slots[i].out = tp[i].data_ptr()
        slots[i].grad = tg[i].data_ptr()
        slots[i].m1 = t1[i].data_ptr()
        slots[i].m2 = t2[i].data_ptr()
        slots[i].count = s
        slots[i].chunk0 = chunk
        slots[i].step = steps[i]
        chunk += (s + capi.TL_OPT_CHUNK - 1) // capi.TL_OPT_CHUNK
    raw = np.frombuffer(bytes(slots), np.uint8)
    dslots = dev.t(raw, dtype=np.uint8)
    sq = dev.t([0.0])
    nb = dev.lib.tl_multi_clip_adamw_workspace_size(chunk)
    ws = dev.ws(nb)
    scal = [dev.t([v]) for v in (b1v, b2v, np.float32(1) - np.float32(lr) * np.float32(wd), lr)]
    dev.call("tl_multi_clip_adamw", dev.p(dslots), len(sizes), chunk, dev.p(sq), ctypes.c_float(clip),
             *[dev.p(s) for s in scal], ctypes.c_float(eps), dev.p(ws), nb, dev.stream)
    assert abs(float(dev.host(sq)[0]) - n2) <= 1e-5 * n2
    for i in range(len(sizes)):
        close(dev.host(tp[i]), want[i][0], rtol=1e-5, atol=1e-7)
        close(dev.host(t1[i]), want[i][1], rtol=1e-5, atol=1e-9)
        close(dev.host(t2[i]), want[i][2], rtol=1e-5, atol=1e-12)
        close(dev.host(tg[i]), ops.clip(gs[i], n2, clip), rtol=1e-6, atol=1e-9)
