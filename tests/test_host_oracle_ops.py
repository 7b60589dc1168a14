"""Pins the host oracle runtime (oracle/cpu_gpt/host_runtime.h: the ops the
GPT-step oracle runs under the reference's passes::Compiled) op by op,
through its C entry points (oracle/_build/libhost_ops.so):

  * against the reference's own known answers (tests/golden/
    known_answers.json, restated from JTPuffer/TempLit tests/
    test_metal_runtime.cpp and tests/test_meta.cpp), with their tolerances;
  * against the float64 restatement oracle/ops.py on seeded inputs at the
    GPT step's row widths, with broadcast, batched, ragged and empty-row
    cases: 1e-6 relative for the float ops (the host runtime accumulates in
    double and rounds once to float), bit-exact for argmax, gather and the
    scatter of integers.

So the GPT-level parity tests compare the CUDA runtime with an oracle whose
every op is itself checked.  CPU only."""
import ctypes
import os

import numpy as np
import pytest

from oracle import ops
from tests.helpers import known_answers
from tests.test_oracle_golden import compare

LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle",
                   "_build", "libhost_ops.so")

F32P = ctypes.POINTER(ctypes.c_float)
U32P = ctypes.POINTER(ctypes.c_uint32)


@pytest.fixture(scope="module")
def host():
    if not os.path.exists(LIB):
        pytest.fail("host oracle ops not built (make -C oracle/cpu_gpt ops)")
    return HostOps(ctypes.CDLL(LIB))


def f32(x):
    return np.ascontiguousarray(np.asarray(x, np.float32))


def u32(x):
    return np.ascontiguousarray(np.asarray(x, np.uint32))


def fp(a):
    return a.ctypes.data_as(F32P) if a is not None else None


def up(a):
    return a.ctypes.data_as(U32P)


class HostOps:
    def __init__(self, lib):
        self.lib = lib
        lib.tlo_h_error.restype = ctypes.c_char_p

    def _ok(self, rc):
        if rc != 0:
            raise ValueError(self.lib.tlo_h_error().decode())

    def binary(self, kind, a, a_shape, b, b_shape, out_shape):
        a, b = f32(a), f32(b)
        out = np.zeros(int(np.prod(out_shape)), np.float32)
        sa, sb, so = u32(a_shape), u32(b_shape), u32(out_shape)
        self._ok(self.lib.tlo_h_binary(kind.encode(), fp(a), up(sa), len(sa), fp(b), up(sb),
                                       len(sb), fp(out), up(so), len(so)))
        return out.reshape(out_shape)

    def scalar(self, kind, x, s):
        x = f32(x).ravel()
        out = np.zeros_like(x)
        self._ok(self.lib.tlo_h_scalar(kind.encode(), fp(x), x.size, ctypes.c_float(s), fp(out)))
        return out

    def unary(self, kind, x):
        x = f32(x).ravel()
        out = np.zeros_like(x)
        self._ok(self.lib.tlo_h_unary(kind.encode(), fp(x), x.size, fp(out)))
        return out

    def mult(self, a, b, out_shape):
        a, b = f32(a), f32(b)
        out = np.zeros(out_shape, np.float32)
        sa, sb, so = u32(a.shape), u32(b.shape), u32(out_shape)
        self._ok(self.lib.tlo_h_mult(fp(a), up(sa), len(sa), fp(b), up(sb), len(sb), fp(out),
                                     up(so), len(so)))
        return out

    def transpose(self, x, da, db):
        x = f32(x)
        shape = list(x.shape)
        shape[da], shape[db] = shape[db], shape[da]
        out = np.zeros(shape, np.float32)
        sx, so = u32(x.shape), u32(shape)
        self._ok(self.lib.tlo_h_transpose(fp(x), up(sx), len(sx), da, db, fp(out), up(so)))
        return out

    def reduce(self, kind, x, out_shape):
        x = f32(x)
        out = np.zeros(out_shape, np.float32)
        sx, so = u32(x.shape), u32(out_shape)
        self._ok(self.lib.tlo_h_reduce(kind.encode(), fp(x), up(sx), len(sx), fp(out), up(so),
                                       len(so)))
        return out

    def rows(self, kind, x):
        x = f32(x)
        shape = list(x.shape[:-1]) + [1] if kind == "rms" else list(x.shape)
        out = np.zeros(shape, np.float32)
        sx, so = u32(x.shape), u32(shape)
        self._ok(self.lib.tlo_h_rows(kind.encode(), fp(x), up(sx), len(sx), fp(out), up(so),
                                     len(so)))
        return out

    def xent(self, z, t, derivative):
        z, t = f32(z), u32(t)
        shape = list(z.shape) if derivative else list(z.shape[:-1]) + [1]
        out = np.zeros(shape, np.float32)
        sz, so = u32(z.shape), u32(shape)
        self._ok(self.lib.tlo_h_xent(int(derivative), fp(z), up(sz), len(sz), up(t), fp(out),
                                     up(so), len(so)))
        return out

    def argmax(self, x):
        x = f32(x).ravel()
        out = ctypes.c_uint32()
        self._ok(self.lib.tlo_h_argmax(fp(x), x.size, ctypes.byref(out)))
        return out.value

    def gather(self, w, ids):
        w, ids = f32(w), u32(ids)
        out = np.zeros((ids.size, w.shape[1]), np.float32)
        self._ok(self.lib.tlo_h_gather(fp(w), w.shape[0], w.shape[1], up(ids), ids.size, fp(out)))
        return out

    def scatter(self, values, ids, n_rows, base=None):
        values, ids = f32(values), u32(ids)
        base = None if base is None else f32(base)
        out = np.zeros((n_rows, values.shape[1]), np.float32)
        self._ok(self.lib.tlo_h_scatter(fp(values), up(ids), ids.size, values.shape[1], fp(base),
                                        fp(out), n_rows))
        return out

    def clip(self, grads, max_norm):
        gs = [f32(g).ravel() for g in grads]
        outs = [np.zeros_like(g) for g in gs]
        gp = (F32P * len(gs))(*[fp(g) for g in gs])
        op = (F32P * len(gs))(*[fp(o) for o in outs])
        counts = u32([g.size for g in gs])
        sq = ctypes.c_float()
        self._ok(self.lib.tlo_h_clip(gp, up(counts), len(gs), ctypes.c_float(max_norm),
                                     ctypes.byref(sq), op))
        return sq.value, outs

    def adamw(self, p, g, m1, m2, lr, beta1, beta2, eps, weight_decay, step):
        p, g, m1, m2 = (f32(v).ravel().copy() for v in (p, g, m1, m2))
        decay = np.float32(1) - np.float32(lr) * np.float32(weight_decay)
        self._ok(self.lib.tlo_h_adamw(fp(p), fp(g), fp(m1), fp(m2), p.size, ctypes.c_float(beta1),
                                      ctypes.c_float(beta2), ctypes.c_float(decay),
                                      ctypes.c_float(lr), ctypes.c_float(eps), step))
        return p, m1, m2


# ------------------------------------------------- the reference's answers
def host_eval(h, case):
    op, i = case["op"], case["inputs"]
    if op == "binary":
        return h.binary(i["kind"], i["a"], i["a_shape"], i["b"], i["b_shape"], i["out_shape"])
    if op == "scalar":
        return h.scalar(i["kind"], i["x"], i["s"])
    if op == "unary":
        return h.unary(i["kind"], i["x"])
    if op in ("rms", "rmsnorm", "softmax"):
        return h.rows(op, np.reshape(i["x"], i["shape"]))
    if op == "matmul":
        a, b = np.reshape(i["a"], i["a_shape"]), np.reshape(i["b"], i["b_shape"])
        return h.mult(a, b, np.matmul(a, b).shape)
    if op in ("sum_to_shape", "max_to_shape"):
        return h.reduce(op, np.reshape(i["x"], i["shape"]), i["out_shape"])
    if op == "transpose":
        return h.transpose(np.reshape(i["x"], i["shape"]), *i["dims"])
    if op in ("cross_entropy", "cross_entropy_derivative"):
        z = np.reshape(i["logits"], i["shape"])
        return h.xent(z, np.reshape(i["targets"], z.shape[:-1]), op != "cross_entropy")
    if op == "argmax":
        return [h.argmax(i["x"])]
    if op == "embedding_lookup":
        return h.gather(np.reshape(i["weights"], i["w_shape"]), i["ids"])
    if op == "scatter":
        base = None if i["base"] is None else np.reshape(i["base"], (i["n_rows"], i["dim"]))
        return h.scatter(np.reshape(i["values"], (-1, i["dim"])), i["ids"], i["n_rows"], base)
    if op == "clip":
        sq, clipped = h.clip(i["grads"], i["max_norm"])
        return {"sqnorm": sq, "clipped": clipped}
    if op == "adamw":
        p, g = i["param"], i["grad"]
        m1 = m2 = np.zeros(len(p))
        out = []
        for step in (1, 2):
            p, m1, m2 = h.adamw(p, g, m1, m2, i["lr"], i["beta1"], i["beta2"], i["eps"],
                                i["weight_decay"], step)
            out.append(p)
        return out
    return None  # compositions through the executor: covered by the GPT tests


CASES = [c for c in known_answers()
         if c["op"] not in ("rms_backward_sgd", "embedding_sgd", "cross_entropy_sgd")]


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_host_ops_match_reference_known_answers(host, case):
    compare(host_eval(host, case), case)


# ----------------------------------------------------- the float64 oracle
def close(got, want, rtol=1e-6, atol=1e-7):
    np.testing.assert_allclose(np.asarray(got, np.float64), np.asarray(want, np.float64),
                               rtol=rtol, atol=atol)


@pytest.fixture
def rng():
    return np.random.default_rng(20)


def test_broadcast_binary(host, rng):
    for kind in ("add", "sub", "mul", "div"):
        for sa, sb, so in (((4, 6, 8), (8,), (4, 6, 8)), ((4, 1, 8), (6, 1), (4, 6, 8)),
                           ((3, 5), (3, 5), (3, 5))):
            a = rng.standard_normal(sa).astype(np.float32)
            b = rng.standard_normal(sb).astype(np.float32) + (3.0 if kind == "div" else 0.0)
            close(host.binary(kind, a, sa, b, sb, so), ops.broadcast_binary(kind, a, b, so))
    with pytest.raises(ValueError):
        host.binary("add", np.zeros(6), (2, 3), np.zeros(4), (4,), (2, 3))


def test_batched_and_broadcast_products(host, rng):
    for sa, sb in (((7, 384), (384, 96)), ((2, 3, 17, 64), (2, 3, 64, 33)),
                   ((4, 24, 16), (16, 40)), ((1, 5, 8), (3, 8, 6))):
        a = rng.standard_normal(sa).astype(np.float32)
        b = rng.standard_normal(sb).astype(np.float32)
        want = ops.matmul(a, b)
        close(host.mult(a, b, want.shape), want, rtol=1e-5, atol=1e-5)


def test_transpose_reductions_and_rows(host, rng):
    x = rng.standard_normal((3, 5, 7, 4)).astype(np.float32)
    for da, db in ((-2, -1), (1, 2), (0, 3)):
        np.testing.assert_array_equal(host.transpose(x, da, db), ops.transpose(x, da, db))
    for out in ((1, 5, 1, 4), (3, 1, 7, 1), (1,), (5, 7, 4)):
        close(host.reduce("sum_to_shape", x, out), ops.sum_to_shape(x, out), atol=1e-6)
    close(host.reduce("max_to_shape", x, (3, 5, 7, 1)), ops.max_to_shape(x, (3, 5, 7, 1)))
    r = rng.standard_normal((48, 384)).astype(np.float32)
    close(host.rows("softmax", r), ops.softmax_rows(r))
    close(host.rows("rms", r), ops.rms(r))
    close(host.rows("rmsnorm", r), ops.rmsnorm(r))
    z = np.zeros((2, 8), np.float32)  # rms of a zero row is the reference's eps floor
    close(host.rows("rms", z), ops.rms(z))


def test_cross_entropy_gather_scatter_argmax(host, rng):
    z = rng.standard_normal((6, 32, 2048)).astype(np.float32) * 3
    t = rng.integers(0, 2048, (6, 32))
    close(host.xent(z, t, False), ops.cross_entropy(z, t))
    close(host.xent(z, t, True), ops.cross_entropy_derivative(z, t), atol=1e-9)
    t_bad = t.copy()
    t_bad[0, 0] = 2048  # an out-of-range target gives +inf, as the reference
    assert np.isinf(host.xent(z, t_bad, False)[0, 0, 0])
    w = rng.standard_normal((2048, 384)).astype(np.float32)
    ids = rng.integers(0, 2048, 300)
    np.testing.assert_array_equal(host.gather(w, ids), w[ids])
    v = rng.standard_normal((300, 384)).astype(np.float32)
    base = rng.standard_normal((2048, 384)).astype(np.float32)
    close(host.scatter(v, ids, 2048, base), ops.scatter_add(v, ids, 2048, base), atol=1e-6)
    iv = rng.integers(-8, 8, (300, 16)).astype(np.float32)  # integers: exact in any order
    np.testing.assert_array_equal(host.scatter(iv, ids, 2048), ops.scatter_add(iv, ids, 2048))
    x = rng.standard_normal(1000).astype(np.float32)
    assert host.argmax(x) == ops.argmax(x)


def test_norm_clip_and_adamw(host, rng):
    grads = [rng.standard_normal(n).astype(np.float32) for n in (384 * 384, 384, 7)]
    sq, clipped = host.clip(grads, 1.0)
    n2 = ops.grad_sqnorm(grads)
    close([sq], [n2])
    for g, c in zip(grads, clipped):
        close(c, ops.clip(g, n2, 1.0), atol=1e-10)
    p, g = (rng.standard_normal(4096).astype(np.float32) for _ in range(2))
    m1 = rng.standard_normal(4096).astype(np.float32) * 1e-3
    m2 = np.abs(rng.standard_normal(4096)).astype(np.float32) * 1e-4
    got = host.adamw(p, g, m1, m2, 3e-4, 0.9, 0.95, 1e-8, 0.1, 3)
    want = ops.adamw(p, g, m1, m2, 3e-4, 0.9, 0.95, 1e-8, 0.1, 3)
    for a, b in zip(got, want):
        close(a, b, atol=1e-9)
    with pytest.raises(ValueError):
        host.adamw(p, g, m1, m2, 3e-4, 0.9, 0.95, 1e-8, 0.1, 0)  # step 0 is refused
