"""Pins the CPU oracle (oracle/ops.py) against the reference's own known
answers (tests/golden/known_answers.json, restated from JTPuffer/TempLit
tests/test_metal_runtime.cpp and tests/test_meta.cpp) and against the
reference CPU runtime's outputs (tests/golden/cpu_ref_fixtures.npz, made by
running src/CPU/cpu.cpp compiled from the reference sources).  CPU only."""
import os

import numpy as np
import pytest

from oracle import ops
from tests.helpers import GOLDEN, known_answers


def oracle_eval(case):
    op, i = case["op"], case["inputs"]
    if op == "binary":
        a = np.reshape(i["a"], i["a_shape"])
        b = np.reshape(i["b"], i["b_shape"])
        return ops.broadcast_binary(i["kind"], a, b, i["out_shape"])
    if op == "scalar":
        return ops.scalar_op(i["kind"], i["x"], i["s"])
    if op == "unary":
        return {"sigmoid": ops.sigmoid, "exp": np.exp, "sqrt": np.sqrt, "gelu": ops.gelu,
                "gelu_derivative": ops.gelu_derivative}[i["kind"]](np.asarray(i["x"], np.float64))
    if op == "rms":
        return ops.rms(np.reshape(i["x"], i["shape"]))
    if op == "rmsnorm":
        return ops.rmsnorm(np.reshape(i["x"], i["shape"]))
    if op == "matmul":
        return ops.matmul(np.reshape(i["a"], i["a_shape"]), np.reshape(i["b"], i["b_shape"]))
    if op == "sum_to_shape":
        return ops.sum_to_shape(np.reshape(i["x"], i["shape"]), i["out_shape"])
    if op == "max_to_shape":
        return ops.max_to_shape(np.reshape(i["x"], i["shape"]), i["out_shape"])
    if op == "transpose":
        return ops.transpose(np.reshape(i["x"], i["shape"]), *i["dims"])
    if op == "softmax":
        return ops.softmax_rows(np.reshape(i["x"], i["shape"]))
    if op == "cross_entropy":
        z = np.reshape(i["logits"], i["shape"])
        return ops.cross_entropy(z, np.reshape(i["targets"], z.shape[:-1]))
    if op == "cross_entropy_derivative":
        z = np.reshape(i["logits"], i["shape"])
        return ops.cross_entropy_derivative(z, np.reshape(i["targets"], z.shape[:-1]))
    if op == "argmax":
        return [ops.argmax(i["x"])]
    if op == "embedding_lookup":
        return ops.embedding_gather(np.reshape(i["weights"], i["w_shape"]), i["ids"])
    if op == "scatter":
        base = None if i["base"] is None else np.reshape(i["base"], (i["n_rows"], i["dim"]))
        return ops.scatter_add(np.reshape(i["values"], (-1, i["dim"])), i["ids"], i["n_rows"], base)
    if op == "clip":
        n2 = ops.grad_sqnorm(i["grads"])
        return {"sqnorm": n2, "clipped": [ops.clip(g, n2, i["max_norm"]) for g in i["grads"]]}
    if op == "adamw":
        p, g = i["param"], i["grad"]
        m1 = m2 = np.zeros(len(p))
        out = []
        for step in (1, 2):
            p, m1, m2 = ops.adamw(p, g, m1, m2, i["lr"], i["beta1"], i["beta2"], i["eps"],
                                  i["weight_decay"], step)
            out.append(p)
        return out
    if op == "rms_backward_sgd":
        # d rms / dx through the RMS rule of autograd (RMS = sqrt(mean(x^2)+eps)):
        # the reference expects x - lr * x / (D * rms)
        x = np.asarray([i["x"]], np.float64)
        r = ops.rms(x)
        return (x - i["lr"] * x / (x.shape[-1] * r)).ravel()
    if op == "embedding_sgd":
        w = np.reshape(i["weights"], i["w_shape"]).astype(np.float64)
        grad = ops.scatter_add(np.ones((len(i["ids"]), w.shape[1])), i["ids"], w.shape[0])
        return (w - i["lr"] * grad).ravel()
    if op == "cross_entropy_sgd":
        z = np.reshape(i["logits"], i["shape"])
        d = ops.cross_entropy_derivative(z, i["targets"], row_scale=np.asarray(i["root_grad"]))
        return (z - i["lr"] * d).ravel()
    raise KeyError(op)


def compare(got, case):
    exp, eps = case["expected"], case["eps"]
    if case["op"] == "clip":
        assert abs(got["sqnorm"] - exp["sqnorm"]) < eps
        for g, e in zip(got["clipped"], exp["clipped"]):
            np.testing.assert_allclose(np.ravel(g), e, atol=eps, rtol=0)
        return
    if case["op"] == "adamw":
        for g, e in zip(got, exp):
            np.testing.assert_allclose(np.ravel(g), e, atol=eps, rtol=0)
        return
    got = np.ravel(np.asarray(got, np.float64))
    exp = np.asarray(exp, np.float64)
    if eps == 0:
        np.testing.assert_array_equal(got, exp)
    else:
        np.testing.assert_allclose(got, exp, atol=eps, rtol=0)


CASES = known_answers()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_oracle_matches_reference_known_answers(case):
    compare(oracle_eval(case), case)


def test_oracle_rejects_what_the_reference_rejects():
    with pytest.raises(ValueError):
        ops.broadcast_binary("add", np.zeros((2, 3)), np.zeros(4), (2, 3))
    with pytest.raises(ValueError):
        ops.sum_to_shape(np.zeros((2, 3)), (3, 2))
    with pytest.raises(ValueError):
        ops.max_to_shape(np.zeros((2, 3, 4)), (1, 3, 1))


def test_oracle_edge_cases():
    # invalid cross-entropy targets give +inf rows (math.metal:893-896,921-925)
    z = np.array([[1.0, 2.0, 3.0], [0.0, 0.0, 0.0]])
    loss = ops.cross_entropy(z, [5, 1])
    assert np.isinf(loss[0, 0]) and np.isfinite(loss[1, 0])
    d = ops.cross_entropy_derivative(z, [5, 1])
    assert np.all(np.isinf(d[0])) and np.all(np.isfinite(d[1]))
    # argmax: NaN and -inf never win; all-(-inf) gives 0
    assert ops.argmax([np.nan, -np.inf, 3.0, 3.0]) == 2
    assert ops.argmax([-np.inf, -np.inf]) == 0
    # RMS of a zero row is sqrt(1e-6)
    np.testing.assert_allclose(ops.rms(np.zeros((1, 8))), [[1e-3]])


FIXTURES = os.path.join(GOLDEN, "cpu_ref_fixtures.npz")


@pytest.mark.skipif(not os.path.exists(FIXTURES), reason="cpu_ref fixtures not generated")
def test_oracle_matches_reference_cpu_runtime():
    """Outputs of the reference's own CPU runtime (src/CPU/cpu.cpp) on seeded
    inputs, recorded by tests/golden/make_cpu_ref_fixtures.py."""
    fx = np.load(FIXTURES)
    names = sorted({k.split("__")[0] for k in fx.files})
    assert names
    for name in names:
        op = str(fx[name + "__op"])
        a = fx[name + "__a"]
        want = fx[name + "__out"]
        if op == "mult":
            got = ops.matmul(a, fx[name + "__b"])
            tol = 1e-5 * np.abs(a).sum(axis=1).max() * np.abs(fx[name + "__b"]).max()
        elif op in ("add", "sub", "hadamard", "divide"):
            kind = {"add": "add", "sub": "sub", "hadamard": "mul", "divide": "div"}[op]
            got = ops.broadcast_binary(kind, a, fx[name + "__b"], want.shape)
            tol = 1e-6 * max(1.0, np.abs(want).max())
        elif op == "softmax":
            got = ops.softmax_rows(a)
            tol = 1e-6
        elif op == "sum_to_shape":
            got = ops.sum_to_shape(a, want.shape)
            tol = 1e-5 * np.abs(a).sum()
        elif op == "transpose":
            got = ops.transpose(a)
            tol = 0
        elif op == "sigmoid":
            got = ops.sigmoid(a)
            tol = 1e-6
        elif op == "sqrt":
            got = np.sqrt(a.astype(np.float64))
            tol = 1e-6
        else:
            raise KeyError(op)
        np.testing.assert_allclose(got, want, atol=tol, rtol=1e-6, err_msg=name)


def test_oracle_attention_gradients_match_finite_differences():
    """The attention backward of the oracle (product rules + softmax
    derivative) agrees with central differences of its forward, so the
    GPU attention parity tests check against the right gradients."""
    rng = np.random.default_rng(5)
    B, H, T, D = 1, 2, 5, 3
    q, k, v, d_o = (rng.standard_normal((B, H, T, D)) for _ in range(4))
    mask = ops.causal_mask(T)
    div = np.sqrt(D)
    p, _ = ops.attention_forward(q, k, v, div, mask)
    grads = ops.attention_backward(q, k, v, p, div, d_o)

    def loss(qq, kk, vv):
        return float((ops.attention_forward(qq, kk, vv, div, mask)[1] * d_o).sum())

    h = 1e-6
    for which, g in enumerate(grads):
        args = [q, k, v]
        num = np.zeros_like(args[which])
        for idx in np.ndindex(num.shape):
            plus = [a.copy() for a in args]
            minus = [a.copy() for a in args]
            plus[which][idx] += h
            minus[which][idx] -= h
            num[idx] = (loss(*plus) - loss(*minus)) / (2 * h)
        np.testing.assert_allclose(g, num, rtol=1e-6, atol=1e-8)
    # the mask zeroes every weight above the diagonal
    assert not np.triu(p, 1).any()
