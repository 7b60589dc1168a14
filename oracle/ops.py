"""CPU oracle: float64 numpy restatement of the TempLit runtime ops.

TEST INFRASTRUCTURE ONLY.  Nothing in the product imports this module; it
is the checker that tests/, ``__graft_entry__.smoke()`` and bench.py's CPU
baseline compare the CUDA backend against.

Each function restates the arithmetic of one op of the reference Metal
runtime of JTPuffer/TempLit (kernel bodies in include/my_metal/math.metal,
host-side composition in src/my_metal/runtime.cpp, executor compound rules
in include/passes/execute.h), cited per function.  It is pinned against
(a) the closed-form expectations of the reference's own runtime tests
(tests/golden/known_answers.json, made by tests/golden/make_known_answers.py
from tests/test_metal_runtime.cpp and tests/test_meta.cpp) and (b) outputs of
the reference's CPU runtime (src/CPU/cpu.cpp) compiled from its sources by
oracle/ref_cpu (tests/golden/cpu_ref_fixtures.npz).

Values are computed in float64 from float32 inputs unless a function says
otherwise, so the oracle is at least as accurate as the fp32 kernels.
"""
from __future__ import annotations

import numpy as np

F64 = np.float64
GELU_A = 0.7978845608  # sqrt(2/pi) as written in math.metal:843
GELU_B = 0.044715      # math.metal:832,844
RMS_EPS = 1e-6         # runtime.cpp:1044


def _f(x):
    return np.asarray(x, dtype=F64)


# ------------------------------------------------------------- elementwise
def broadcast_binary(op: str, a, b, out_shape):
    """add/sub/hadamard/divide with trailing-aligned size-1 broadcasting of
    each operand to the destination shape (runtime.cpp:18-39,65-95;
    math.metal:401-510)."""
    out_shape = tuple(int(s) for s in out_shape)
    for s in (np.shape(a), np.shape(b)):
        if len(s) > len(out_shape):
            raise ValueError("invalid broadcast")
        off = len(out_shape) - len(s)
        for i, d in enumerate(s):
            if d != out_shape[off + i] and d != 1:
                raise ValueError("invalid broadcast")
    x = np.broadcast_to(_f(a), out_shape)
    y = np.broadcast_to(_f(b), out_shape)
    return {"add": np.add, "sub": np.subtract, "mul": np.multiply,
            "div": np.divide}[op](x, y)


def scalar_op(op: str, x, s):
    """x + s, x / s, pow(x, s) (math.metal:427-434,511-518,527-534)."""
    x = _f(x)
    if op == "add":
        return x + F64(s)
    if op == "div":
        return x / F64(s)
    if op == "pow":
        return np.power(x, F64(s))
    raise ValueError(op)


def sigmoid(x):
    """1 / (1 + exp(-x)) (math.metal:542-548)."""
    return 1.0 / (1.0 + np.exp(-_f(x)))


def gelu(x):
    """tanh-approximation GELU with sqrt(2/3.14159265) (math.metal:821-834)."""
    x = _f(x)
    k = np.sqrt(2.0 / 3.14159265)
    return 0.5 * x * (1.0 + np.tanh(k * (x + GELU_B * x ** 3)))


def gelu_derivative(x):
    """Analytic derivative of the tanh GELU (math.metal:835-855)."""
    x = _f(x)
    u = GELU_A * (x + GELU_B * x ** 3)
    t = np.tanh(u)
    return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * GELU_A * (1.0 + 3.0 * GELU_B * x * x)


def gelu_backward(x, grad):
    """GELU'(x) * grad: the GELU derivative rule followed by the chain-rule
    hadamard of include/passes/autograd.h."""
    return gelu_derivative(x) * _f(grad)


# -------------------------------------------------------------- reductions
def _aligned(a_shape, out_shape):
    if len(out_shape) > len(a_shape):
        raise ValueError("cannot reduce to a shape with a higher rank")
    al = (1,) * (len(a_shape) - len(out_shape)) + tuple(out_shape)
    axes = []
    for i, (d, o) in enumerate(zip(a_shape, al)):
        if d != o:
            if o != 1:
                raise ValueError("invalid reduce_to_shape")
            axes.append(i)
    return al, tuple(axes)


def sum_to_shape(a, out_shape):
    """Sum over every dim where the trailing-aligned output has 1
    (runtime.cpp:661-739; math.metal:618-679)."""
    a = _f(a)
    al, axes = _aligned(a.shape, out_shape)
    r = a.sum(axis=axes, keepdims=True) if axes else a.copy()
    return r.reshape(tuple(out_shape))


def max_to_shape(a, out_shape):
    """Max over the single shrinking dim (runtime.cpp:595-659,741-745;
    math.metal:681-714)."""
    a = _f(a)
    if len(out_shape) != a.ndim:
        raise ValueError("cannot reduce to shape if ranks differ")
    _, axes = _aligned(a.shape, out_shape)
    if len(axes) > 1:
        raise ValueError("reduce_to_shape currently supports only one shrinking dimension")
    return a.max(axis=axes, keepdims=True) if axes else a.copy()


def argmax(x):
    """First index of the maximum; values that are not > -inf (NaN, -inf)
    never win and an empty candidate set gives 0 (math.metal:715-777)."""
    v = _f(x).ravel()
    cand = np.where(v > -np.inf)[0]
    if cand.size == 0:
        return 0
    m = v[cand].max()
    return int(cand[np.argmax(v[cand] == m)])


def transpose(a, dim_a=-2, dim_b=-1):
    """Materialised swap of two axes (runtime.cpp:529-569; math.metal:566-584)."""
    return np.swapaxes(_f(a), dim_a, dim_b).copy()


# ----------------------------------------------------------- row operators
def softmax_rows(x):
    """max-subtracted softmax over the last dim (math.metal:857-882)."""
    x = _f(x)
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / e.sum(axis=-1, keepdims=True)


def softmax_backward(grad, y):
    """dS = y * (g - sum(g * y)): SFTMX_DERIVATIVE (execute.h:291-308)."""
    g, y = _f(grad), _f(y)
    return y * (g - (g * y).sum(axis=-1, keepdims=True))


def rms(x):
    """sqrt(sum(x^2)/D + 1e-6) over the last dim (runtime.cpp:1031-1053)."""
    x = _f(x)
    return np.sqrt((x * x).sum(axis=-1, keepdims=True) / x.shape[-1] + RMS_EPS)


def rmsnorm(x):
    """x / rms(x) (runtime.cpp:1061-1072; no learnable gain, rms_norm.h)."""
    return _f(x) / rms(x)


def rmsnorm_backward(grad, x, y):
    """dx = (g - y * mean(g * y)) / rms(x): RMSN_DERIVATIVE (execute.h:330-356)."""
    g, y = _f(grad), _f(y)
    mean = (g * y).sum(axis=-1, keepdims=True) / y.shape[-1]
    return (g - y * mean) / rms(x)


def cross_entropy(logits, targets):
    """loss = max + log(sum(exp(z - max))) - z[t], +inf for t >= vocab;
    shape targets.shape + (1,) (runtime.cpp:768-804; math.metal:884-910)."""
    z = _f(logits)
    t = np.asarray(targets, dtype=np.int64)
    v = z.shape[-1]
    zr = z.reshape(-1, v)
    tr = t.reshape(-1)
    m = zr.max(axis=1)
    lse = m + np.log(np.exp(zr - m[:, None]).sum(axis=1))
    out = np.full(tr.shape, np.inf)
    ok = tr < v
    out[ok] = lse[ok] - zr[np.arange(zr.shape[0])[ok], tr[ok]]
    return out.reshape(t.shape + (1,))


def cross_entropy_derivative(logits, targets, row_scale=None):
    """softmax(z) - onehot(t), rows with t >= vocab all +inf, optionally
    times the per-row root gradient (runtime.cpp:806-841;
    math.metal:912-953; the executor's hadamard, execute.h:261-268)."""
    z = _f(logits)
    t = np.asarray(targets, dtype=np.int64)
    v = z.shape[-1]
    p = softmax_rows(z).reshape(-1, v)
    tr = t.reshape(-1)
    ok = tr < v
    p[np.arange(p.shape[0])[ok], tr[ok]] -= 1.0
    p[~ok, :] = np.inf
    if row_scale is not None:
        p = p * _f(row_scale).reshape(-1, 1)
    return p.reshape(z.shape)


# -------------------------------------------------------------- embedding
def embedding_gather(weights, ids):
    """out[i,:] = W[ids[i],:] (runtime.cpp:920-944; math.metal:778-793)."""
    w = _f(weights)
    return w[np.asarray(ids, dtype=np.int64)]


def scatter_add(values, ids, n_rows, base=None):
    """dst = base (or zeros) + rows of values added at ids
    (runtime.cpp:983-1030; math.metal:794-820)."""
    vals = _f(values)
    dim = vals.shape[-1]
    out = np.zeros((n_rows, dim)) if base is None else _f(base).copy()
    np.add.at(out, np.asarray(ids, dtype=np.int64).reshape(-1), vals.reshape(-1, dim))
    return out


# -------------------------------------------------------------- optimiser
def grad_sqnorm(grads):
    """sum of g^2 over all gradients (math.metal:955-983)."""
    return float(sum((_f(g) ** 2).sum() for g in grads))


def clip(grad, sqnorm, max_norm):
    """g * min(1, c / sqrt(max(n^2, 1e-12))) (math.metal:985-1006)."""
    return _f(grad) * min(1.0, max_norm / np.sqrt(max(sqnorm, 1e-12)))


def adamw(param, grad, m1, m2, lr, beta1, beta2, eps, weight_decay, step):
    """One AdamW update with decoupled decay p * (1 - lr * wd)
    (math.metal:1008-1043; include/optimiser/AdamW.h:26-37,75-82).
    Returns (param, m1, m2)."""
    p, g = _f(param), _f(grad)
    m1 = beta1 * _f(m1) + (1.0 - beta1) * g
    m2 = beta2 * _f(m2) + (1.0 - beta2) * g * g
    decay = 1.0 - lr * weight_decay
    c1 = 1.0 - beta1 ** step
    c2 = 1.0 - beta2 ** step
    p = p * decay - lr * (m1 / c1) / (np.sqrt(m2 / c2) + eps)
    return p, m1, m2


# ------------------------------------------------------------------- GEMM
def matmul(a, b):
    """C = A B over the last two dims with broadcast batch dims
    (runtime.cpp:375-505; shape rule include/RTensor/infer_shape.h:65-112)."""
    return np.matmul(_f(a), _f(b))


def gemm(a, b, trans_a=False, trans_b=False, bias=None, c=None, beta=0.0):
    """The tl_gemm contract: op(A) op(B) (+ bias) (+ beta * C), the
    executor's transpose+mult pairs (execute.h:187-232) and linear
    (execute.h:241-252) folded into one product."""
    x = np.swapaxes(_f(a), -1, -2) if trans_a else _f(a)
    y = np.swapaxes(_f(b), -1, -2) if trans_b else _f(b)
    r = np.matmul(x, y)
    if bias is not None:
        r = r + _f(bias)
    if beta:
        r = _f(c) + r
    return r


# -------------------------------------------------------------- attention
def causal_mask(t):
    """[T, T] mask, -inf above the diagonal, 0 elsewhere (nn::causal_mask,
    include/nn/attention.h:10-22)."""
    return np.triu(np.full((t, t), -np.inf), 1)


def attention_forward(q, k, v, divisor, mask=None):
    """Attention core of MultiHeadAttention on head-split [B, H, T, D]
    operands (include/nn/multi_head.h:45-52): P = softmax(Q K^T / divisor +
    mask), O = P V.  Returns (P, O)."""
    s = np.matmul(_f(q), np.swapaxes(_f(k), -1, -2)) / F64(divisor)
    if mask is not None:
        s = s + _f(mask)
    p = softmax_rows(s)
    return p, np.matmul(p, _f(v))


def attention_backward(q, k, v, p, divisor, d_o):
    """Gradients of attention_forward by the executor's rules: the product
    rule of mult (execute.h:187-232), SFTMX_DERIVATIVE (execute.h:291-308)
    and the divide by a constant.  Returns (dQ, dK, dV)."""
    q, k, v, p, d_o = _f(q), _f(k), _f(v), _f(p), _f(d_o)
    dp = np.matmul(d_o, np.swapaxes(v, -1, -2))
    ds = softmax_backward(dp, p) / F64(divisor)
    return (np.matmul(ds, k), np.matmul(np.swapaxes(ds, -1, -2), q),
            np.matmul(np.swapaxes(p, -1, -2), d_o))
