"""Parity of the attention entry points (tl_attention_fwd / tl_attention_bwd)
with the float64 restatement of nn::MultiHeadAttention's core
(include/nn/multi_head.h:45-52, causal mask include/nn/attention.h:10-22,
softmax derivative include/passes/execute.h:291-308) in oracle/ops.py.

Configuration 3 of the benchmark plan: B=64, T=192, H=6, D=64, Q, K, V, dO
~ N(0, 1) seeded, [B, H, T, D], causal mask, divisor sqrt(64) = 8; plus
ragged, unmasked and [B, T, H, D] cases and the argument errors.

Tolerance, ||X - X_ref||_F / ||X_ref||_F per output:
  FP32 products: 1e-5.
  TF32 products: 1e-3 per TF32 product on the output's path (the single
  GEMM bound of the GEMM tests, compounded along the chain): P 1, O 2,
  dV 2, dQ and dK 3 products.  A float64 model of TF32 operand truncation
  (10-bit mantissa) on this configuration gives 0.7e-3, 1.3e-3, 1.3e-3 and
  1.9e-3 for them."""
import numpy as np
import pytest

from oracle import ops
from templit_b200 import capi
from tests.helpers import Dev

pytestmark = pytest.mark.gpu

CHAIN = {"p": 1, "o": 2, "dq": 3, "dk": 3, "dv": 2}


@pytest.fixture(scope="module")
def dev():
    return Dev()


def fro(got, want):
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64).reshape(want.shape)
    return np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30)


def inputs(B, H, T, D, seed):
    rng = np.random.default_rng(seed)
    return [rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(4)]


def run_case(dev, B, H, T, D, masked, layout, precision, seed=0, mask=None):
    q, k, v, d_o = inputs(B, H, T, D, seed)
    if mask is None and masked:
        mask = ops.causal_mask(T)
    divisor = float(np.sqrt(np.float32(D)))
    p, o = ops.attention_forward(q, k, v, divisor, mask)
    dq, dk, dv = ops.attention_backward(q, k, v, p, divisor, d_o)
    want = {"p": p, "o": o, "dq": dq, "dk": dk, "dv": dv}
    if layout == capi.TL_ATTN_BTHD:
        to = lambda x: np.ascontiguousarray(np.swapaxes(x, 1, 2))
        got = dev.attention(to(q), to(k), to(v), divisor, mask, to(d_o), layout, precision)
        got = (got[0],) + tuple(np.swapaxes(x, 1, 2) for x in got[1:])
    else:
        got = dev.attention(q, k, v, divisor, mask, d_o, layout, precision)
    errs = {n: fro(g, want[n]) for n, g in zip(("p", "o", "dq", "dk", "dv"), got)}
    for n, e in errs.items():
        bound = 1e-5 if precision == capi.TL_GEMM_FP32 else 1e-3 * CHAIN[n]
        assert e <= bound, (n, e, bound, errs)
    if masked and np.isneginf(np.triu(mask, 1)).all():  # exactly zero above the diagonal
        assert not np.triu(got[0], 1).any()
    return errs


@pytest.mark.parametrize("precision", [capi.TL_GEMM_TF32, capi.TL_GEMM_FP32])
def test_config3_causal(dev, precision):
    run_case(dev, 64, 6, 192, 64, True, capi.TL_ATTN_BHTD, precision)


def test_backward_bit_identical_across_runs(dev):
    """Configuration 3 at B 64 (768 query tiles: CTAs start while others run
    on the same SM): twelve backward passes give the same bits.  A run-to-run
    difference in a few rows of dS showed up here once two query-side CTAs
    shared an SM's tensor memory."""
    B, H, T, D = 64, 6, 192, 64
    q, k, v, d_o = inputs(B, H, T, D, 0)
    divisor = float(np.sqrt(np.float32(D)))
    mask = ops.causal_mask(T)
    first = dev.attention(q, k, v, divisor, mask, d_o, capi.TL_ATTN_BHTD, capi.TL_GEMM_TF32)
    for _ in range(11):
        got = dev.attention(q, k, v, divisor, mask, d_o, capi.TL_ATTN_BHTD, capi.TL_GEMM_TF32)
        for name, a, b in zip(("p", "o", "dq", "dk", "dv"), got, first):
            assert np.array_equal(a, b), name


@pytest.mark.parametrize("B,H,T,D,masked", [
    (2, 3, 100, 64, True),    # T not a tile multiple
    (1, 2, 37, 16, True),     # unaligned rows: CUDA-core products
    (3, 2, 64, 32, False),    # no mask
    (1, 1, 1, 8, True),       # one token
])
def test_ragged(dev, B, H, T, D, masked):
    run_case(dev, B, H, T, D, masked, capi.TL_ATTN_BHTD, capi.TL_GEMM_TF32, seed=T)


@pytest.mark.parametrize("kind", ["additive", "causal_but_one"])
def test_general_masks(dev, kind):
    """A mask that is not the causal one is read element by element: an
    arbitrary additive mask, and the causal mask with one entry changed."""
    T = 192
    rng = np.random.default_rng(11)
    if kind == "additive":
        mask = (0.5 * rng.standard_normal((T, T))).astype(np.float32)
    else:
        mask = ops.causal_mask(T).astype(np.float32)
        mask[100, 7] = -3.0
    run_case(dev, 2, 3, T, 64, True, capi.TL_ATTN_BHTD, capi.TL_GEMM_TF32, seed=4, mask=mask)


def test_heads_in_place_layout(dev):
    """[B, T, H, D] operands (the projections before the head split) give the
    same result as [B, H, T, D] ones."""
    run_case(dev, 4, 6, 192, 64, True, capi.TL_ATTN_BTHD, capi.TL_GEMM_TF32, seed=3)


def test_argument_errors(dev):
    import ctypes
    q = dev.empty((1, 1, 8, 8))
    ws = dev.ws(dev.lib.tl_attention_workspace_size(1, 8, 1, 8))
    p = dev.empty((1, 1, 8, 8))
    d = dev.t(np.asarray([1.0], np.float32))
    null = ctypes.c_void_p(0)

    def fwd(qp, layout=capi.TL_ATTN_BHTD, precision=capi.TL_GEMM_TF32, wsb=None):
        return dev.lib.tl_attention_fwd(qp, dev.p(q), dev.p(q), dev.p(d), null, dev.p(p),
                                        dev.p(q), 1, 8, 1, 8, layout, precision, dev.p(ws),
                                        ws.numel() if wsb is None else wsb, dev.stream)
    assert fwd(dev.p(q)) == capi.TL_OK
    assert fwd(null) == capi.TL_ERR_INVALID
    assert fwd(dev.p(q), layout=7) == capi.TL_ERR_INVALID
    assert fwd(dev.p(q), precision=9) == capi.TL_ERR_INVALID
    assert fwd(dev.p(q), wsb=16) == capi.TL_ERR_INVALID
    assert dev.lib.tl_attention_fwd(dev.p(q), dev.p(q), dev.p(q), dev.p(d), null, dev.p(p),
                                    dev.p(q), 0, 8, 1, 8, 0, 0, dev.p(ws), ws.numel(),
                                    dev.stream) == capi.TL_ERR_INVALID
