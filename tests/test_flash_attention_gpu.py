"""Parity of the flash attention kernels (tl_flash_attention_*: any T, the
forward keeps only O and the row log-sum-exp, the backward recomputes P on
the tensor cores) with the float64 restatement of nn::MultiHeadAttention's
core (include/nn/multi_head.h:45-52, causal mask include/nn/attention.h:
10-22, softmax derivative include/passes/execute.h:291-308) in oracle/ops.py.

Cases: configuration 3 (B 64, T 192, H 6, D 64, causal, divisor 8), the
configuration-5 sequence length (T 1024), a T that is not a block multiple,
no mask, an arbitrary additive mask, heads read in place from [B, T, H, D]
tensors, K stored transposed (the executor's K^T copy), and the
probabilities rebuilt from the log-sum-exp.

Tolerance, ||X - X_ref||_F / ||X_ref||_F per output, TF32 products: 1e-3
per TF32 product on the output's path (as the fused-attention tests): P 1,
O 2, dV 2, dQ and dK 3; the log-sum-exp within 3e-3 relative (its error is
the TF32 error of the row's largest scores; measured up to 1.35e-3).  With
a single token the exact dQ and dK are zero (dS = P (dP - rowsum(dP P)) with
P = 1) and the kernels' rowsum(dO O) leaves TF32 rounding there instead, so
that case bounds them absolutely.  Repeated runs are bit-identical (no
atomics)."""
import ctypes

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


def view(t, layout, k_trans=False):
    """tl_attn_view of a device tensor: [B, H, T, D], [B, T, H, D] or, with
    k_trans, [B, H, D, T]."""
    v = capi.TlAttnView()
    v.p = t.data_ptr()
    s = t.stride()
    if k_trans:  # [B, H, D, T]
        v.batch_stride, v.head_stride, v.row_stride, v.transposed = s[0], s[1], s[2], 1
    elif layout == "bthd":
        v.batch_stride, v.head_stride, v.row_stride = s[0], s[2], s[1]
    else:
        v.batch_stride, v.head_stride, v.row_stride = s[0], s[1], s[2]
    return v


def oracle_lse(q, k, divisor, mask):
    s = np.matmul(q.astype(np.float64), np.swapaxes(k.astype(np.float64), -1, -2)) / divisor
    if mask is not None:
        s = s + mask.astype(np.float64)
    m = s.max(-1, keepdims=True)
    return (m + np.log(np.exp(s - m).sum(-1, keepdims=True)))[..., 0]


def run(dev, B, H, T, seed=0, causal=True, mask=None, layout="bhtd", k_trans=False,
        check_probs=False, repeat=False):
    D = 64
    rng = np.random.default_rng(seed)
    q, k, v, d_o = (rng.standard_normal((B, H, T, D)).astype(np.float32) for _ in range(4))
    if mask is None and causal:
        mask = ops.causal_mask(T).astype(np.float32)
    divisor = float(np.sqrt(np.float32(D)))
    p, o = ops.attention_forward(q, k, v, divisor, mask)
    dq, dk, dv = ops.attention_backward(q, k, v, p, divisor, d_o)
    want = {"o": o, "dq": dq, "dk": dk, "dv": dv}
    lse_want = oracle_lse(q, k, divisor, mask)

    def dev_t(x, kt=False):
        if kt:
            return dev.t(np.ascontiguousarray(np.swapaxes(x, -1, -2)))
        if layout == "bthd":
            return dev.t(np.ascontiguousarray(np.swapaxes(x, 1, 2)))
        return dev.t(x)

    tq, tk, tv, tdo = dev_t(q), dev_t(k, k_trans), dev_t(v), dev_t(d_o)
    to, tdq, tdk, tdv = (dev_t(np.zeros_like(q)) for _ in range(4))
    tdiv = dev.t(np.asarray([divisor], np.float32))
    tmask = dev.t(mask) if mask is not None else None
    flag = dev.torch.zeros(4, dtype=dev.torch.int32, device=dev.dev)
    lse = dev.empty((B, H, T))
    delta = dev.empty((B, H, T))
    d = capi.TlFlashDesc(B=B, T=T, H=H, D=D)
    d.q, d.k, d.v = view(tq, layout), view(tk, layout, k_trans), view(tv, layout)
    d.o, d.d_o = view(to, layout), view(tdo, layout)
    d.dq, d.dk, d.dv = view(tdq, layout), view(tdk, layout), view(tdv, layout)
    d.divisor = tdiv.data_ptr()
    d.lse, d.delta = lse.data_ptr(), delta.data_ptr()
    if tmask is not None:
        d.mask = tmask.data_ptr()
        d.mask_flag = flag.data_ptr()
        dev.call("tl_attention_mask_check", ctypes.c_void_p(tmask.data_ptr()), T,
                 ctypes.c_void_p(flag.data_ptr()), dev.stream)
        is_causal = bool(np.array_equal(mask, ops.causal_mask(T).astype(np.float32)))
        assert int(dev.host(flag)[0]) == int(is_causal)
    assert dev.lib.tl_flash_attention_supported(ctypes.byref(d)) == 1
    dev.call("tl_flash_attention_fwd", ctypes.byref(d), dev.stream)
    dev.call("tl_flash_attention_bwd", ctypes.byref(d), dev.stream)

    def host(t):
        x = dev.host(t)
        return np.swapaxes(x, 1, 2) if layout == "bthd" else x
    got = {"o": host(to), "dq": host(tdq), "dk": host(tdk), "dv": host(tdv)}
    errs = {n: fro(got[n], want[n]) for n in want}
    lse_err = float((np.abs(dev.host(lse) - lse_want) / np.abs(lse_want).clip(1.0)).max())
    print(f"B {B} H {H} T {T} {layout}{' K^T' if k_trans else ''}: {errs}, lse {lse_err:.2e}")
    for n, e in errs.items():
        if T == 1 and n in ("dq", "dk"):
            assert np.abs(got[n]).max() <= 5e-2, (n, np.abs(got[n]).max())
            continue
        assert e <= 1e-3 * CHAIN[n], (n, e, errs)
    assert lse_err <= 3e-3
    if check_probs:
        tp = dev.empty((B, H, T, T))
        dev.call("tl_flash_attention_probs", ctypes.byref(d), ctypes.c_void_p(tp.data_ptr()),
                 dev.stream)
        gp = dev.host(tp)
        assert fro(gp, p) <= 1e-3 * CHAIN["p"]
        if mask is not None and np.array_equal(mask, ops.causal_mask(T).astype(np.float32)):
            assert not np.triu(gp, 1).any()
    if repeat:
        first = {n: x.copy() for n, x in got.items()}
        dev.call("tl_flash_attention_fwd", ctypes.byref(d), dev.stream)
        dev.call("tl_flash_attention_bwd", ctypes.byref(d), dev.stream)
        again = {"o": host(to), "dq": host(tdq), "dk": host(tdk), "dv": host(tdv)}
        for n in first:
            np.testing.assert_array_equal(first[n], again[n])
    return errs


def test_config3_causal(dev):
    run(dev, 64, 6, 192, seed=1, check_probs=True, repeat=True)


def test_config5_sequence_length(dev):
    run(dev, 2, 3, 1024, seed=2)


@pytest.mark.parametrize("T", [100, 37, 1, 320])
def test_ragged_lengths(dev, T):
    run(dev, 2, 3, T, seed=T)


def test_no_mask(dev):
    run(dev, 3, 2, 256, seed=4, causal=False)


@pytest.mark.parametrize("kind", ["additive", "causal_but_one"])
def test_general_masks(dev, kind):
    T = 192
    rng = np.random.default_rng(11)
    if kind == "additive":
        mask = (0.5 * rng.standard_normal((T, T))).astype(np.float32)
    else:
        mask = ops.causal_mask(T).astype(np.float32)
        mask[100, 7] = -3.0
    run(dev, 2, 3, T, seed=5, mask=mask, check_probs=True)


def test_heads_in_place_layout(dev):
    run(dev, 4, 6, 192, seed=3, layout="bthd")


@pytest.mark.parametrize("T", [192, 1024])
def test_k_transposed(dev, T):
    run(dev, 2, 6, T, seed=6, k_trans=True)


def test_argument_errors(dev):
    d = capi.TlFlashDesc(B=1, T=8, H=1, D=32)
    assert dev.lib.tl_flash_attention_supported(ctypes.byref(d)) == 0
    assert dev.lib.tl_flash_attention_fwd(ctypes.byref(d), dev.stream) == capi.TL_ERR_UNSUPPORTED
    d.D = 64
    assert dev.lib.tl_flash_attention_fwd(ctypes.byref(d), dev.stream) == capi.TL_ERR_INVALID
