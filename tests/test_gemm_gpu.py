"""GEMM parity (tl_gemm: tcgen05 kind::tf32 tensor cores, and the exact-fp32
CUDA-core path) with the float64 oracle on the configuration-2 sweep
(M, N, K in {192, 384, 1536, 12288}, NN / NT / TN), the batched and
broadcast-batch products of the attention composite, and the fused
epilogues (bias, accumulate, GELU).

Tolerance (<= 1e-3 relative for TF32 paths):
  TF32: ||C - C_ref||_F / ||C_ref||_F <= 1e-3 and
        max|C - C_ref| <= 4e-3 * max|C_ref|
  FP32 and 3xTF32 (split tf32 operands on the tensor cores):
        |C - C_ref| <= 1e-5 * (|A| |B|) elementwise bound."""
import ctypes
import itertools

import numpy as np
import pytest

from oracle import ops
from templit_b200 import capi
from tests.helpers import Dev

pytestmark = pytest.mark.gpu

TF32_FRO = 1e-3
TF32_MAX = 4e-3


@pytest.fixture(scope="module")
def dev():
    return Dev()


def check_tf32(got, want):
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64).reshape(want.shape)
    err = got - want
    fro = np.linalg.norm(err) / max(np.linalg.norm(want), 1e-30)
    mx = np.abs(err).max() / max(np.abs(want).max(), 1e-30)
    assert fro <= TF32_FRO and mx <= TF32_MAX, (fro, mx)


def check_fp32(got, want, a, b, trans_a=False, trans_b=False):
    x = np.swapaxes(np.abs(a), -1, -2) if trans_a else np.abs(a)
    y = np.swapaxes(np.abs(b), -1, -2) if trans_b else np.abs(b)
    bound = 1e-5 * np.matmul(x.astype(np.float64), y.astype(np.float64)) + 1e-30
    assert np.all(np.abs(np.asarray(got, np.float64) - want) <= bound)


def operands(r, m, n, k, trans_a, trans_b, batch=()):
    a = r.standard_normal(batch + ((k, m) if trans_a else (m, k))).astype(np.float32)
    b = r.standard_normal(batch + ((n, k) if trans_b else (k, n))).astype(np.float32)
    return a, b


SWEEP = [s for s in itertools.product([192, 384, 1536], repeat=3)]


@pytest.mark.parametrize("form", ["NN", "NT", "TN"])
@pytest.mark.parametrize("m,n,k", SWEEP)
def test_sweep_tf32(dev, m, n, k, form):
    r = np.random.default_rng(m * 7 + n * 3 + k)
    ta, tb = form[0] == "T", form[1] == "T"
    a, b = operands(r, m, n, k, ta, tb)
    got = dev.gemm(a, b, trans_a=ta, trans_b=tb)
    check_tf32(got, ops.gemm(a, b, ta, tb))


@pytest.mark.parametrize("form", ["NN", "NT", "TN"])
@pytest.mark.parametrize("m,n,k", [(12288, 384, 384), (12288, 1536, 384), (12288, 384, 1536),
                                   (12288, 2048, 384), (384, 384, 12288), (384, 1536, 12288),
                                   (1536, 384, 12288)])
def test_large_tf32_sampled(dev, m, n, k, form):
    """12288-dim cases are checked on 4096 sampled outputs in float64."""
    r = np.random.default_rng(m + n + k)
    ta, tb = form[0] == "T", form[1] == "T"
    a, b = operands(r, m, n, k, ta, tb)
    got = dev.gemm(a, b, trans_a=ta, trans_b=tb)
    A = (a.T if ta else a).astype(np.float64)
    B = (b.T if tb else b).astype(np.float64)
    rows = r.integers(0, m, 4096)
    cols = r.integers(0, n, 4096)
    want = np.einsum("ij,ji->i", A[rows], B[:, cols])
    check_tf32(got[rows, cols], want)


@pytest.mark.parametrize("form", ["NN", "NT", "TN"])
@pytest.mark.parametrize("m,n,k", [(192, 192, 192), (33, 17, 65), (2, 3, 2), (128, 64, 8),
                                   (130, 258, 36)])
def test_fp32_path(dev, m, n, k, form):
    r = np.random.default_rng(m + 2 * n + 3 * k)
    ta, tb = form[0] == "T", form[1] == "T"
    a, b = operands(r, m, n, k, ta, tb)
    got = dev.gemm(a, b, trans_a=ta, trans_b=tb, precision=capi.TL_GEMM_FP32)
    check_fp32(got, ops.gemm(a, b, ta, tb), a, b, ta, tb)


@pytest.mark.parametrize("form", ["NN", "NT", "TN"])
@pytest.mark.parametrize("m,n,k", [(192, 192, 192), (384, 1536, 384), (1536, 384, 1536),
                                   (130, 258, 36), (200, 100, 600)])
def test_3xtf32_path(dev, m, n, k, form):
    """Big / small tf32 halves of both operands (three tensor-core products
    per k-step) reach the exact-fp32 bound, ragged tiles included."""
    r = np.random.default_rng(m + 5 * n + 7 * k)
    ta, tb = form[0] == "T", form[1] == "T"
    a, b = operands(r, m, n, k, ta, tb)
    d = capi.TlGemmDesc(m=m, n=n, k=k, trans_a=int(ta), trans_b=int(tb),
                        precision=capi.TL_GEMM_3XTF32)
    lda, ldb = (m if ta else k), (k if tb else n)  # TMA wants 16-byte row strides
    tc = m * n * k >= 1 << 20 and lda % 4 == 0 and ldb % 4 == 0
    assert dev.lib.tl_gemm_on_tensor_cores(ctypes.byref(d)) == int(tc)
    got = dev.gemm(a, b, trans_a=ta, trans_b=tb, precision=capi.TL_GEMM_3XTF32)
    check_fp32(got, ops.gemm(a, b, ta, tb), a, b, ta, tb)


@pytest.mark.parametrize("m,n,k,form", [(12288, 384, 384, "NN"), (384, 384, 12288, "TN"),
                                        (12288, 2048, 384, "NT")])
def test_3xtf32_large_sampled(dev, m, n, k, form):
    """Configuration-4 shapes, split-K weight gradient included, on 4096
    sampled outputs in float64 against the exact-fp32 bound."""
    r = np.random.default_rng(m + n + k + 1)
    ta, tb = form[0] == "T", form[1] == "T"
    a, b = operands(r, m, n, k, ta, tb)
    bias = r.standard_normal(n).astype(np.float32)
    got = dev.gemm(a, b, trans_a=ta, trans_b=tb, bias=bias, precision=capi.TL_GEMM_3XTF32)
    A = (a.T if ta else a).astype(np.float64)
    B = (b.T if tb else b).astype(np.float64)
    rows = r.integers(0, m, 4096)
    cols = r.integers(0, n, 4096)
    want = np.einsum("ij,ji->i", A[rows], B[:, cols]) + bias[cols]
    bound = 1e-5 * (np.einsum("ij,ji->i", np.abs(A[rows]), np.abs(B[:, cols])) + np.abs(bias[cols]))
    assert np.all(np.abs(got[rows, cols] - want) <= bound)


def test_gemm_counters(dev):
    """Launch counts by path: a product below the tensor-core threshold runs
    on the CUDA cores, one that asks for tensor cores but has a 4-byte-aligned
    operand is refused by that path and counted."""
    def counts():
        c = [ctypes.c_uint64() for _ in range(3)]
        dev.lib.tl_gemm_counters(*[ctypes.byref(x) for x in c])
        return [x.value for x in c]
    r = np.random.default_rng(1)
    a = r.standard_normal((256, 384)).astype(np.float32)
    b = r.standard_normal((384, 256)).astype(np.float32)
    t0 = counts()
    dev.gemm(a, b)
    t1 = counts()
    assert t1[0] == t0[0] + 1 and t1[1] == t0[1]
    dev.gemm(a[:8, :8], b[:8, :8])
    t2 = counts()
    assert t2[1] == t1[1] + 1 and t2[2] == t1[2]
    ta, tb = dev.t(np.concatenate([[0.0], a.ravel()]).astype(np.float32)), dev.t(b)
    tc = dev.empty((256, 256))
    d = capi.TlGemmDesc(a=ta.data_ptr() + 4, b=tb.data_ptr(), c=tc.data_ptr(), m=256, n=256,
                        k=384)
    assert dev.lib.tl_gemm_on_tensor_cores(ctypes.byref(d)) == 0
    dev.call("tl_gemm", ctypes.byref(d), dev.stream)
    t3 = counts()
    assert t3[1] == t2[1] + 1 and t3[2] == t2[2] + 1
    np.testing.assert_allclose(dev.host(tc), ops.gemm(a, b), rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("m,n,k", [(130, 258, 36), (200, 100, 60), (129, 65, 33), (192, 256, 1000)])
def test_ragged_tiles_tf32(dev, m, n, k):
    """Edges of the 128 x BN x 32 tile grid (masked rows/cols, zero-filled k)."""
    r = np.random.default_rng(17)
    for ta, tb in ((False, False), (False, True), (True, False)):
        a, b = operands(r, m, n, k, ta, tb)
        check_tf32(dev.gemm(a, b, trans_a=ta, trans_b=tb), ops.gemm(a, b, ta, tb))


def test_attention_batched_and_broadcast(dev):
    """QK^T and PV of the attention composite (nn/multi_head.h:45-52), batch
    [64, 6], and a broadcast batch operand."""
    r = np.random.default_rng(3)
    q = r.standard_normal((64, 6, 192, 64)).astype(np.float32)
    kt = r.standard_normal((64, 6, 64, 192)).astype(np.float32)
    check_tf32(dev.gemm(q, kt), ops.matmul(q, kt))
    # the 192-wide tile in every operand form, with the epilogue extras
    check_tf32(dev.gemm(q, q, trans_b=True), ops.gemm(q, q, False, True))
    check_tf32(dev.gemm(kt, kt, trans_a=True), ops.gemm(kt, kt, True, False))
    bias = r.standard_normal((192,)).astype(np.float32)
    add = r.standard_normal((64, 6, 192, 192)).astype(np.float32)
    prod = dev.gemm(q, kt, bias=bias)
    check_tf32(prod, ops.gemm(q, kt, bias=bias))
    np.testing.assert_array_equal(dev.gemm(q, kt, bias=bias, addend=add),
                                  dev.binary("add", add, prod, prod.shape))
    p = r.random((64, 6, 192, 192)).astype(np.float32)
    v = r.standard_normal((64, 6, 192, 64)).astype(np.float32)
    check_tf32(dev.gemm(p, v), ops.matmul(p, v))
    w = r.standard_normal((384, 384)).astype(np.float32)
    x = r.standard_normal((64, 192, 384)).astype(np.float32)
    check_tf32(dev.gemm(x, w), ops.matmul(x, w))
    xb = r.standard_normal((4, 1, 96, 40)).astype(np.float32)
    yb = r.standard_normal((1, 3, 40, 72)).astype(np.float32)
    check_tf32(dev.gemm(xb, yb), ops.matmul(xb, yb))
    # batched transposed forms (weight gradient as one K = B*T product is the
    # fused path; the executor's batched [64,384,192] x [64,192,N] as well)
    xt = r.standard_normal((8, 192, 384)).astype(np.float32)
    g = r.standard_normal((8, 192, 256)).astype(np.float32)
    check_tf32(dev.gemm(xt, g, trans_a=True), ops.gemm(xt, g, True, False))


def test_epilogues(dev):
    r = np.random.default_rng(4)
    a = r.standard_normal((512, 384)).astype(np.float32)
    b = r.standard_normal((384, 1536)).astype(np.float32)
    bias = r.standard_normal((1536,)).astype(np.float32)
    c0 = r.standard_normal((512, 1536)).astype(np.float32)
    out, g = dev.gemm(a, b, bias=bias, gelu=True)
    want = ops.gemm(a, b, bias=bias)
    check_tf32(out, want)
    check_tf32(g, ops.gelu(want))
    acc = dev.gemm(a, b, c=c0, beta=1.0)
    check_tf32(acc, ops.gemm(a, b, c=c0, beta=1.0))
    # addend (a residual or gradient added to the product): bit-identical to
    # the product followed by the separate add kernel
    prod = dev.gemm(a, b, bias=bias)
    np.testing.assert_array_equal(dev.gemm(a, b, bias=bias, addend=c0),
                                  dev.binary("add", c0, prod, prod.shape))
    k_long = r.standard_normal((12288, 64)).astype(np.float32)  # split-K path
    g_long = r.standard_normal((12288, 96)).astype(np.float32)
    add = r.standard_normal((64, 96)).astype(np.float32)
    prod = dev.gemm(k_long, g_long, trans_a=True)
    np.testing.assert_array_equal(dev.gemm(k_long, g_long, trans_a=True, addend=add),
                                  dev.binary("add", add, prod, prod.shape))
    out32, g32 = dev.gemm(a[:64], b, bias=bias, gelu=True, precision=capi.TL_GEMM_FP32)
    np.testing.assert_array_equal(dev.gemm(a[:64], b, bias=bias, addend=c0[:64],
                                           precision=capi.TL_GEMM_FP32),
                                  dev.binary("add", c0[:64], out32, out32.shape))
    np.testing.assert_allclose(out32, ops.gemm(a[:64], b, bias=bias), rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose(g32, ops.gelu(ops.gemm(a[:64], b, bias=bias)), rtol=1e-4, atol=1e-3)


def test_zero_and_empty(dev):
    r = np.random.default_rng(5)
    a = np.zeros((256, 128), np.float32)
    b = r.standard_normal((128, 256)).astype(np.float32)
    assert np.all(dev.gemm(a, b) == 0)
    # identity: exact in TF32 for small integers (tests/test_metal_runtime.cpp:307-342)
    eye = np.broadcast_to(np.eye(64, dtype=np.float32), (2, 64, 64)).copy()
    vals = (np.arange(2 * 64 * 64) % 31 - 15).astype(np.float32).reshape(2, 64, 64)
    np.testing.assert_array_equal(dev.gemm(eye, vals), vals)
    big = np.broadcast_to(np.eye(256, dtype=np.float32), (3, 256, 256)).copy()
    vb = (np.arange(3 * 256 * 256) % 31 - 15).astype(np.float32).reshape(3, 256, 256)
    np.testing.assert_array_equal(dev.gemm(big, vb), vb)


def _strided_gemm(dev, a, b, c_shape, m, n, k, trans_a, trans_b, batch, sa, sb, sc,
                  lda, ldb, ldc, precision):
    """tl_gemm on raw buffers with explicit strides; returns C's buffer."""
    ta, tb = dev.t(a), dev.t(b)
    tc = dev.empty(c_shape)
    d = capi.TlGemmDesc()
    d.a, d.b, d.c = ta.data_ptr(), tb.data_ptr(), tc.data_ptr()
    d.m, d.n, d.k = m, n, k
    d.trans_a, d.trans_b = int(trans_a), int(trans_b)
    d.precision = precision
    d.batch_rank = len(batch)
    for i, s in enumerate(batch):
        d.batch_shape[i] = s
        d.a_batch_stride[i], d.b_batch_stride[i], d.c_batch_stride[i] = sa[i], sb[i], sc[i]
    d.lda, d.ldb, d.ldc = lda, ldb, ldc
    nbytes = dev.lib.tl_gemm_workspace_size(ctypes.byref(d))
    ws = dev.ws(nbytes) if nbytes else None
    if ws is not None:
        d.workspace, d.workspace_bytes = ws.data_ptr(), nbytes
    dev.call("tl_gemm", ctypes.byref(d), dev.stream)
    return dev.host(tc)


@pytest.mark.parametrize("precision", [capi.TL_GEMM_TF32, capi.TL_GEMM_FP32,
                                       capi.TL_GEMM_3XTF32])
def test_head_strided_operands(dev, precision):
    """Attention heads read and written in place in [B, T, H, D] tensors:
    batch dims (B, H) with strides (T*H*D, D), row stride H*D."""
    r = np.random.default_rng(21)
    B, T, H, D = 8, 192, 6, 64
    q = r.standard_normal((B, T, H, D)).astype(np.float32)
    kk = r.standard_normal((B, T, H, D)).astype(np.float32)
    v = r.standard_normal((B, T, H, D)).astype(np.float32)
    qh, kh, vh = (np.swapaxes(x, 1, 2) for x in (q, kk, v))  # [B, H, T, D] views
    hs = (T * H * D, D)
    # S = Qh Kh^T (NT): C dense [B, H, T, T]
    s = _strided_gemm(dev, q, kk, (B, H, T, T), T, T, D, False, True, (B, H), hs, hs,
                      (H * T * T, T * T), H * D, H * D, 0, precision)
    want = np.matmul(qh.astype(np.float64), np.swapaxes(kh, -1, -2).astype(np.float64))
    check = check_tf32 if precision == capi.TL_GEMM_TF32 else (
        lambda g, w: np.testing.assert_allclose(g, w, rtol=1e-4, atol=1e-3))
    check(s, want)
    # O = P Vh written straight into [B, T, H, D] (C row stride H*D)
    p = r.random((B, H, T, T)).astype(np.float32)
    o = _strided_gemm(dev, p, v, (B, T, H, D), T, D, T, False, False, (B, H),
                      (H * T * T, T * T), hs, hs, 0, H * D, H * D, precision)
    want = np.swapaxes(np.matmul(p.astype(np.float64), vh.astype(np.float64)), 1, 2)
    check(o, want)
    # dK^T-style TN product from a head view: Qh^T P (A stored [K=T, M=D], lda = H*D)
    g = _strided_gemm(dev, q, p, (B, H, D, T), D, T, T, True, False, (B, H), hs,
                      (H * T * T, T * T), (H * D * T, D * T), H * D, 0, 0, precision)
    want = np.matmul(np.swapaxes(qh, -1, -2).astype(np.float64), p.astype(np.float64))
    check(g, want)


def _grouped(dev, mode, a_list, b_list, m, n, k, trans_a, trans_b, bias_list=None,
             precision=capi.TL_GEMM_TF32):
    """tl_gemm with group_mode; returns the output(s)."""
    ta = [dev.t(a) for a in a_list]
    tb = [dev.t(b) for b in b_list]
    groups = len(b_list)
    outs = [dev.empty((m, n)) for _ in range(groups if mode == capi.TL_GEMM_GROUP_N else 1)]
    tbias = [dev.t(b) for b in bias_list] if bias_list else None
    d = capi.TlGemmDesc()
    d.a, d.b, d.c = ta[0].data_ptr(), tb[0].data_ptr(), outs[0].data_ptr()
    d.m, d.n, d.k = m, n, k
    d.trans_a, d.trans_b = int(trans_a), int(trans_b)
    d.precision = precision
    d.group_mode, d.groups = mode, groups
    for i in range(groups):
        d.a_group[i] = ta[min(i, len(ta) - 1)].data_ptr()
        d.b_group[i] = tb[i].data_ptr()
        if mode == capi.TL_GEMM_GROUP_N:
            d.c_group[i] = outs[i].data_ptr()
            if tbias:
                d.bias_group[i] = tbias[i].data_ptr()
    nbytes = dev.lib.tl_gemm_workspace_size(ctypes.byref(d))
    ws = dev.ws(nbytes) if nbytes else None
    if ws is not None:
        d.workspace, d.workspace_bytes = ws.data_ptr(), nbytes
    dev.call("tl_gemm", ctypes.byref(d), dev.stream)
    return [dev.host(o) for o in outs]


@pytest.mark.parametrize("precision", [capi.TL_GEMM_TF32, capi.TL_GEMM_FP32,
                                       capi.TL_GEMM_3XTF32])
def test_grouped_products(dev, precision):
    """One launch for the Q, K and V projections of one input (N groups),
    for their weight gradients (N groups, split K), and for the input
    gradient summed over the three (K groups)."""
    r = np.random.default_rng(23)

    def check(g, w, a, b, ta=False, tb=False):
        if precision == capi.TL_GEMM_TF32:
            check_tf32(g, w)
        else:  # FP32 and 3xTF32: the exact-fp32 bound
            check_fp32(g, w, a, b, ta, tb)
    x = r.standard_normal((2048, 384)).astype(np.float32)
    ws = [r.standard_normal((384, 384)).astype(np.float32) for _ in range(3)]
    bs = [r.standard_normal((384,)).astype(np.float32) for _ in range(3)]
    outs = _grouped(dev, capi.TL_GEMM_GROUP_N, [x], ws, 2048, 384, 384, False, False, bs,
                    precision)
    for o, w, b in zip(outs, ws, bs):
        check(o - b, ops.gemm(x, w), x, w)
    # weight gradients: X^T dY_g, K = 12288 (split-K slices per group)
    xl = r.standard_normal((12288, 384)).astype(np.float32)
    dys = [r.standard_normal((12288, 384)).astype(np.float32) for _ in range(3)]
    outs = _grouped(dev, capi.TL_GEMM_GROUP_N, [xl], dys, 384, 384, 12288, True, False, bs,
                    precision=precision)
    for o, dy, b in zip(outs, dys, bs):  # one slice-sum launch, each group its bias
        check(o - b, ops.gemm(xl, dy, True, False), xl, dy, True, False)
    # input gradient: sum_g dY_g W_g^T over the concatenated K
    gs = [r.standard_normal((2048, 384)).astype(np.float32) for _ in range(3)]
    (out,) = _grouped(dev, capi.TL_GEMM_GROUP_K, gs, ws, 2048, 384, 384, False, True,
                      precision=precision)
    want = sum(ops.gemm(g, w, False, True) for g, w in zip(gs, ws))
    check(out, want, np.concatenate(gs, axis=1), np.concatenate(ws, axis=1), False, True)


@pytest.mark.parametrize("m,n,k,form,precision", [
    (12288, 1536, 384, "NT", capi.TL_GEMM_TF32),   # the FFN's dH = dY W2^T
    (384, 384, 12288, "TN", capi.TL_GEMM_TF32),    # split-K: the slice-sum kernel's epilogue
    (100, 70, 40, "NN", capi.TL_GEMM_TF32),        # ragged: per-thread stores
    (257, 96, 64, "NT", capi.TL_GEMM_FP32),        # CUDA-core path
    (12288, 1536, 384, "NT", capi.TL_GEMM_3XTF32),
])
def test_gelu_backward_epilogue(dev, m, n, k, form, precision):
    """C = GELU'(x) * (A B): bit-identical to the product followed by the GELU
    backward kernel (the executor's GELU_derivative then hadamard)."""
    rng = np.random.default_rng(m + n)
    ta, tb = form[0] == "T", form[1] == "T"
    a = rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32) / 8
    x = rng.standard_normal((m, n)).astype(np.float32)
    prod = dev.gemm(a, b, trans_a=ta, trans_b=tb, precision=precision)
    want = dev.gelu_backward(x, prod)
    got = dev.gemm(a, b, trans_a=ta, trans_b=tb, precision=precision, gelu_grad_x=x)
    np.testing.assert_array_equal(got, want)


@pytest.mark.parametrize("precision", [capi.TL_GEMM_TF32, capi.TL_GEMM_3XTF32])
@pytest.mark.parametrize("groups", [1, 3])
def test_head_split_store(dev, groups, precision):
    """C stored as [B, H, T, D] (tl_gemm_desc.c_heads): the query / key /
    value projections of nn::MultiHeadAttention with split_heads folded into
    the store.  Bit-identical to the [M, N] product transposed afterwards."""
    B, T, H, D, K = 4, 64, 6, 64, 128
    M, N = B * T, H * D
    r = np.random.default_rng(11)
    x = r.standard_normal((M, K)).astype(np.float32)
    ws = [r.standard_normal((K, N)).astype(np.float32) / 8 for _ in range(groups)]
    bs = [r.standard_normal(N).astype(np.float32) for _ in range(groups)]
    plain = [dev.gemm(x, w, bias=b, precision=precision) for w, b in zip(ws, bs)]
    tx = dev.t(x)
    tw, tb = [dev.t(w) for w in ws], [dev.t(b) for b in bs]
    outs = [dev.empty((B, H, T, D)) for _ in range(groups)]
    d = capi.TlGemmDesc(a=tx.data_ptr(), b=tw[0].data_ptr(), c=outs[0].data_ptr(),
                        bias=tb[0].data_ptr(), m=M, n=N, k=K, precision=precision)
    d.c_heads, d.c_head_rows = H, T
    if groups > 1:
        d.group_mode, d.groups = capi.TL_GEMM_GROUP_N, groups
        for i in range(groups):
            d.b_group[i], d.c_group[i] = tw[i].data_ptr(), outs[i].data_ptr()
            d.bias_group[i] = tb[i].data_ptr()
    lib = capi.cuda_lib()
    capi.check(lib.tl_gemm(ctypes.byref(d), dev.stream), lib, "tl_gemm heads")
    for o, p_ in zip(outs, plain):
        np.testing.assert_array_equal(dev.host(o), p_.reshape(B, T, H, D).transpose(0, 2, 1, 3))
    d.c_head_rows = 48  # rows of a head not a multiple of 32: refused
    assert lib.tl_gemm(ctypes.byref(d), dev.stream) == capi.TL_ERR_INVALID
