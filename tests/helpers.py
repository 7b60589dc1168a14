"""Shared helpers for the tests: known-answer fixtures, and thin wrappers
that run one C-ABI kernel of include/templit_cuda.h on torch-allocated
device memory (torch is only the device allocator / stream here)."""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np

from templit_b200 import capi

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def known_answers():
    with open(os.path.join(GOLDEN, "known_answers.json")) as f:
        return json.load(f)["cases"]


# ---------------------------------------------------------------- device side
class Dev:
    """Runs C-ABI kernels on the current torch CUDA stream."""

    def __init__(self):
        import torch
        self.torch = torch
        self.lib = capi.cuda_lib()
        self.dev = torch.device("cuda", torch.cuda.current_device())

    @property
    def stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    def t(self, arr, dtype=np.float32):
        a = np.ascontiguousarray(np.asarray(arr, dtype=dtype))
        return self.torch.from_numpy(a).to(self.dev)

    def empty(self, shape, dtype=None):
        return self.torch.empty(tuple(int(s) for s in shape),
                                dtype=dtype or self.torch.float32, device=self.dev)

    def ws(self, nbytes):
        return self.torch.empty(max(int(nbytes), 16), dtype=self.torch.uint8, device=self.dev)

    @staticmethod
    def p(x):
        return ctypes.c_void_p(x.data_ptr()) if x is not None else ctypes.c_void_p(0)

    def host(self, x):
        self.torch.cuda.synchronize()
        return x.cpu().numpy()

    def call(self, name, *args):
        rc = getattr(self.lib, name)(*args)
        capi.check(rc, self.lib, name)

    def status(self):
        flags = ctypes.c_uint32(0)
        capi.check(self.lib.tl_device_status(ctypes.byref(flags), self.stream), self.lib,
                   "tl_device_status")
        return flags.value

    # --- one wrapper per op family -----------------------------------------
    def binary(self, kind, a, b, out_shape):
        op = {"add": capi.TL_ADD, "sub": capi.TL_SUB, "mul": capi.TL_MUL, "div": capi.TL_DIV}[kind]
        a = np.asarray(a, np.float32)
        b = np.asarray(b, np.float32)
        ta, tb = self.t(a), self.t(b)
        out = self.empty(out_shape)
        self.call("tl_binary", op, self.p(ta), capi.shape_arr(a.shape), a.ndim, self.p(tb),
                  capi.shape_arr(b.shape), b.ndim, self.p(out), capi.shape_arr(out_shape),
                  len(out_shape), self.stream)
        return self.host(out)

    def scalar(self, kind, x, s):
        op = {"add": capi.TL_SCALAR_ADD, "div": capi.TL_SCALAR_DIV, "pow": capi.TL_SCALAR_POW}[kind]
        tx = self.t(x)
        out = self.empty(tx.shape)
        self.call("tl_scalar", op, self.p(tx), ctypes.c_float(s), self.p(out), tx.numel(), self.stream)
        return self.host(out)

    def unary(self, kind, x):
        op = {"sigmoid": capi.TL_SIGMOID, "sqrt": capi.TL_SQRT, "exp": capi.TL_EXP,
              "gelu": capi.TL_GELU, "gelu_derivative": capi.TL_GELU_DERIVATIVE}[kind]
        tx = self.t(x)
        out = self.empty(tx.shape)
        self.call("tl_unary", op, self.p(tx), self.p(out), tx.numel(), self.stream)
        return self.host(out)

    def gelu_backward(self, x, g):
        tx, tg = self.t(x), self.t(g)
        out = self.empty(tx.shape)
        self.call("tl_gelu_backward", self.p(tx), self.p(tg), self.p(out), tx.numel(), self.stream)
        return self.host(out)

    def reduce(self, kind, x, out_shape):
        op = capi.TL_REDUCE_SUM if kind == "sum" else capi.TL_REDUCE_MAX
        x = np.asarray(x, np.float32)
        tx = self.t(x)
        xs, os_ = capi.shape_arr(x.shape), capi.shape_arr(out_shape)
        nbytes = self.lib.tl_reduce_workspace_size(xs, x.ndim, os_, len(out_shape))
        ws = self.ws(nbytes)
        out = self.empty(out_shape)
        self.call("tl_reduce", op, self.p(tx), xs, x.ndim, self.p(out), os_, len(out_shape),
                  self.p(ws), nbytes, self.stream)
        return self.host(out)

    def argmax(self, x):
        tx = self.t(np.asarray(x, np.float32).ravel())
        nbytes = self.lib.tl_argmax_workspace_size(tx.numel())
        ws = self.ws(nbytes)
        out = self.torch.zeros(1, dtype=self.torch.int32, device=self.dev)
        self.call("tl_argmax", self.p(tx), tx.numel(), self.p(out), self.p(ws), nbytes, self.stream)
        return int(self.host(out).view(np.uint32)[0])

    def transpose(self, x, da, db):
        x = np.asarray(x, np.float32)
        tx = self.t(x)
        out = self.empty(np.swapaxes(x, da, db).shape)
        self.call("tl_transpose", self.p(tx), capi.shape_arr(x.shape), x.ndim, da, db, self.p(out),
                  self.stream)
        return self.host(out)

    def rows(self, name, *arrays, extra_out=False):
        x = np.asarray(arrays[0], np.float32)
        cols = x.shape[-1]
        rows = x.size // cols if cols else 0
        ts = [self.t(a) for a in arrays]
        if name == "rms":
            out = self.empty(x.shape[:-1] + (1,))
        else:
            out = self.empty(x.shape)
        args = [self.p(t) for t in ts]
        if name in ("softmax_bwd", "rmsnorm_bwd"):
            args.append(ctypes.c_void_p(0))  # no divisor / addend
        args.append(self.p(out))
        if name == "rmsnorm":
            args.append(ctypes.c_void_p(0))
        self.call({"softmax": "tl_softmax_rows", "softmax_bwd": "tl_softmax_backward_rows",
                   "rms": "tl_rms_rows", "rmsnorm": "tl_rmsnorm_rows",
                   "rmsnorm_bwd": "tl_rmsnorm_backward_rows"}[name], *args, rows, cols, self.stream)
        return self.host(out)

    def softmax_scaled_masked(self, x, divisor=None, mask=None):
        x = np.asarray(x, np.float32)
        cols = x.shape[-1]
        tx = self.t(x)
        td = self.t(np.asarray([divisor], np.float32)) if divisor is not None else None
        tm = self.t(np.asarray(mask, np.float32)) if mask is not None else None
        mask_rows = (np.asarray(mask).size // cols) if mask is not None else 0
        out = self.empty(x.shape)
        self.call("tl_softmax_scaled_masked_rows", self.p(tx), self.p(td), self.p(tm), mask_rows,
                  self.p(out), x.size // cols, cols, self.stream)
        return self.host(out)

    def attention(self, q, k, v, divisor, mask=None, d_o=None, layout=capi.TL_ATTN_BHTD,
                  precision=capi.TL_GEMM_TF32):
        """tl_attention_fwd (and tl_attention_bwd when d_o is given) on
        operands in `layout`; returns (p, o) or (p, o, dq, dk, dv)."""
        q, k, v = (np.asarray(x, np.float32) for x in (q, k, v))
        if layout == capi.TL_ATTN_BHTD:
            B, H, T, D = q.shape
        else:
            B, T, H, D = q.shape
        tq, tk, tv = self.t(q), self.t(k), self.t(v)
        td = self.t(np.asarray([divisor], np.float32))
        tm = self.t(np.asarray(mask, np.float32)) if mask is not None else None
        ws = self.ws(self.lib.tl_attention_workspace_size(B, T, H, D))
        p, o = self.empty((B, H, T, T)), self.empty(q.shape)
        self.call("tl_attention_fwd", self.p(tq), self.p(tk), self.p(tv), self.p(td), self.p(tm),
                  self.p(p), self.p(o), B, T, H, D, layout, precision, self.p(ws), ws.numel(),
                  self.stream)
        if d_o is None:
            return self.host(p), self.host(o)
        tg = self.t(d_o)
        dq, dk, dv = self.empty(q.shape), self.empty(q.shape), self.empty(q.shape)
        self.call("tl_attention_bwd", self.p(tq), self.p(tk), self.p(tv), self.p(p), self.p(td),
                  self.p(tg), self.p(dq), self.p(dk), self.p(dv), B, T, H, D, layout, precision,
                  self.p(ws), ws.numel(), self.stream)
        return tuple(self.host(x) for x in (p, o, dq, dk, dv))

    def softmax_bwd_div(self, g, y, divisor):
        g = np.asarray(g, np.float32)
        cols = g.shape[-1]
        tg, ty = self.t(g), self.t(y)
        td = self.t(np.asarray([divisor], np.float32))
        out = self.empty(g.shape)
        self.call("tl_softmax_backward_rows", self.p(tg), self.p(ty), self.p(td), self.p(out),
                  g.size // cols, cols, self.stream)
        return self.host(out)

    def rmsnorm_bwd_add(self, g, x, y, addend, in_place=False):
        g = np.asarray(g, np.float32)
        cols = g.shape[-1]
        tg, tx, ty, ta = self.t(g), self.t(x), self.t(y), self.t(addend)
        out = ta if in_place else self.empty(g.shape)
        self.call("tl_rmsnorm_backward_rows", self.p(tg), self.p(tx), self.p(ty), self.p(ta),
                  self.p(out), g.size // cols, cols, self.stream)
        return self.host(out)

    def xent(self, logits, targets, backward=False, row_scale=None):
        z = np.asarray(logits, np.float32)
        t = np.asarray(targets, np.uint32)
        tz, tt = self.t(z), self.t(t.view(np.int32), dtype=np.int32)
        vocab = z.shape[-1]
        rows = t.size
        if backward:
            out = self.empty(z.shape)
            ts = self.t(row_scale) if row_scale is not None else None
            self.call("tl_xent_backward_rows", self.p(tz), self.p(tt), self.p(ts), self.p(out),
                      rows, vocab, self.stream)
        else:
            out = self.empty(t.shape + (1,))
            self.call("tl_xent_rows", self.p(tz), self.p(tt), self.p(out), rows, vocab, self.stream)
        return self.host(out)

    def gather(self, w, ids):
        w = np.asarray(w, np.float32)
        ids = np.asarray(ids, np.uint32)
        tw, ti = self.t(w), self.t(ids.view(np.int32), dtype=np.int32)
        out = self.empty(ids.shape + (w.shape[1],))
        self.call("tl_embedding_gather", self.p(tw), w.shape[0], w.shape[1], self.p(ti), ids.size,
                  self.p(out), self.stream)
        return self.host(out)

    def scatter(self, values, ids, n_rows, base=None):
        v = np.asarray(values, np.float32)
        ids = np.asarray(ids, np.uint32)
        dim = v.shape[-1]
        tv, ti = self.t(v), self.t(ids.view(np.int32), dtype=np.int32)
        tb = self.t(base) if base is not None else None
        out = self.empty((n_rows, dim))
        nbytes = self.lib.tl_embedding_scatter_workspace_size(ids.size, n_rows, dim)
        ws = self.ws(nbytes)
        self.call("tl_embedding_scatter_add", self.p(tv), self.p(ti), ids.size, dim, self.p(tb),
                  self.p(out), n_rows, self.p(ws), nbytes, self.stream)
        return self.host(out)

    def gemm(self, a, b, trans_a=False, trans_b=False, bias=None, c=None, beta=0.0, gelu=False,
             precision=capi.TL_GEMM_TF32, addend=None, gelu_grad_x=None):
        a = np.asarray(a, np.float32)
        b = np.asarray(b, np.float32)
        ta, tb = self.t(a), self.t(b)
        m = a.shape[-1] if trans_a else a.shape[-2]
        k = a.shape[-2] if trans_a else a.shape[-1]
        n = b.shape[-2] if trans_b else b.shape[-1]
        batch = np.broadcast_shapes(a.shape[:-2], b.shape[:-2])
        out_shape = tuple(batch) + (m, n)
        tc = self.t(np.broadcast_to(np.asarray(c, np.float32), out_shape)) if c is not None \
            else self.empty(out_shape)
        tg = self.empty(out_shape) if gelu else None
        tbias = self.t(bias) if bias is not None else None
        tadd = self.t(np.broadcast_to(np.asarray(addend, np.float32), out_shape)) \
            if addend is not None else None
        tgx = self.t(np.broadcast_to(np.asarray(gelu_grad_x, np.float32), out_shape)) \
            if gelu_grad_x is not None else None
        d = capi.TlGemmDesc()
        d.addend = tadd.data_ptr() if tadd is not None else None
        d.gelu_grad_x = tgx.data_ptr() if tgx is not None else None
        d.a, d.b, d.c = ta.data_ptr(), tb.data_ptr(), tc.data_ptr()
        d.bias = tbias.data_ptr() if tbias is not None else None
        d.gelu_out = tg.data_ptr() if tg is not None else None
        d.m, d.n, d.k = m, n, k
        d.trans_a, d.trans_b = int(trans_a), int(trans_b)
        d.precision = precision
        d.beta = beta
        d.batch_rank = len(batch)

        def strides(shape, mat):
            full = (1,) * (len(batch) - (len(shape) - 2)) + tuple(shape[:-2])
            st, acc = [], mat
            for s in reversed(full):
                st.append(0 if s == 1 else acc)
                acc *= s
            return list(reversed(st))
        sa, sb, sc = strides(a.shape, m * k), strides(b.shape, k * n), strides(out_shape, m * n)
        for i, s in enumerate(batch):
            d.batch_shape[i] = s
            d.a_batch_stride[i] = sa[i]
            d.b_batch_stride[i] = sb[i]
            d.c_batch_stride[i] = sc[i]
        nbytes = self.lib.tl_gemm_workspace_size(ctypes.byref(d))
        ws = self.ws(nbytes) if nbytes else None
        if ws is not None:
            d.workspace = ws.data_ptr()
            d.workspace_bytes = nbytes
        self.call("tl_gemm", ctypes.byref(d), self.stream)
        return (self.host(tc), self.host(tg)) if gelu else self.host(tc)
