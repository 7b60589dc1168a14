"""ctypes access to the host oracle of the GPT training step
(oracle/_build/libgpt_cpu.so, built by oracle/cpu_gpt/Makefile): the
reference's nn::GPT and passes::Compiled on a CPU restatement of every
runtime op.  TEST INFRASTRUCTURE ONLY: GPT-level parity tests and the
CPU baseline of bench.py."""
from __future__ import annotations

import ctypes
import os
import time
from ctypes import POINTER, c_char_p, c_float, c_int, c_uint32, c_uint64, c_void_p

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build", "libgpt_cpu.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        from templit_b200.capi import TlgConfig
        _lib = ctypes.CDLL(LIB_PATH)
        U32P = POINTER(c_uint32)
        sig = {
            "tlo_last_error": (c_char_p, []),
            "tlo_create": (c_int, [POINTER(TlgConfig), POINTER(c_void_p)]),
            "tlo_destroy": (c_int, [c_void_p]),
            "tlo_set_batch": (c_int, [c_void_p, U32P, U32P]),
            "tlo_train_step": (c_int, [c_void_p, POINTER(c_float)]),
            "tlo_forward": (c_int, [c_void_p, POINTER(c_float)]),
            "tlo_param_count": (c_int, [c_void_p, POINTER(c_uint64), POINTER(c_uint32)]),
            "tlo_get_params": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
            "tlo_set_params": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
            "tlo_set_allreduce": (c_int, [c_void_p, ALLREDUCE_FN, c_void_p]),
            "tlo_loader_batches": (c_int, [c_char_p, ctypes.c_double, c_int, c_uint32, c_uint32,
                                           c_uint32, c_uint32, U32P, U32P]),
            "tlo_save": (c_int, [c_void_p, c_char_p, c_int]),
            "tlo_load": (c_int, [c_void_p, c_char_p, c_int]),
            "tlo_infer_create": (c_int, [POINTER(TlgConfig), POINTER(c_void_p)]),
            "tlo_infer_destroy": (c_int, [c_void_p]),
            "tlo_infer_set_params": (c_int, [c_void_p, POINTER(c_float), c_uint64]),
            "tlo_infer_logits": (c_int, [c_void_p, U32P, POINTER(c_float)]),
            "tlo_infer_generate": (c_int, [c_void_p, U32P, c_uint32, c_uint32, c_uint32, c_uint32,
                                           c_float, c_uint32, U32P, c_uint32, U32P]),
        }
        for name, (res, args) in sig.items():
            f = getattr(_lib, name)
            f.restype, f.argtypes = res, args
    return _lib


def _check(rc):
    if rc:
        raise RuntimeError(lib().tlo_last_error().decode())


# void (*)(float *data, uint64_t count, void *ctx): sums a gradient across ranks
ALLREDUCE_FN = ctypes.CFUNCTYPE(None, POINTER(c_float), c_uint64, c_void_p)


class OracleGPT:
    """The reference GPT (family 4) on the host oracle runtime."""

    def __init__(self, cfg):
        self.h = c_void_p()
        _check(lib().tlo_create(ctypes.byref(cfg), ctypes.byref(self.h)))
        self.n = cfg.batch * cfg.seq

    def set_batch(self, x, y):
        x = np.ascontiguousarray(x, np.uint32).ravel()
        y = np.ascontiguousarray(y, np.uint32).ravel()
        u = POINTER(c_uint32)
        _check(lib().tlo_set_batch(self.h, x.ctypes.data_as(u), y.ctypes.data_as(u)))

    def train_step(self):
        v = c_float()
        _check(lib().tlo_train_step(self.h, ctypes.byref(v)))
        return v.value

    def forward(self):
        out = np.zeros(self.n, np.float32)
        _check(lib().tlo_forward(self.h, out.ctypes.data_as(POINTER(c_float))))
        return out

    def params(self):
        n, t = c_uint64(), c_uint32()
        _check(lib().tlo_param_count(self.h, ctypes.byref(n), ctypes.byref(t)))
        out = np.zeros(n.value, np.float32)
        _check(lib().tlo_get_params(self.h, out.ctypes.data_as(POINTER(c_float)), n.value))
        return out

    def set_allreduce(self, fn):
        """fn(array) sums a float32 gradient (numpy view) across ranks in
        place; called once per gradient before the optimiser reads it."""
        def cb(data, count, ctx):
            fn(np.ctypeslib.as_array(data, shape=(count,)))
        self._cb = ALLREDUCE_FN(cb)  # kept alive with the handle
        _check(lib().tlo_set_allreduce(self.h, self._cb, None))

    def set_params(self, p):
        p = np.ascontiguousarray(p, np.float32)
        _check(lib().tlo_set_params(self.h, p.ctypes.data_as(POINTER(c_float)), p.size))

    def save(self, path, optimiser=True):
        """Checkpoint through the reference's Archive (commit)."""
        _check(lib().tlo_save(self.h, str(path).encode(), int(optimiser)))

    def load(self, path, optimiser=True):
        _check(lib().tlo_load(self.h, str(path).encode(), int(optimiser)))

    def close(self):
        if self.h:
            lib().tlo_destroy(self.h)
            self.h = c_void_p()


def train_tokens_per_s(batch, seq, steps, threads, warmup=0):
    """Times `steps` GPT d384 training steps on the host oracle (all
    `threads` OpenMP threads) after `warmup` untimed ones; returns
    (tokens/s, seconds)."""
    from templit_b200.capi import TlgConfig
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    cfg = TlgConfig(family=4, batch=batch, seq=seq, seed=1234, init_std=0.02, lr=3e-4,
                    beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0, world=1,
                    fusion=0, graphs=0, gemm_precision=1)
    rng = np.random.default_rng(7)
    g = OracleGPT(cfg)
    try:
        x = rng.integers(0, 2048, (batch, seq))
        y = rng.integers(0, 2048, (batch, seq))
        g.set_batch(x, y)
        for _ in range(warmup):
            g.train_step()
        t0 = time.perf_counter()
        for _ in range(steps):
            g.train_step()
        secs = time.perf_counter() - t0
    finally:
        g.close()
    return batch * seq * steps / secs, secs


class OracleGPTInference:
    """Forward-only inference of the reference GPT (family 4, batch 1) on the
    host oracle runtime: the model of src/generate.cpp driven by the
    reference's inference::autoregression."""

    def __init__(self, cfg):
        self.h = c_void_p()
        _check(lib().tlo_infer_create(ctypes.byref(cfg), ctypes.byref(self.h)))
        self.seq = cfg.seq

    def set_params(self, p):
        p = np.ascontiguousarray(p, np.float32)
        _check(lib().tlo_infer_set_params(self.h, p.ctypes.data_as(POINTER(c_float)), p.size))

    def logits(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32).ravel()
        out = np.zeros((self.seq, 2048), np.float32)
        _check(lib().tlo_infer_logits(self.h, t.ctypes.data_as(POINTER(c_uint32)),
                                      out.ctypes.data_as(POINTER(c_float))))
        return out

    def generate(self, prompt, eos, seed, top_k, temperature, min_length, max_out=4096):
        pr = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max_out, np.uint32)
        n = c_uint32()
        u = POINTER(c_uint32)
        _check(lib().tlo_infer_generate(self.h, pr.ctypes.data_as(u), pr.size, eos, seed, top_k,
                                        temperature, min_length, out.ctypes.data_as(u), max_out,
                                        ctypes.byref(n)))
        return out[:min(n.value, max_out)].tolist()

    def close(self):
        if self.h:
            lib().tlo_infer_destroy(self.h)
            self.h = c_void_p()


def loader_batches(path, training_fraction, validation, batch, seq, seed, n):
    """n batches from the reference's own Dataset::load_tokens + Loader."""
    x = np.zeros((n, batch, seq), np.uint32)
    y = np.zeros((n, batch, seq), np.uint32)
    u = POINTER(c_uint32)
    _check(lib().tlo_loader_batches(str(path).encode(), training_fraction, int(validation), batch,
                                    seq, seed, n, x.ctypes.data_as(u), y.ctypes.data_as(u)))
    return x, y
