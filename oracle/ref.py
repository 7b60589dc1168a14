"""ctypes access to the reference's own CPU runtime, compiled from the
JTPuffer/TempLit sources by oracle/ref_cpu/Makefile into
oracle/_ref/libref_cpu.so.  TEST INFRASTRUCTURE ONLY (oracle pinning and the
"reference" CPU baseline); the product never loads it."""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_double, c_float, c_int, c_uint32

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref", "libref_cpu.so")
OPS = {"mult": 0, "add": 1, "sub": 2, "hadamard": 3, "divide": 4, "softmax": 5,
       "sum_to_shape": 6, "transpose": 7, "sigmoid": 8, "sqrt": 9}
FP = POINTER(c_float)

_lib = None


def available() -> bool:
    return os.path.exists(LIB_PATH)


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(LIB_PATH)
        _lib.ref_last_error.restype = c_char_p
        _lib.ref_op.restype = c_int
        _lib.ref_op.argtypes = [c_int, FP, c_uint32, c_uint32, FP, c_uint32, c_uint32, FP,
                                c_uint32, c_uint32]
        _lib.ref_mlp_train.restype = c_int
        _lib.ref_mlp_train.argtypes = [FP, c_uint32, c_uint32, c_uint32, c_uint32, FP, FP, FP, FP,
                                       FP, c_float, c_float, c_int, FP, POINTER(c_double)]
    return _lib


def _fp(a):
    return a.ctypes.data_as(FP)


def op(name, a, b=None, out_shape=None):
    """Runs one rank-2 op of the reference cpu:: runtime on float32 arrays."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b if b is not None else np.zeros((1, 1)), np.float32)
    if out_shape is None:
        if name == "mult":
            out_shape = (a.shape[0], b.shape[1])
        elif name == "transpose":
            out_shape = (a.shape[1], a.shape[0])
        elif name in ("add", "sub", "hadamard", "divide"):
            out_shape = (max(a.shape[0], b.shape[0]), max(a.shape[1], b.shape[1]))
        else:
            out_shape = a.shape
    out = np.zeros(out_shape, np.float32)
    rc = lib().ref_op(OPS[name], _fp(a), a.shape[0], a.shape[1], _fp(b), b.shape[0], b.shape[1],
                      _fp(out), out.shape[0], out.shape[1])
    if rc:
        raise RuntimeError(lib().ref_last_error().decode())
    return out


def mlp_train(X, W1, b1, W2, b2, Y, root, lr, steps):
    """Configuration-1 MLP on the reference compiled path; returns updated
    (W1, b1, W2, b2), per-step summed losses and wall seconds."""
    X = np.ascontiguousarray(X, np.float32)
    Y = np.ascontiguousarray(Y, np.float32)
    W1, b1, W2, b2 = (np.array(v, np.float32, copy=True) for v in (W1, b1, W2, b2))
    losses = np.zeros(steps, np.float32)
    secs = c_double(0)
    rc = lib().ref_mlp_train(_fp(X), X.shape[0], X.shape[1], W1.shape[1], W2.shape[1], _fp(W1),
                             _fp(b1), _fp(W2), _fp(b2), _fp(Y), root, lr, steps, _fp(losses),
                             ctypes.byref(secs))
    if rc:
        raise RuntimeError(lib().ref_last_error().decode())
    return (W1, b1, W2, b2), losses, secs.value
