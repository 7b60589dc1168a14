"""Writes tests/golden/cpu_ref_fixtures.npz: outputs of the reference's own
CPU runtime (JTPuffer/TempLit src/CPU/cpu.cpp, compiled from the reference
sources into oracle/_ref/libref_cpu.so by oracle/ref_cpu/Makefile) on seeded
inputs, and the configuration-1 MLP trained 20 steps on the reference's
compiled path.  The fixtures travel with the repository, so the GPU box
(which has no reference checkout) can compare the CUDA kernels against the
reference's own numbers.

Run:  make -C oracle/ref_cpu && python tests/golden/make_cpu_ref_fixtures.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import ref  # noqa: E402


def mlp_inputs(seed=0, batch=64, inp=128, hidden=256, out=10):
    """Configuration 1 of BASELINE.json: X ~ U(-1,1), Xavier-uniform weights,
    zero biases, targets ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    X = rng.uniform(-1, 1, (batch, inp)).astype(np.float32)
    l1 = np.sqrt(6.0 / (inp + hidden))
    l2 = np.sqrt(6.0 / (hidden + out))
    W1 = rng.uniform(-l1, l1, (inp, hidden)).astype(np.float32)
    W2 = rng.uniform(-l2, l2, (hidden, out)).astype(np.float32)
    b1 = np.zeros((1, hidden), np.float32)
    b2 = np.zeros((1, out), np.float32)
    Y = rng.standard_normal((batch, out)).astype(np.float32)
    return X, W1, b1, W2, b2, Y


def main():
    rng = np.random.default_rng(1234)
    fx = {}

    def rec(name, op, a, b=None, out_shape=None):
        out = ref.op(op, a, b, out_shape)
        fx[name + "__op"] = np.array(op)
        fx[name + "__a"] = np.asarray(a, np.float32)
        if b is not None:
            fx[name + "__b"] = np.asarray(b, np.float32)
        fx[name + "__out"] = out

    for m, k, n in ((64, 64, 64), (96, 40, 72), (192, 192, 192), (33, 17, 65)):
        rec(f"mult_{m}x{k}x{n}", "mult", rng.standard_normal((m, k)), rng.standard_normal((k, n)))
    x = rng.standard_normal((48, 40))
    rec("add_same", "add", x, rng.standard_normal((48, 40)))
    rec("add_row", "add", x, rng.standard_normal((1, 40)))
    rec("sub_col", "sub", x, rng.standard_normal((48, 1)))
    rec("hadamard_scalar", "hadamard", x, rng.standard_normal((1, 1)))
    rec("divide_row", "divide", x, rng.uniform(0.5, 2.0, (1, 40)))
    rec("softmax_rows", "softmax", rng.standard_normal((64, 192)) * 3)
    rec("sum_rows", "sum_to_shape", x, out_shape=(48, 1))
    rec("sum_cols", "sum_to_shape", x, out_shape=(1, 40))
    rec("sum_all", "sum_to_shape", x, out_shape=(1, 1))
    rec("transpose_48x40", "transpose", x)
    rec("sigmoid", "sigmoid", x)
    rec("sqrt", "sqrt", np.abs(x))

    X, W1, b1, W2, b2, Y = mlp_inputs()
    (w1, c1, w2, c2), losses, _ = ref.mlp_train(X, W1, b1, W2, b2, Y, 1.0 / 640.0, 0.01, 20)
    mlp = dict(X=X, W1=W1, b1=b1, W2=W2, b2=b2, Y=Y, W1_out=w1, b1_out=c1, W2_out=w2,
               b2_out=c2, losses=losses)

    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "cpu_ref_fixtures.npz")
    np.savez_compressed(out, **fx)
    np.savez_compressed(os.path.join(os.path.dirname(out), "mlp_ref_fixture.npz"), **mlp)
    print("wrote", out, "and mlp_ref_fixture.npz")


if __name__ == "__main__":
    main()
