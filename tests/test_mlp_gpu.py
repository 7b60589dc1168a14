"""Configuration 1: the MLP training step
compiled by the reference's passes::compile, run 20 SGD steps on
cuda::Runtime, against the same 20 steps on the reference's own CPU runtime
(tests/golden/mlp_ref_fixture.npz, recorded from src/CPU/cpu.cpp compiled
from the reference sources by tests/golden/make_cpu_ref_fixtures.py).

Target (BASELINE): <= 1e-5 relative on the weights after 20 steps with
exact-fp32 GEMMs; TF32 tensor-core GEMMs within 1e-3."""
import ctypes
import os

import numpy as np
import pytest

from templit_b200 import capi
from tests.helpers import GOLDEN

pytestmark = pytest.mark.gpu


def run_cuda(fx, precision, steps=20):
    lib = capi.gpt_lib()
    W1, b1, W2, b2 = (np.array(fx[k], np.float32, copy=True) for k in ("W1", "b1", "W2", "b2"))
    X, Y = np.ascontiguousarray(fx["X"]), np.ascontiguousarray(fx["Y"])
    losses = np.zeros(steps, np.float32)
    secs = ctypes.c_double()
    fp = ctypes.POINTER(ctypes.c_float)
    rc = lib.tlg_mlp_train(X.ctypes.data_as(fp), X.shape[0], X.shape[1], W1.shape[1], W2.shape[1],
                           W1.ctypes.data_as(fp), b1.ctypes.data_as(fp), W2.ctypes.data_as(fp),
                           b2.ctypes.data_as(fp), Y.ctypes.data_as(fp), 1.0 / 640.0, 0.01, steps,
                           precision, losses.ctypes.data_as(fp), ctypes.byref(secs))
    assert rc == 0, lib.tlg_mlp_last_error()
    return (W1, b1, W2, b2), losses


@pytest.fixture(scope="module")
def fx():
    return np.load(os.path.join(GOLDEN, "mlp_ref_fixture.npz"))


def test_mlp_fp32_matches_reference_cpu_runtime(fx):
    (W1, b1, W2, b2), losses = run_cuda(fx, capi.TL_GEMM_FP32)
    for got, name in ((W1, "W1"), (b1, "b1"), (W2, "W2"), (b2, "b2")):
        want = fx[name + "_out"]
        assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max(), name
    np.testing.assert_allclose(losses, fx["losses"], rtol=1e-5)
    assert losses[-1] < losses[0]


def test_mlp_tf32_within_tf32_tolerance(fx):
    (W1, b1, W2, b2), losses = run_cuda(fx, capi.TL_GEMM_TF32)
    for got, name in ((W1, "W1"), (b1, "b1"), (W2, "W2"), (b2, "b2")):
        want = fx[name + "_out"]
        assert np.abs(got - want).max() <= 1e-3 * np.abs(want).max(), name
    np.testing.assert_allclose(losses, fx["losses"], rtol=1e-3)
