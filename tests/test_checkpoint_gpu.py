"""Checkpoint I/O of device tensors: the
parameters and the AdamW state of the GPT step saved from the CUDA runtime
in the reference's archive format (src/model_utils/archive.cpp:33-73, via
Compiled::save / save_optimisers) and restored.

  * the restored parameters are bit-identical, and training resumed from
    the checkpoint follows the uninterrupted run within the GPT-step
    tolerances of tests/test_gpt_gpu.py (losses 1e-5 relative, parameter
    updates 1% in norm): a fresh runtime runs its first windows before the
    window-local fusions apply, so its reduction orders differ at first;
  * a CUDA checkpoint is read by the reference's own Archive::restore (the
    host oracle) and an oracle checkpoint by tlg_load: parameters bit-exact,
    the next step within the FP32 tolerance of tests/test_gpt_gpu.py."""
import numpy as np
import pytest

from templit_b200 import capi
from tests.test_gpt_gpu import CudaGPT, config, oracle, zipf

pytestmark = pytest.mark.gpu

B, T = 4, 64


def batches(n, seed=3):
    rng = np.random.default_rng(seed)
    return [zipf(rng, B, T) for _ in range(n)]


def test_resume_follows_the_uninterrupted_run(tmp_path):
    data = batches(5)
    path = tmp_path / "step3.ckpt"
    a = CudaGPT(config(B, T, seed=21))
    b = CudaGPT(config(B, T, seed=99))  # different initial weights: all come from the file
    try:
        for x, y in data[:3]:
            a.set_batch(x, y)
            a.train_step()
        a.save(path)
        b.load(path)
        p0 = a.params()
        np.testing.assert_array_equal(b.params(), p0)
        for x, y in data[3:]:
            a.set_batch(x, y)
            b.set_batch(x, y)
            la, lb = a.train_step(), b.train_step()
            assert abs(la - lb) <= 1e-5 * abs(la), (la, lb)
        da, db = a.params() - p0, b.params() - p0
        assert np.linalg.norm(da - db) <= 1e-2 * np.linalg.norm(da)
    finally:
        a.close()
        b.close()


def test_checkpoint_is_the_reference_format(tmp_path):
    cg = oracle()
    data = batches(3, seed=4)
    cfg = config(B, T, precision=capi.TL_GEMM_FP32, seed=31, deferred=0)
    a = CudaGPT(cfg)
    o = cg.OracleGPT(cfg)
    c = CudaGPT(config(B, T, precision=capi.TL_GEMM_FP32, seed=77, deferred=0))
    try:
        for x, y in data[:2]:
            a.set_batch(x, y)
            a.train_step()
        a.save(tmp_path / "cuda.ckpt")
        o.load(tmp_path / "cuda.ckpt")  # the reference's Archive::restore
        np.testing.assert_array_equal(o.params(), a.params())
        x, y = data[2]
        a.set_batch(x, y)
        o.set_batch(x, y)
        la, lo = a.train_step(), o.train_step()
        assert abs(la - lo) <= 1e-5 * abs(lo), (la, lo)
        o.save(tmp_path / "oracle.ckpt")  # the reference's Archive::commit
        c.load(tmp_path / "oracle.ckpt")
        np.testing.assert_array_equal(c.params(), o.params())
    finally:
        a.close()
        o.close()
        c.close()


def test_missing_checkpoint_and_uninitialised_state(tmp_path):
    a = CudaGPT(config(B, T, seed=5))
    try:
        with pytest.raises(capi.TlError, match="cannot open"):
            a.load(tmp_path / "absent.ckpt")
        # no step yet: the reference refuses to save uninitialised AdamW state
        with pytest.raises(capi.TlError, match="uninitialised AdamW"):
            a.save(tmp_path / "early.ckpt", optimiser=True)
        a.save(tmp_path / "params.ckpt", optimiser=False)
    finally:
        a.close()
