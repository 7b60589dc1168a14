"""The reference's archive round trip on the host oracle (CPU): a GPT step's
parameters and AdamW state committed by the reference's Archive and restored
into a fresh model give the same parameters and the same next step.  Pins
the checker that tests/test_checkpoint_gpu.py reads CUDA checkpoints with."""
import numpy as np
import pytest

from oracle import cpu_gpt
from templit_b200 import capi

pytestmark = pytest.mark.skipif(not cpu_gpt.available(), reason="oracle GPT library not built")


def cfg(seed):
    return capi.TlgConfig(family=4, batch=2, seq=16, seed=seed, init_std=0.02, lr=3e-4,
                          beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0, world=1,
                          fusion=1, graphs=1, gemm_precision=capi.TL_GEMM_FP32, deferred_wait=0)


def test_oracle_archive_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    data = [(rng.integers(0, 2048, (2, 16)), rng.integers(0, 2048, (2, 16))) for _ in range(3)]
    a, b = cpu_gpt.OracleGPT(cfg(1)), cpu_gpt.OracleGPT(cfg(2))
    try:
        for x, y in data[:2]:
            a.set_batch(x, y)
            a.train_step()
        a.save(tmp_path / "a.ckpt")
        b.load(tmp_path / "a.ckpt")
        np.testing.assert_array_equal(b.params(), a.params())
        x, y = data[2]
        a.set_batch(x, y)
        b.set_batch(x, y)
        assert a.train_step() == b.train_step()
        np.testing.assert_array_equal(b.params(), a.params())
    finally:
        a.close()
        b.close()
