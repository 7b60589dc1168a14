"""Configuration 5's model: the 12-block, d_model 768, 12-head, FFN 3072
GPT (the reference's decoder blocks, embeddings and projection in
templit_b200/gpt/deep_gpt.h) on cuda::Runtime, against the same model on
the host oracle (oracle/cpu_gpt/gpt_cpu_deep.cpp: the reference executor
on the CPU restatement of the runtime ops), at batch 1 and T = 256 (the
oracle's step takes seconds there; the bench runs T = 1024).

Above T = 192 the attention runs on the flash kernels by default (TF32
products, P never stored); flash_attention = -1 keeps the executor's
composite (products on the GEMM kernels).  FP32 products always take the
composite.

Tolerances (relative): per-token forward losses and the first step's mean
loss within 1e-5 with FP32 and 3xTF32 products and 1e-3 with TF32 (the
north star's GEMM-path bound); per-token losses after one clipped AdamW
step within 1e-5 (FP32), 3e-5 (3xTF32) and 1e-2 (TF32: measured 4.4e-3,
the largest of 256 tokens; AdamW's first step moves each of the 89 M
parameters by about lr * sign(g), so gradients within TF32 rounding of zero
move differently, more of them than in the 8.7 M-parameter configuration
4).  Micro-batching:
two passes of one sequence then one step equal one pass of both sequences
within 1e-5 (losses) and 1e-4 in update norm (FP32; only the summation
order of the gradients differs)."""
import numpy as np
import pytest

from templit_b200 import capi
from tests.test_gpt_gpu import CudaGPT, oracle, zipf

pytestmark = pytest.mark.gpu

T = 256


def config(batch, precision=capi.TL_GEMM_TF32, micro=1, seed=5, flash=0):
    return capi.TlgConfig(family=12, batch=batch, seq=T, seed=seed, init_std=0.02, lr=3e-4,
                          beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0, world=1,
                          fusion=1, graphs=1, gemm_precision=precision, deferred_wait=1,
                          micro_batches=micro, flash_attention=flash)


@pytest.fixture(scope="module")
def deep_oracle():
    cg = oracle()
    rng = np.random.default_rng(31)
    x, y = zipf(rng, 1, T)
    cpu = cg.OracleGPT(config(1, precision=capi.TL_GEMM_FP32))
    out = {"x": x, "y": y, "p0": cpu.params()}
    cpu.set_batch(x, y)
    out["f0"] = cpu.forward()
    out["step"] = cpu.train_step()
    out["f1"] = cpu.forward()
    cpu.close()
    return out


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.abs(b)))


@pytest.mark.parametrize("precision,flash,rtol,rtol_after", [
    (capi.TL_GEMM_FP32, 0, 1e-5, 1e-5),
    (capi.TL_GEMM_3XTF32, -1, 1e-5, 3e-5),
    (capi.TL_GEMM_TF32, -1, 1e-3, 1e-2),
    (capi.TL_GEMM_TF32, 0, 1e-3, 1e-2)])
def test_config5_model_matches_oracle(deep_oracle, precision, flash, rtol, rtol_after, tmp_path):
    o = deep_oracle
    gpu = CudaGPT(config(1, precision=precision, flash=flash))
    # embeddings 2048 x 768 + 1024 x 768; per block 4 (768^2 + 768) attention
    # and 2 x 768 x 3072 + 3072 + 768 feed-forward; projection 768 x 2048 + 2048
    assert o["p0"].size == gpu.params().size == 88_951_808
    gpu.set_params(o["p0"])
    gpu.set_batch(o["x"], o["y"])
    f0 = gpu.forward()
    step = gpu.train_step()
    f1 = gpu.forward()
    if precision == capi.TL_GEMM_TF32:
        # which attention path ran: the flash rewrite skips S, which needs
        # the runtime's window liveness (established over the first steps)
        for _ in range(3):
            gpu.train_step()
        ops = gpu.profile_ops(tmp_path)
        assert any(o.startswith("flash_fwd") for o in ops) == (flash == 0), ops
    gpu.close()
    r0, rs, r1 = rel(f0, o["f0"]), rel([step], [o["step"]]), rel(f1, o["f1"])
    print(f"precision {precision}, flash {flash}: per-token losses {r0:.2e}, step loss {rs:.2e}, "
          f"after the step {r1:.2e}")
    assert r0 <= rtol and rs <= rtol and r1 <= rtol_after
    assert abs(f0.mean() - np.log(2048)) < 0.5  # N(0, 0.02) weights: near-uniform logits


def test_config5_micro_batches_accumulate():
    rng = np.random.default_rng(8)
    x, y = zipf(rng, 2, T)
    one = CudaGPT(config(2, precision=capi.TL_GEMM_FP32))
    two = CudaGPT(config(1, precision=capi.TL_GEMM_FP32, micro=2))
    p0 = one.params()
    two.set_params(p0)
    one.set_batch(x, y)
    two.set_batch(x, y)
    la, lb = one.train_step(), two.train_step()
    pa, pb = one.params(), two.params()
    one.close()
    two.close()
    assert abs(la - lb) <= 1e-5 * abs(la)
    da, db = pa.astype(np.float64) - p0, pb.astype(np.float64) - p0
    assert np.linalg.norm(da - db) <= 1e-4 * np.linalg.norm(da)
