"""Data parallelism over NCCL on two GPUs: two ranks, each on its own GPU
with half of the batch and `world = 2`, exchange their gradients through
the runtime's all-reduce (one NCCL group of per-tensor sums, or with
TL_FLAT_ALLREDUCE=1 every gradient packed into one flat buffer and one
NCCL sum) before the fused clip + AdamW; their parameters after two steps
follow one process on the whole batch.  Skipped with fewer than two GPUs.

Tolerance: FP32 products; only the summation order of the gradients
differs (per-rank sums, then the cross-rank sum), so the two steps' parameter
updates agree within 1e-4 of the update's norm, and the ranks' parameters
are bit-identical to each other (both apply the same summed gradient)."""
import ctypes
import multiprocessing as mp

import numpy as np
import pytest

from templit_b200 import capi

pytestmark = pytest.mark.gpu

B, T, STEPS = 8, 64, 2


def _config(batch, world):
    return capi.TlgConfig(family=4, batch=batch, seq=T, seed=3, init_std=0.02, lr=3e-4,
                          beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0,
                          world=world, fusion=1, graphs=1, gemm_precision=capi.TL_GEMM_FP32,
                          deferred_wait=1)


def _batches():
    from tests.test_gpt_gpu import zipf
    rng = np.random.default_rng(5)
    return [zipf(rng, B, T) for _ in range(STEPS)]


def _rank(rank, uid, p0, out, flat):
    import os
    os.environ["TL_FLAT_ALLREDUCE"] = "1" if flat else "0"
    import torch
    torch.cuda.set_device(rank)
    from tests.test_gpt_gpu import CudaGPT
    g = CudaGPT(_config(B // 2, 2))
    lib = g.lib
    capi.check(lib.tlg_set_communicator(g.h, (ctypes.c_uint8 * 128).from_buffer_copy(uid), 2,
                                        rank), lib, "communicator")
    g.set_params(p0)
    half = slice(rank * B // 2, (rank + 1) * B // 2)
    for x, y in _batches():
        g.set_batch(x[half], y[half])
        g.train_step()
    out.put((rank, g.params()))
    g.close()


@pytest.mark.parametrize("flat", [0, 1])
def test_two_ranks_follow_one_process(flat):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from tests.test_gpt_gpu import CudaGPT
    one = CudaGPT(_config(B, 1))
    p0 = one.params()
    for x, y in _batches():
        one.set_batch(x, y)
        one.train_step()
    want = one.params()
    one.close()

    uid = (ctypes.c_uint8 * 128)()
    capi.check(capi.gpt_lib().tlg_nccl_unique_id(uid), capi.gpt_lib(), "nccl id")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, bytes(uid), p0, out, flat)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(out.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    np.testing.assert_array_equal(got[0], got[1])
    d_one, d_dp = want.astype(np.float64) - p0, got[0].astype(np.float64) - p0
    assert np.linalg.norm(d_dp - d_one) <= 1e-4 * np.linalg.norm(d_one)
