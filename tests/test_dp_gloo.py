"""Data parallelism on the CPU (gloo, world size 2), the multi-GPU path's
host logic: every rank starts from the same initialisation, scales its
root gradient by 1 / (world x its tokens), and sums every gradient across
ranks before the clipped AdamW step - the CUDA runtime's one all-reduce
ahead of the optimiser window.  Two ranks on half batches must then follow
a single process on the whole batch.  The ranks run the host oracle of the
GPT step (oracle/cpu_gpt); no GPU is involved."""
import os
import socket

import numpy as np
import pytest

from templit_b200 import capi

B, T, STEPS = 2, 32, 3


def _config(batch, world):
    return capi.TlgConfig(family=4, batch=batch, seq=T, seed=17, init_std=0.02, lr=3e-4,
                          beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0,
                          world=world, fusion=0, graphs=0, gemm_precision=1, deferred_wait=0)


def _batches():
    rng = np.random.default_rng(4)
    return [(rng.integers(0, 2048, (B, T)), rng.integers(0, 2048, (B, T))) for _ in range(STEPS)]


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    from oracle import cpu_gpt
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    g = cpu_gpt.OracleGPT(_config(B // world, world))

    def allreduce(arr):
        t = torch.from_numpy(arr)
        dist.all_reduce(t)

    g.set_allreduce(allreduce)
    losses = []
    for x, y in _batches():
        g.set_batch(x[rank::world], y[rank::world])
        losses.append(g.train_step())
    out[rank] = (g.params(), losses)
    g.close()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_available():
    try:
        from oracle import cpu_gpt
        cpu_gpt.lib()
        return True
    except Exception:
        return False


@pytest.mark.skipif(not _oracle_available(), reason="host oracle library not built")
def test_two_gloo_ranks_follow_one_process():
    import torch.multiprocessing as mp
    from oracle import cpu_gpt
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        out = manager.dict()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=600)
            assert p.exitcode == 0
        (p0, l0), (p1, l1) = out[0], out[1]
    assert np.array_equal(p0, p1)  # every rank applies the same update
    single = cpu_gpt.OracleGPT(_config(B, 1))
    losses = []
    for x, y in _batches():
        single.set_batch(x, y)
        losses.append(single.train_step())
    ps = single.params()
    single.close()
    # the per-rank losses average to the whole batch's loss
    np.testing.assert_allclose((np.array(l0) + np.array(l1)) / 2, losses, rtol=1e-5)
    np.testing.assert_allclose(p0, ps, rtol=0, atol=1e-6)
