"""Writes tests/golden/gpt_curve_b4_t192.npz: the host oracle's 100-step
training curve of the reference GPT (vocab 2048, T 192, d 384, 4 blocks, 6
heads) at batch 4, the configuration-4 model at a quarter-size batch.

The oracle (oracle/cpu_gpt: the reference's nn::GPT and passes::Compiled on
a double-accumulating CPU restatement of every runtime op) needs minutes for
these 100 steps, so its curve is recorded once here and the GPU test
(tests/test_gpt_gpu.py) compares the CUDA runtime's curve with it.  The
fixture holds the ten Zipf(1.1) batches the curve cycles through, the
oracle's per-step losses, and the SHA-256 of the oracle's initial
parameters: the GPU test re-creates them with the oracle (the same seed),
checks the hash and loads them into the CUDA model, so both curves start
from the same bits (the two libraries draw the seed's normal variates with
different floating-point contraction, so their own draws differ in the last
bits).

Run:  make -C oracle/cpu_gpt && python tests/golden/make_gpt_curve_fixture.py
"""
import hashlib
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import cpu_gpt  # noqa: E402
from templit_b200 import capi  # noqa: E402

B, T, STEPS, SEED = 4, 192, 100, 11
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "gpt_curve_b4_t192.npz")


def zipf(rng, b, t):
    """p(k) proportional to (k + 1)^-1.1 over [0, 2048), windows of t + 1."""
    p = 1.0 / np.arange(1, 2049) ** 1.1
    s = rng.choice(2048, b * (t + 1), p=p / p.sum()).reshape(b, t + 1)
    return s[:, :t].astype(np.uint32), s[:, 1:].astype(np.uint32)


def config():
    return capi.TlgConfig(family=4, batch=B, seq=T, seed=SEED, init_std=0.02, lr=3e-4,
                          beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0, world=1,
                          fusion=1, graphs=1, gemm_precision=capi.TL_GEMM_FP32, deferred_wait=1)


def main():
    rng = np.random.default_rng(9)
    batches = [zipf(rng, B, T) for _ in range(10)]
    cpu = cpu_gpt.OracleGPT(config())
    p0 = cpu.params()
    losses = []
    t0 = time.time()
    for s in range(STEPS):
        x, y = batches[s % len(batches)]
        cpu.set_batch(x, y)
        losses.append(cpu.train_step())
        if s % 10 == 9:
            print(f"step {s + 1}: loss {losses[-1]:.6f} ({time.time() - t0:.0f} s)", flush=True)
    cpu.close()
    np.savez_compressed(
        OUT, x=np.stack([b[0] for b in batches]), y=np.stack([b[1] for b in batches]),
        losses=np.array(losses, np.float32),
        params0_sha256=np.frombuffer(hashlib.sha256(p0.tobytes()).digest(), np.uint8),
        batch=B, seq=T, seed=SEED)
    print("wrote", OUT)


if __name__ == "__main__":
    main()
