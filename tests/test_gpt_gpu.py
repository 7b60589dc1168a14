"""The GPT training step (the reference's nn::GPT + passes::Compiled on
cuda::Runtime, include/templit_gpt.h) against the host oracle of the same
step (oracle/cpu_gpt: the reference executor on a double-accumulating CPU
restatement of the runtime ops), plus determinism and the program-replay
machinery.

Tolerances (relative, stated per test below):
  * Configuration 4 itself (batch 64, T 192): the per-token forward losses
    and the two clipped AdamW steps' mean losses within 1e-5 for FP32 and
    3xTF32 products and 1e-3 for TF32; the per-token losses after the two
    steps within 1e-5 (FP32), 3e-5 (3xTF32) and 3e-3 (TF32).  AdamW's first
    steps move each parameter by lr * g / (|g| + eps): about lr * sign(g),
    so an element whose gradient is within rounding of zero (or of eps) may
    move differently.  The parameter updates agree within 1e-4 in norm for
    FP32 (measured 1.3e-5; and within 1e-5 relative per element except at
    most 0.5 % of the elements, measured 0.14 %), 1e-3 for 3xTF32 (measured
    5.0e-4) and 0.1 for TF32 (measured 1.75e-2).
  * The 100-step loss curve at batch 4, T 192 (the oracle's curve is a
    committed fixture, tests/golden/make_gpt_curve_fixture.py): within
    1e-3 of the oracle at every step for FP32 and 3xTF32 products.  Plain
    TF32 products (10-bit significands) drift as the model fits the
    repeated batches: measured at 0.21 at one step (the trajectories take
    a loss spike at different steps), so the per-step bound is 0.3 and the
    final loss must agree within 2 %."""
import ctypes
import hashlib
import os

import numpy as np
import pytest

from templit_b200 import capi

pytestmark = pytest.mark.gpu


def config(batch, seq, precision=capi.TL_GEMM_TF32, fusion=1, graphs=1, seed=11, deferred=1,
           flash=0):
    return capi.TlgConfig(family=4, batch=batch, seq=seq, seed=seed, init_std=0.02, lr=3e-4,
                          beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0, world=1,
                          fusion=fusion, graphs=graphs, gemm_precision=precision,
                          deferred_wait=deferred, flash_attention=flash)


class CudaGPT:
    def __init__(self, cfg):
        self.lib = capi.gpt_lib()
        self.h = ctypes.c_void_p()
        capi.check(self.lib.tlg_create(ctypes.byref(cfg), ctypes.byref(self.h)), self.lib, "create")
        self.n = cfg.batch * cfg.seq

    def set_batch(self, x, y):
        x = np.ascontiguousarray(x, np.uint32).ravel()
        y = np.ascontiguousarray(y, np.uint32).ravel()
        u = ctypes.POINTER(ctypes.c_uint32)
        capi.check(self.lib.tlg_set_batch(self.h, x.ctypes.data_as(u), y.ctypes.data_as(u)),
                   self.lib, "batch")

    def train_step(self):
        v = ctypes.c_float()
        capi.check(self.lib.tlg_train_step(self.h, ctypes.byref(v)), self.lib, "step")
        return v.value

    def forward(self):
        out = np.zeros(self.n, np.float32)
        capi.check(self.lib.tlg_forward(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))),
                   self.lib, "forward")
        return out

    def params(self):
        n, t = ctypes.c_uint64(), ctypes.c_uint32()
        capi.check(self.lib.tlg_param_count(self.h, ctypes.byref(n), ctypes.byref(t)), self.lib, "n")
        out = np.zeros(n.value, np.float32)
        capi.check(self.lib.tlg_get_params(self.h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                           n.value), self.lib, "params")
        return out

    def set_params(self, p):
        p = np.ascontiguousarray(p, np.float32)
        capi.check(self.lib.tlg_set_params(self.h, p.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                           p.size), self.lib, "set_params")

    def stats(self):
        s = (ctypes.c_uint64 * 11)()
        capi.check(self.lib.tlg_stats(self.h, s), self.lib, "stats")
        return dict(zip(["windows", "recorded", "launched", "kernels", "replays", "captures",
                         "fused", "peak_bytes", "record_ns", "submit_ns", "plan_hits"], list(s)))

    def profile_ops(self, tmp_path):
        """Names of the ops of the next train step (per-op profile)."""
        import json
        path = str(tmp_path / "profile.json")
        capi.check(self.lib.tlg_profile(self.h, path.encode(), 1), self.lib, "profile")
        self.train_step()
        with open(path) as f:
            return [o["op"] for o in json.load(f)["ops"]]

    def save(self, path, optimiser=True):
        capi.check(self.lib.tlg_save(self.h, str(path).encode(), int(optimiser)), self.lib, "save")

    def load(self, path, optimiser=True):
        capi.check(self.lib.tlg_load(self.h, str(path).encode(), int(optimiser)), self.lib, "load")

    def close(self):
        capi.check(self.lib.tlg_destroy(self.h), self.lib, "destroy")


def zipf(rng, b, t):
    p = 1.0 / np.arange(1, 2049) ** 1.1
    s = rng.choice(2048, b * (t + 1), p=p / p.sum()).reshape(b, t + 1)
    return s[:, :t].astype(np.uint32), s[:, 1:].astype(np.uint32)


def oracle():
    from oracle import cpu_gpt
    if not cpu_gpt.available():
        pytest.fail("host GPT oracle not built (make -C oracle/cpu_gpt)")
    return cpu_gpt


def test_parameter_layout_and_init():
    g = CudaGPT(config(2, 16))
    p = g.params()
    assert p.size == 8_740_352  # nn::GPT<2048,192,384,6>: 8.74 M parameters
    assert abs(p.std() - 0.02) < 0.002  # N(0, 0.02) weights, zero biases
    g.close()


def test_forward_and_three_steps_match_host_oracle_fp32():
    cg = oracle()
    rng = np.random.default_rng(5)
    B, T = 2, 24
    x, y = zipf(rng, B, T)
    gpu = CudaGPT(config(B, T, precision=capi.TL_GEMM_FP32))
    cpu = cg.OracleGPT(config(B, T, precision=capi.TL_GEMM_FP32))
    p0 = gpu.params()
    cpu.set_params(p0)
    gpu.set_batch(x, y)
    cpu.set_batch(x, y)
    lg, lc = gpu.forward(), cpu.forward()
    np.testing.assert_allclose(lg, lc, rtol=1e-5, atol=1e-5)
    for _ in range(3):
        a, b = gpu.train_step(), cpu.train_step()
        assert abs(a - b) <= 1e-5 * abs(b)
    dg, dc = gpu.params() - p0, cpu.params() - p0
    assert np.linalg.norm(dg - dc) <= 1e-2 * np.linalg.norm(dc)
    gpu.close()
    cpu.close()


CURVE_FIXTURE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                             "gpt_curve_b4_t192.npz")


@pytest.mark.parametrize("precision,rtol,flash", [
    (capi.TL_GEMM_FP32, 1e-3, 0),    # exact fp32 products (CUDA cores)
    (capi.TL_GEMM_3XTF32, 1e-3, 0),  # split tf32 operands on the tensor cores
    (capi.TL_GEMM_TF32, 0.3, 0),     # plain TF32: the benchmark path's drift
    (capi.TL_GEMM_TF32, 0.3, 1)])    # ... with attention on the flash kernels
def test_loss_curve_100_steps_tracks_oracle(precision, rtol, flash):
    fx = np.load(CURVE_FIXTURE)
    B, T = int(fx["batch"]), int(fx["seq"])
    cfg = config(B, T, precision=precision, seed=int(fx["seed"]), flash=flash)
    # the oracle's initial weights (the ones the fixture's curve starts from)
    cpu = oracle().OracleGPT(config(B, T, precision=capi.TL_GEMM_FP32, seed=int(fx["seed"])))
    p0 = cpu.params()
    cpu.close()
    assert hashlib.sha256(p0.tobytes()).digest() == fx["params0_sha256"].tobytes()
    gpu = CudaGPT(cfg)
    gpu.set_params(p0)
    want = fx["losses"].astype(np.float64)
    got = []
    for s in range(want.size):
        i = s % fx["x"].shape[0]
        gpu.set_batch(fx["x"][i], fx["y"][i])
        got.append(gpu.train_step())
    gpu.close()
    got = np.array(got, np.float64)
    dev = np.abs(got - want) / np.abs(want)
    print(f"precision {precision}: max relative deviation {dev.max():.3e} "
          f"(step {int(dev.argmax())}), final loss {got[-1]:.5f} vs {want[-1]:.5f}")
    assert want[-1] < want[0] - 1.0  # the model learns on repeated batches
    assert dev.max() <= rtol
    assert abs(got[-1] - want[-1]) <= 2e-2 * want[-1]


@pytest.fixture(scope="module")
def config4_oracle():
    """The oracle at configuration 4: per-token losses, two clipped AdamW
    steps, per-token losses again, and the parameters after the steps."""
    cg = oracle()
    rng = np.random.default_rng(21)
    x, y = zipf(rng, 64, 192)
    cpu = cg.OracleGPT(config(64, 192, precision=capi.TL_GEMM_FP32))
    out = {"x": x, "y": y, "p0": cpu.params()}
    cpu.set_batch(x, y)
    out["f0"] = cpu.forward()
    out["steps"] = np.array([cpu.train_step() for _ in range(2)], np.float64)
    out["f2"] = cpu.forward()
    out["p2"] = cpu.params()
    cpu.close()
    return out


def param_sizes(g, tmp_path):
    """Element counts of the parameter tensors, in tlg_get_params order, from
    a checkpoint (the reference archive layout: u32 name length, name, u32
    blob length, blob; entries parameters/<i>/size hold the shapes)."""
    path = tmp_path / "sizes.bin"
    g.save(path, optimiser=False)
    raw = path.read_bytes()
    shapes, off = {}, 0
    while off < len(raw):
        n = int.from_bytes(raw[off:off + 4], "little")
        name = raw[off + 4:off + 4 + n].decode()
        off += 4 + n
        m = int.from_bytes(raw[off:off + 4], "little")
        blob = raw[off + 4:off + 4 + m]
        off += 4 + m
        parts = name.split("/")
        if parts[0] == "parameters" and parts[2] == "size":
            shapes[int(parts[1])] = np.frombuffer(blob, np.uint32)
    return [int(np.prod(shapes[i])) for i in range(len(shapes))]


@pytest.mark.parametrize("precision,rtol,rtol_after,flash", [
    (capi.TL_GEMM_FP32, 1e-5, 1e-5, 0),
    (capi.TL_GEMM_3XTF32, 1e-5, 3e-5, 0),
    (capi.TL_GEMM_TF32, 1e-3, 3e-3, 0),
    (capi.TL_GEMM_TF32, 1e-3, 3e-3, 1)])  # attention on the flash kernels (P never stored)
def test_config4_step_matches_oracle(config4_oracle, precision, rtol, rtol_after, flash,
                                     tmp_path):
    o = config4_oracle
    gpu = CudaGPT(config(64, 192, precision=precision, flash=flash))
    p0 = o["p0"]
    gpu.set_params(p0)  # the oracle's initial weights
    assert np.array_equal(gpu.params(), p0)
    gpu.set_batch(o["x"], o["y"])
    f0 = gpu.forward()
    steps = np.array([gpu.train_step() for _ in range(2)], np.float64)
    f2 = gpu.forward()
    p2 = gpu.params()
    sizes = param_sizes(gpu, tmp_path)
    gpu.close()
    assert sum(sizes) == p2.size == 8_740_352

    def rel(a, b):
        return float(np.max(np.abs(a.astype(np.float64) - b) / np.abs(b.astype(np.float64))))
    r0, rs, r2 = rel(f0, o["f0"]), rel(steps, o["steps"]), rel(f2, o["f2"])
    print(f"precision {precision}: per-token losses {r0:.2e}, step losses {rs:.2e}, "
          f"after two steps {r2:.2e}")
    assert r0 <= rtol and rs <= rtol and r2 <= rtol_after
    d_g, d_c = p2.astype(np.float64) - p0, o["p2"].astype(np.float64) - p0
    upd = np.linalg.norm(d_g - d_c) / np.linalg.norm(d_c)
    print(f"update difference in norm {upd:.3e}")
    if precision == capi.TL_GEMM_TF32:
        # TF32 gradients differ from the exact ones at 1e-3, so AdamW's
        # sign-like first steps differ on more elements
        assert upd <= 0.1
        return
    if precision == capi.TL_GEMM_3XTF32:
        assert upd <= 1e-3
        return
    assert upd <= 1e-4
    flipped, worst, off = 0, 0.0, 0
    for n in sizes:
        g, c = p2[off:off + n].astype(np.float64), o["p2"][off:off + n].astype(np.float64)
        off += n
        bad = np.abs(g - c) > rtol * np.abs(c)
        flipped += int(bad.sum())
        ok = ~bad
        if ok.any():
            worst = max(worst, float(np.max(np.abs(g[ok] - c[ok]) / np.abs(c[ok]).clip(1e-30))))
    print(f"elements outside {rtol:g}: {flipped} of {p2.size}; worst other {worst:.2e}")
    assert flipped <= p2.size // 200  # measured 0.14 % for FP32


def test_deterministic_and_graph_replay_is_bit_exact():
    rng = np.random.default_rng(3)
    x, y = zipf(rng, 4, 64)
    runs = []
    p0 = None
    for graphs, fusion, deferred in ((1, 1, 1), (0, 1, 1), (0, 0, 1), (1, 1, 0)):
        g = CudaGPT(config(4, 64, graphs=graphs, fusion=fusion, deferred=deferred))
        if p0 is None:
            p0 = g.params()
        g.set_batch(x, y)
        losses = [g.train_step() for _ in range(4)]
        runs.append((losses, g.params(), g.stats()))
        g.close()
    (l1, p1, s1), (l2, p2, s2), (l3, p3, s3), (l4, p4, _) = runs
    assert l1 == l2 and np.array_equal(p1, p2)  # replay == eager, bit for bit
    assert l1 == l4 and np.array_equal(p1, p4)  # run to run (and deferred wait), bit for bit
    assert s1["replays"] > 0 and s1["captures"] > 0
    assert s1["plan_hits"] > 0 and s3["plan_hits"] == 0  # optimised programs reused
    assert s2["replays"] == 0
    assert s1["fused"] > 0 and s3["fused"] == 0
    # fused kernels vs the unfused program: same math, different rounding
    # order; the updates agree to 1% in norm (AdamW normalises every update)
    d1, d3 = p1 - p0, p3 - p0
    assert np.linalg.norm(d1 - d3) <= 1e-2 * np.linalg.norm(d3)
    np.testing.assert_allclose(l1, l3, rtol=1e-4)


def test_full_size_step_runs():
    rng = np.random.default_rng(1)
    g = CudaGPT(config(64, 192))
    x, y = zipf(rng, 64, 192)
    g.set_batch(x, y)
    first = g.train_step()
    for _ in range(3):
        last = g.train_step()
    assert abs(first - np.log(2048)) < 0.5 and last < first
    g.close()


def test_flash_attention_replay_is_bit_exact():
    """Attention on the flash kernels (P kept as its recipe between the
    forward and backward windows): graph replay equals eager launches bit
    for bit, run to run, and tracks the short-sequence kernels' step."""
    rng = np.random.default_rng(4)
    x, y = zipf(rng, 4, 128)
    runs = []
    for graphs, flash in ((1, 1), (0, 1), (1, 1), (1, 0)):
        g = CudaGPT(config(4, 128, graphs=graphs, flash=flash))
        g.set_batch(x, y)
        runs.append(([g.train_step() for _ in range(4)], g.params()))
        g.close()
    (l1, p1), (l2, p2), (l3, p3), (l4, _) = runs
    assert l1 == l2 and np.array_equal(p1, p2)  # replay == eager
    assert l1 == l3 and np.array_equal(p1, p3)  # run to run
    np.testing.assert_allclose(l1, l4, rtol=1e-3)  # flash vs fused short-sequence kernels
