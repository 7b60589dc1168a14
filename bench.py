#!/usr/bin/env python3
"""Benchmark of the TempLit B200 backend on BASELINE.json's headline metric:
tokens/s of the GPT d384 training step (configuration 4: vocab 2048, T 192,
d_model 384, 4 pre-RMSNorm blocks, 6 heads, FFN 1536, batch 64 per GPU,
Zipf(1.1) tokens, N(0, 0.02) weights, AdamW 3e-4 (0.9, 0.95) wd 0.1,
clip 1.0), run through the reference's own model and compiler
(nn::GPT + passes::Compiled) on cuda::Runtime via include/templit_gpt.h.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

One process per GPU (torchrun for N > 1); data parallel with one NCCL
gradient all-reduce per step inside the runtime, per-GPU batch fixed
(weak scaling).  Rank 0 prints one JSON line.  --impl reference times the
CPU implementation of the same step (the oracle port of the reference's
runtime ops, all host threads) on a bounded sample.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GPT d384 train tokens/s at 1/2/4/8 B200; GEMM/attn/HBM % roofline"
VOCAB, SEQ, DMODEL, BLOCKS, HEADS, FFN = 2048, 192, 384, 4, 6, 1536
WORKLOAD = ("configs[3] GPT train step: vocab 2048, T=192, d=384, 4 pre-RMSNorm blocks, "
            "6 heads, GELU FFN 1536, batch 64 per GPU, AdamW 3e-4 (0.9,0.95) wd 0.1, clip 1.0")
WORKLOAD5 = ("configs[4] data-parallel GPT train step: vocab 2048, T=1024, d=768, 12 pre-RMSNorm "
             "blocks, 12 heads, GELU FFN 3072, global batch 256 sequences split over the GPUs, "
             "micro-batches (config.micro_batch sequences each) accumulated before one clipped "
             "AdamW step, NCCL gradient all-reduce, AdamW 3e-4 (0.9,0.95) wd 0.1, clip 1.0")


def _measured_hbm_gbs():
    """HBM copy bandwidth of this pool's B200s (MEASURED_PEAKS.json, written
    by the pool's driver; 6546.2 GB/s when it was measured for this repo)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6546.2


HBM_PEAK_GBS = _measured_hbm_gbs()


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    p.add_argument("--batch", type=int, default=64, help="sequences per GPU (configuration 4)")
    p.add_argument("--micro-batch", type=int, default=4,
                   help="configuration 5: sequences per forward/backward pass; the GPU's 256 / "
                        "n_gpus sequences of a step run as micro-batches of this size")
    p.add_argument("--config", type=int, choices=[4, 5], default=4,
                   help="4: the d384 GPT of configs[3] (the headline); 5: the 12-block d768 "
                        "T=1024 data-parallel GPT of configs[4]")
    p.add_argument("--no-fusion", action="store_true")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--profile", default="", help="write the per-op profile JSON here")
    p.add_argument("--kernel", choices=["gemm", "attention", "flash", "hbm", "infer"], default="",
                   help="time one kernel case instead of the training step (profiling "
                        "driver): a tl_gemm shape, configuration 3's attention (short-"
                        "sequence fused kernels), the flash kernels at configurations 3 and "
                        "5, or the step's memory-bound kernels at configuration 4's shapes")
    p.add_argument("--shape", default="12288x384x384:NN",
                   help="--kernel gemm: MxNxK:form[:gelu_grad|:addend|:bias_gelu]")
    return p.parse_args()


# ------------------------------------------------------------------ inputs
def zipf_batch(rng, batch, seq, vocab=VOCAB, s=1.1):
    """One Zipf(1.1) token stream over [0, vocab) cut into `batch` windows of
    seq + 1 (inputs = [:seq], targets = [1:], as the reference loader)."""
    p = 1.0 / np.arange(1, vocab + 1, dtype=np.float64) ** s
    stream = rng.choice(vocab, size=batch * (seq + 1), p=p / p.sum()).astype(np.uint32)
    w = stream.reshape(batch, seq + 1)
    return np.ascontiguousarray(w[:, :seq]), np.ascontiguousarray(w[:, 1:])


# --------------------------------------------------------------- clocks
class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.rows = []
        self.proc = None
        self.thread = None
        self.start = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            # nvidia-smi takes a moment to start: wait (at most 10 s) for its
            # first row, so samples cover the timed region that follows
            t0 = time.monotonic()
            while not self.rows and self.proc.poll() is None and time.monotonic() - t0 < 10:
                time.sleep(0.02)
            self.start = len(self.rows)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *exc):
        if self.proc:
            # one more row when the region was shorter than the interval
            t0, n = time.monotonic(), len(self.rows)
            while (len(self.rows) == n and len(self.rows) < 3 and self.proc.poll() is None
                   and time.monotonic() - t0 < 1):
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        # the rows taken during the region (the one after it if none was)
        rows = self.rows[self.start:] or self.rows[-1:]
        sm = [float(r[1]) for r in rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows if len(r) >= 9
                          for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------ CPU baseline
def cpu_baseline_gpt(steps=1, batch=2, warmup=1):
    """The same GPT step on the host: the oracle port of the reference's
    runtime ops (oracle/cpu_ref) driven by the reference's passes::Compiled,
    all host threads.  Bounded sample: `batch` sequences of 192 tokens."""
    from oracle import cpu_gpt
    if not cpu_gpt.available():
        return None
    threads = os.cpu_count() or 1
    tok_s, secs = cpu_gpt.train_tokens_per_s(batch=batch, seq=SEQ, steps=steps, threads=threads,
                                             warmup=warmup)
    return {"value": tok_s, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} GPT d384 train step(s) at batch {batch} x T {SEQ} "
                      f"({secs:.1f} s of CPU work) after {warmup} untimed, oracle port of the "
                      "reference runtime ops under the reference passes::Compiled executor"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    warm = max(3, min(args.warmup, 5))
    base = cpu_baseline_gpt(steps=max(1, min(args.steps, 3)), batch=2, warmup=warm)
    if base is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle CPU GPT port (oracle/_build/libgpt_cpu.so) is not built"}))
        return 0
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": max(1, min(args.steps, 3)), "warmup": warm,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (Zipf(1.1) tokens, N(0,0.02) weights)",
            # the workload of the cuda arm; what ran is cpu_baseline.sample
            "config": {"workload": WORKLOAD, "model": "nn::GPT<2048,192,384,6> (4 blocks)",
                       "global_batch": args.batch * args.gpus, "seq_len": SEQ,
                       "parallelism": f"dp{args.gpus}"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


# ----------------------------------------------------------------- roofline
def gemm_roofline(profile_path, peak_tflops, peak_source, timed_ms_per_step=None):
    """Dominant kernel: the tcgen05 GEMM.  The profiled step (an event pair
    around every op) gives the GEMMs' share of the step; achieved = executed
    GEMM FLOPs per step / (that share x the timed steps' ms per step)."""
    with open(profile_path) as f:
        prof = json.load(f)["ops"]
    flops = ms = 0.0
    launches = 0
    total_ms = sum(o["ms"] for o in prof)
    for o in prof:
        if not o["op"].startswith("gemm"):
            continue
        parts = o["op"].split()
        m, n, k = (int(v) for v in parts[1].split("x"))
        batch = groups = 1
        for tok in parts[2:]:
            if tok.startswith("b"):
                batch = int(tok[1:])
            elif tok.startswith("g"):  # grouped launch: `groups` products
                groups = int(tok[1:])
        flops += 2.0 * m * n * k * batch * groups * o["calls"]
        ms += o["ms"]
        launches += o["calls"]
    if ms == 0:
        return None, prof
    # fused attention ops (tcgen05 kernels of their own): dense-count FLOPs
    # per pass, 4 B H T^2 D (scores + values, or dP + dQ) and 2 B H T^2 D
    # for the key-side product
    a_flops = a_ms = 0.0
    a_launches = 0
    # flash ops: forward 4 B H T^2 D, backward 8 B H T^2 D (the four
    # products; the recomputed S is not counted), a rebuilt P 2 B H T^2 D
    flash_mult = {"flash_fwd": 4.0, "flash_bwd": 8.0, "flash_probs": 2.0}
    for o in prof:
        name = o["op"].split()[0]
        if o["op"].startswith("attention#"):
            code, dims = o["op"][len("attention#"):].split()
            mult = 2.0 if code == "2" else 4.0
        elif name in flash_mult:
            dims, mult = o["op"].split()[1], flash_mult[name]
        else:
            continue
        b, h, t, d = (int(v) for v in dims.split("x"))
        a_flops += mult * b * h * t * t * d * o["calls"]
        a_ms += o["ms"]
        a_launches += o["calls"]
    share = ms / total_ms if total_ms else 1.0
    gemm_ms = share * timed_ms_per_step if timed_ms_per_step else ms
    achieved = flops / (gemm_ms * 1e-3) / 1e12
    return {"bound": "tensor", "kernel": "tc_gemm_kernel (tcgen05 kind::tf32)",
            "achieved": round(achieved, 1), "peak": peak_tflops, "unit": "TFLOP/s",
            "frac": round(achieved / peak_tflops, 4) if peak_tflops else None,
            "peak_source": peak_source,
            # dram__bytes_read.sum + dram__bytes_write.sum of one launch of the
            # step's most frequent product (ncu capture summarised in
            # profiles/tc_gemm_12288x384x384_NN.md): 19.55 MB = its algorithmic
            # reads (A once, B); C stays in L2 when the kernel ends
            "traffic": 19548928, "traffic_unit": "bytes per launch",
            "traffic_shape": "12288x384x384 NN",
            "flops_per_step": flops, "gemm_ms_per_step": round(gemm_ms, 4),
            "gemm_ms_profiled_step": round(ms, 4),
            "timing": "GEMM share of the profiled step x the timed steps' ms per step",
            "gemm_launches_per_step": launches,
            "gemm_share_of_step": round(ms / total_ms, 3) if total_ms else None,
            "attention": {"kernel": "attn_fwd / attn_bwd_q / attn_bwd_kv, or the flash kernels "
                                    "above T = 192 (tcgen05 kind::tf32; dense-count FLOPs)",
                          "flops_per_step": a_flops, "ms_per_step": round(a_ms, 4),
                          "launches_per_step": a_launches,
                          "achieved_tflops": round(a_flops / (a_ms * 1e-3) / 1e12, 1)
                          if a_ms else None,
                          "frac": round(a_flops / (a_ms * 1e-3) / 1e12 / peak_tflops, 4)
                          if a_ms and peak_tflops else None}}, prof


def hbm_roofline(prof):
    """The memory-bound ops of the profiled step (the runtime records each
    op's algorithmic bytes: operands read once, outputs written once):
    the one with the most device time, and all of them together, against
    the measured HBM copy bandwidth.  Times are per-op CUDA events of the
    profiled step, where events between the ops keep a kernel's launch from
    overlapping the previous kernel's tail (the timed steps overlap them)."""
    mem = [o for o in prof if o.get("bytes", 0) > 0 and o["ms"] > 0]
    if not mem:
        return None
    top = max(mem, key=lambda o: o["ms"])
    gbs = lambda b, ms: b / (ms * 1e-3) / 1e9
    tb, tms = sum(o["bytes"] for o in mem), sum(o["ms"] for o in mem)
    return {"bound": "hbm", "kernel": top["op"], "launches_per_step": top["calls"],
            "achieved": round(gbs(top["bytes"], top["ms"]), 1), "peak": HBM_PEAK_GBS,
            "unit": "GB/s", "frac": round(gbs(top["bytes"], top["ms"]) / HBM_PEAK_GBS, 4),
            "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)",
            "bytes_per_step": top["bytes"], "ms_per_step": round(top["ms"], 4),
            "traffic": None,
            "all_memory_bound_ops": {"ms_per_step": round(tms, 4), "bytes_per_step": tb,
                                     "achieved": round(gbs(tb, tms), 1),
                                     "frac": round(gbs(tb, tms) / HBM_PEAK_GBS, 4)},
            "timing": "per-op CUDA events of one profiled step"}


def measure_tf32_peak(torch):
    """cuBLAS TF32 dense throughput on this GPU (8192^3, best of 10): the
    denominator for the TF32 GEMM (MEASURED_PEAKS.json holds bf16 only)."""
    torch.backends.cuda.matmul.allow_tf32 = True
    n = 8192
    a = torch.randn(n, n, device="cuda")
    b = torch.randn(n, n, device="cuda")
    for _ in range(3):
        a @ b
    torch.cuda.synchronize()
    best = None
    for _ in range(10):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        a @ b
        e.record()
        e.synchronize()
        t = s.elapsed_time(e)
        best = t if best is None else min(best, t)
    del a, b
    return 2.0 * n ** 3 / (best * 1e-3) / 1e12


# ----------------------------------------------------------------- main arm
def run_kernel_case(args):
    """One kernel case on cuda:0, --warmup untimed then --steps timed launches
    (CUDA events, L2 flushed between launches); one JSON line.  gemm: tl_gemm
    on the --shape operands (N(0,1), TF32).  attention: configuration 3
    (B 64, H 6, T 192, D 64, causal, divisor 8) through tl_attention_fwd and
    tl_attention_bwd."""
    import torch
    from templit_b200 import capi
    lib = capi.cuda_lib()
    dev = torch.device("cuda", 0)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def timed(fn):
        """Median device time of fn's launches: L2 flushed before each, and
        a 0.1 ms spin kernel ahead of the start event, so the launches are
        queued behind it and the events see device time only (not the host's
        launch latency, which the step's CUDA graphs do not have)."""
        for _ in range(max(3, args.warmup)):
            fn()
        ts = []
        for _ in range(args.steps):
            flush.zero_()
            torch.cuda._sleep(200_000)
            a, b = torch.cuda.Event(True), torch.cuda.Event(True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        return float(np.median(ts))

    g = torch.Generator(device=dev).manual_seed(0)
    if args.kernel == "infer":
        return run_inference_case(args)
    if args.kernel == "hbm":
        return run_hbm_case(args, lib, dev, stream, timed)
    if args.kernel == "flash":
        return run_flash_case(args, lib, dev, stream, timed)
    if args.kernel == "gemm":
        parts = args.shape.split(":")  # MxNxK:form[:gelu_grad|:addend|:bias_gelu]
        dims, form = parts[0], parts[1]
        aux = parts[2] if len(parts) > 2 else ""
        m, n, k = (int(v) for v in dims.split("x"))
        ta, tb = form[0] == "T", form[1] == "T"
        a = torch.randn((k, m) if ta else (m, k), device=dev, generator=g)
        b = torch.randn((n, k) if tb else (k, n), device=dev, generator=g)
        c = torch.zeros((m, n), device=dev)
        d = capi.TlGemmDesc(a=a.data_ptr(), b=b.data_ptr(), c=c.data_ptr(), m=m, n=n, k=k,
                            trans_a=int(ta), trans_b=int(tb), precision=capi.TL_GEMM_TF32)
        x_aux = torch.randn((m, n), device=dev, generator=g) if aux else None
        bias = torch.randn(n, device=dev, generator=g)
        if aux == "gelu_grad":
            d.gelu_grad_x = x_aux.data_ptr()
        elif aux == "addend":
            d.addend = x_aux.data_ptr()
        elif aux == "bias_gelu":  # the FFN's first product: C = A B + bias, GELU(C)
            d.bias, d.gelu_out = bias.data_ptr(), x_aux.data_ptr()
        wsb = lib.tl_gemm_workspace_size(ctypes.byref(d))
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
        d.workspace, d.workspace_bytes = ws.data_ptr(), wsb
        us = timed(lambda: capi.check(lib.tl_gemm(ctypes.byref(d), stream), lib, "tl_gemm"))
        line = {"kernel": "tl_gemm", "shape": args.shape, "us_per_launch": round(us, 2),
                "tflops": round(2.0 * m * n * k / us / 1e6, 1)}
    else:
        B, H, T, D = 64, 6, 192, 64
        q, k, v, d_o = (torch.randn(B, H, T, D, device=dev, generator=g) for _ in range(4))
        mask = torch.triu(torch.full((T, T), float("-inf"), device=dev), 1)
        div = torch.tensor([8.0], device=dev)
        p = torch.empty(B, H, T, T, device=dev)
        o, dq, dk, dv = (torch.empty_like(q) for _ in range(4))
        ws = torch.empty(lib.tl_attention_workspace_size(B, T, H, D), dtype=torch.uint8,
                         device=dev)
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        fwd = lambda: capi.check(lib.tl_attention_fwd(
            P(q), P(k), P(v), P(div), P(mask), P(p), P(o), B, T, H, D, capi.TL_ATTN_BHTD,
            capi.TL_GEMM_TF32, P(ws), ws.numel(), stream), lib, "tl_attention_fwd")
        bwd = lambda: capi.check(lib.tl_attention_bwd(
            P(q), P(k), P(v), P(p), P(div), P(d_o), P(dq), P(dk), P(dv), B, T, H, D,
            capi.TL_ATTN_BHTD, capi.TL_GEMM_TF32, P(ws), ws.numel(), stream), lib,
            "tl_attention_bwd")
        fwd()
        us_f, us_b = timed(fwd), timed(bwd)
        flops = 4.0 * B * H * T * T * D  # dense count
        line = {"kernel": "tl_attention (configuration 3, causal)", "fwd_us": round(us_f, 2),
                "bwd_us": round(us_b, 2), "fwd_tflops_dense": round(flops / us_f / 1e6, 1),
                "bwd_tflops_dense": round(2 * flops / us_b / 1e6, 1)}
    print(json.dumps(line))
    return 0


def run_hbm_case(args, lib, dev, stream, timed):
    """The memory-bound kernels of the configuration-4 step at the step's own
    shapes (12288 token rows, d 384, FFN 1536, vocab 2048, 8.74 M
    parameters), L2 flushed before every timed launch.  Algorithmic bytes:
    every input element read once and every output element written once."""
    import torch
    from templit_b200 import capi
    P = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)
    c = lambda rc, what: capi.check(rc, lib, what)
    g = torch.Generator(device=dev).manual_seed(1)
    rnd = lambda *shape: torch.randn(*shape, device=dev, generator=g)
    R, D, F, V = 64 * SEQ, DMODEL, FFN, VOCAB
    out = []

    def case(name, nbytes, fn):
        us = timed(fn)
        gbs = nbytes / us / 1e3
        out.append({"kernel": name, "us": round(us, 2), "bytes": int(nbytes),
                    "GB_s": round(gbs, 1), "frac": round(gbs / HBM_PEAK_GBS, 3)})

    x, gr, y, add, o = (rnd(R, D) for _ in range(5))
    case("rmsnorm_rows [12288,384]", 8 * R * D,
         lambda: c(lib.tl_rmsnorm_rows(P(x), P(o), P(None), R, D, stream), "rmsnorm"))
    case("rmsnorm_backward_rows + residual [12288,384]", 20 * R * D,
         lambda: c(lib.tl_rmsnorm_backward_rows(P(gr), P(x), P(y), P(add), P(o), R, D, stream),
                   "rmsnorm backward"))
    sh = capi.shape_arr([R, D])
    case("binary add [12288,384]", 12 * R * D,
         lambda: c(lib.tl_binary(capi.TL_ADD, P(x), sh, 2, P(gr), sh, 2, P(o), sh, 2, stream),
                   "add"))
    for cols in (D, F, V):
        xs, os_ = capi.shape_arr([R, cols]), capi.shape_arr([1, cols])
        src = rnd(R, cols)
        wsb = lib.tl_reduce_workspace_size(xs, 2, os_, 2)
        ws = torch.empty(max(wsb, 16), dtype=torch.uint8, device=dev)
        dst = torch.empty(cols, device=dev)
        case(f"reduce (bias gradient) [12288,{cols}]->[{cols}]", 4 * R * cols,
             lambda src=src, xs=xs, os_=os_, ws=ws, wsb=wsb, dst=dst: c(lib.tl_reduce(
                 capi.TL_REDUCE_SUM, P(src), xs, 2, P(dst), os_, 2, P(ws), wsb, stream), "reduce"))
        del src
    z = rnd(R, V)
    dz = torch.empty_like(z)
    tg = torch.randint(0, V, (R,), device=dev, dtype=torch.int32, generator=g)
    loss = torch.empty(R, device=dev)
    case("xent_rows [12288,2048]", 4 * R * V,
         lambda: c(lib.tl_xent_rows(P(z), P(tg), P(loss), R, V, stream), "xent"))
    case("xent_backward_rows [12288,2048]", 8 * R * V,
         lambda: c(lib.tl_xent_backward_rows(P(z), P(tg), P(None), P(dz), R, V, stream),
                   "xent backward"))
    del z, dz
    table = rnd(V, D)
    emb = torch.empty(R, D, device=dev)
    case("embedding gather [2048,384] x 12288 ids", R * D * 4 + V * D * 4 + R * 4,
         lambda: c(lib.tl_embedding_gather(P(table), V, D, P(tg), R, P(emb), stream), "gather"))
    base = rnd(V, D)
    dst = torch.empty_like(base)
    swb = lib.tl_embedding_scatter_workspace_size(R, V, D)
    sws = torch.empty(max(swb, 16), dtype=torch.uint8, device=dev)
    case("embedding scatter-add 12288 x 384 -> [2048,384]", R * D * 4 + R * 4 + 2 * V * D * 4,
         lambda: c(lib.tl_embedding_scatter_add(P(emb), P(tg), R, D, P(base), P(dst), V, P(sws),
                                                swb, stream), "scatter"))
    # the optimiser pass over nn::GPT<2048,192,384,6>'s 52 parameter tensors
    sizes = [V * D, SEQ * D]
    for _ in range(BLOCKS):
        sizes += [D * D, D] * 4 + [D * F, F, F * D, D]
    sizes += [D * V, V]
    n_par = sum(sizes)
    flat = [rnd(n_par) * 0.02, rnd(n_par) * 0.05, rnd(n_par) * 1e-3, rnd(n_par).abs() * 1e-4]
    slots = (capi.TlParamSlot * len(sizes))()
    off = chunk = 0
    for i, n in enumerate(sizes):
        sl = slots[i]
        sl.param = sl.out = flat[0].data_ptr() + 4 * off
        sl.grad, sl.m1, sl.m2 = (t.data_ptr() + 4 * off for t in flat[1:])
        sl.count, sl.chunk0, sl.step = n, chunk, 3
        chunk += (n + capi.TL_OPT_CHUNK - 1) // capi.TL_OPT_CHUNK
        off += n
    dslots = torch.frombuffer(bytearray(bytes(slots)), dtype=torch.uint8).to(dev)
    sq = torch.zeros(1, device=dev)
    scal = [torch.tensor([v], device=dev) for v in (0.9, 0.95, 1 - 3e-4 * 0.1, 3e-4)]
    owb = lib.tl_multi_clip_adamw_workspace_size(chunk)
    ows = torch.empty(max(owb, 16), dtype=torch.uint8, device=dev)

    def adamw():  # sqnorm accumulates over the calls: the clip factor only changes
        c(lib.tl_multi_clip_adamw(P(dslots), len(sizes), chunk, P(sq), ctypes.c_float(1.0),
                                  *[P(t) for t in scal], ctypes.c_float(1e-8), P(ows), owb,
                                  stream), "adamw")
    case(f"multi-tensor norm + clip + AdamW ({n_par} parameters, 52 tensors)", 32 * n_par, adamw)
    print(json.dumps({"kernel": "memory-bound kernels of the configuration-4 step",
                      "peak_GB_s": HBM_PEAK_GBS, "peak_source": "MEASURED_PEAKS.json hbm_gbs",
                      "l2": "flushed (256 MB written) before every timed launch",
                      "cases": out}))
    return 0


def run_flash_case(args, lib, dev, stream, timed):
    """The flash attention kernels (tl_flash_attention_fwd / _bwd, causal
    mask, divisor 8) at configuration 3 (B 64, H 6, T 192) and at
    configuration 5's T = 1024 (B 8 and B 32, H 12).  FLOPs are the dense
    count of the algorithm's products: forward S = QK^T and O = PV (4 B H T^2
    D); backward dP = dO V^T, dQ = dS K, dK = dS^T Q, dV = P^T dO (8 B H T^2
    D; the recomputation of S is not counted).  The causal kernels skip the
    key blocks above the diagonal, so half of those FLOPs are executed."""
    import torch
    from templit_b200 import capi
    out = []
    for B, H, T in ((64, 6, 192), (8, 12, 1024), (32, 12, 1024)):
        D = 64
        g = torch.Generator(device=dev).manual_seed(T)
        q, k, v, d_o = (torch.randn(B, H, T, D, device=dev, generator=g) for _ in range(4))
        o, dq, dk, dv = (torch.empty_like(q) for _ in range(4))
        mask = torch.triu(torch.full((T, T), float("-inf"), device=dev), 1)
        div = torch.tensor([8.0], device=dev)
        flag = torch.zeros(4, dtype=torch.int32, device=dev)
        lse, delta = torch.empty(B, H, T, device=dev), torch.empty(B, H, T, device=dev)

        def view(t):
            w = capi.TlAttnView()
            w.p = t.data_ptr()
            w.batch_stride, w.head_stride, w.row_stride = t.stride()[:3]
            return w
        d = capi.TlFlashDesc(B=B, T=T, H=H, D=D)
        d.q, d.k, d.v, d.o, d.d_o, d.dq, d.dk, d.dv = (view(t) for t in (q, k, v, o, d_o, dq, dk,
                                                                             dv))
        d.divisor, d.mask, d.mask_flag = div.data_ptr(), mask.data_ptr(), flag.data_ptr()
        d.lse, d.delta = lse.data_ptr(), delta.data_ptr()
        capi.check(lib.tl_attention_mask_check(ctypes.c_void_p(mask.data_ptr()), T,
                                               ctypes.c_void_p(flag.data_ptr()), stream),
                   lib, "mask check")
        fwd = lambda: capi.check(lib.tl_flash_attention_fwd(ctypes.byref(d), stream), lib, "fwd")
        bwd = lambda: capi.check(lib.tl_flash_attention_bwd(ctypes.byref(d), stream), lib, "bwd")
        fwd()
        us_f, us_b = timed(fwd), timed(bwd)
        dense = 4.0 * B * H * T * T * D
        out.append({"B": B, "H": H, "T": T, "fwd_us": round(us_f, 2), "bwd_us": round(us_b, 2),
                    "fwd_tflops_dense": round(dense / us_f / 1e6, 1),
                    "bwd_tflops_dense": round(2 * dense / us_b / 1e6, 1)})
        del q, k, v, d_o, o, dq, dk, dv
    print(json.dumps({"kernel": "tl_flash_attention (causal, D 64)", "cases": out}))
    return 0


def run_inference_case(args):
    """Forward-only generation (src/generate.cpp's set-up: batch 1, T 192,
    top-k 40, temperature 0.6, minimum length 64) through tlg_infer_generate:
    the reference's inference::autoregression recomputes the whole context
    per token and samples on the host.  Wall-clock tokens/s over --steps
    generations, beside the host oracle on a bounded sample."""
    from templit_b200 import capi
    lib = capi.gpt_lib()
    cfg = capi.TlgConfig(family=4, batch=1, seq=SEQ, seed=1234, init_std=0.02, lr=3e-4,
                         beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0, world=1,
                         fusion=1, graphs=1, gemm_precision=capi.TL_GEMM_TF32, deferred_wait=0)
    h = ctypes.c_void_p()
    capi.check(lib.tlg_infer_create(ctypes.byref(cfg), ctypes.byref(h)), lib, "infer create")
    prompt = np.random.default_rng(3).integers(1, VOCAB, 16).astype(np.uint32)
    out = np.zeros(4096, np.uint32)
    n = ctypes.c_uint32()
    U = ctypes.POINTER(ctypes.c_uint32)

    def gen(seed):
        capi.check(lib.tlg_infer_generate(h, prompt.ctypes.data_as(U), prompt.size, 0, seed, 40,
                                          0.6, 64, out.ctypes.data_as(U), out.size,
                                          ctypes.byref(n)), lib, "generate")
        return n.value

    for i in range(max(1, args.warmup)):
        gen(100 + i)
    tokens, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        tokens += gen(i)
    dt = time.perf_counter() - t0
    capi.check(lib.tlg_infer_destroy(h), lib, "infer destroy")
    line = {"kernel": "inference (generate.cpp set-up: B 1, T 192, top-k 40)",
            "tokens": tokens, "tokens_per_s": round(tokens / dt, 1),
            "ms_per_token": round(1e3 * dt / max(tokens, 1), 3)}
    try:
        from oracle import cpu_gpt
        if cpu_gpt.available():
            ref = cpu_gpt.OracleGPTInference(cfg)
            t0 = time.perf_counter()
            ref.logits(np.zeros(SEQ, np.uint32))  # one forward = one generated token
            line["oracle_ms_per_token"] = round(1e3 * (time.perf_counter() - t0), 1)
            ref.close()
    except Exception as exc:  # the line still prints
        line["oracle_error"] = str(exc)
    print(json.dumps(line))
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.kernel:
        return run_kernel_case(args)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from templit_b200 import capi

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    lib = capi.gpt_lib()
    if args.config == 5:
        if 256 % world or (256 // world) % args.micro_batch:
            raise SystemExit("configuration 5 splits 256 sequences: use 1, 2, 4 or 8 GPUs and a "
                             "micro-batch that divides 256 / n_gpus")
        family, seq, batch = 12, 1024, args.micro_batch
        micro = (256 // world) // batch
    else:
        family, seq, batch, micro = 4, SEQ, args.batch, 1
    cfg = capi.TlgConfig(family=family, batch=batch, seq=seq, seed=1234, init_std=0.02,
                         lr=3e-4, beta1=0.9, beta2=0.95, eps=1e-8, weight_decay=0.1, clip=1.0,
                         world=world, fusion=0 if args.no_fusion else 1,
                         graphs=0 if args.no_graphs else 1, deferred_wait=1,
                         micro_batches=micro)
    h = ctypes.c_void_p()
    capi.check(lib.tlg_create(ctypes.byref(cfg), ctypes.byref(h)), lib, "tlg_create")
    if world > 1:
        uid = (ctypes.c_uint8 * 128)()
        if rank == 0:
            capi.check(lib.tlg_nccl_unique_id(uid), lib, "nccl id")
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=0)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(box[0])
        capi.check(lib.tlg_set_communicator(h, uid, world, rank), lib, "communicator")

    stream = torch.cuda.ExternalStream(lib.tlg_stream(h))
    rng = np.random.default_rng(1000 + rank)
    B, T = batch * micro, seq  # sequences of one rank's step (all micro-batches)
    n_tok = B * T
    pin_x = torch.empty(n_tok, dtype=torch.int32).pin_memory()
    pin_y = torch.empty(n_tok, dtype=torch.int32).pin_memory()
    u32 = ctypes.POINTER(ctypes.c_uint32)

    def load(x, y):
        pin_x.numpy().view(np.uint32)[:] = x.ravel()
        pin_y.numpy().view(np.uint32)[:] = y.ravel()
        capi.check(lib.tlg_set_batch(h, ctypes.cast(pin_x.data_ptr(), u32),
                                     ctypes.cast(pin_y.data_ptr(), u32)), lib, "set_batch")

    loss = ctypes.c_float()

    def step():
        capi.check(lib.tlg_train_step(h, ctypes.byref(loss)), lib, "train_step")
        return loss.value

    batches = [zipf_batch(rng, B, T) for _ in range(4)]
    load(*batches[0])
    losses = [step() for _ in range(max(3, args.warmup))]

    # e2e input path: the repo's token pipeline (tlg_loader_*: the reference's
    # Dataset + Loader sampling, pinned buffers, prefetch thread) over a
    # synthetic Zipf(1.1) token file
    import tempfile
    p_zipf = 1.0 / np.arange(1, VOCAB + 1, dtype=np.float64) ** 1.1
    stream_tokens = rng.choice(VOCAB, size=1 << 22, p=p_zipf / p_zipf.sum()).astype(np.uint32)
    tok_file = tempfile.NamedTemporaryFile(suffix=".tokens", delete=False)
    stream_tokens.tofile(tok_file.name)
    tok_file.close()
    loader = ctypes.c_void_p()
    capi.check(lib.tlg_loader_create(tok_file.name.encode(), 0.95, 0, B, T, 1 + rank,
                                     ctypes.byref(loader)), lib, "loader")
    lx, ly = capi.U32P(), capi.U32P()

    def load_next():
        capi.check(lib.tlg_loader_next(loader, ctypes.byref(lx), ctypes.byref(ly)), lib, "next")
        capi.check(lib.tlg_set_batch(h, lx, ly), lib, "set_batch")

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(with_host_io):
        """K steps between two events on the backend stream (max over
        ranks), plus an event after every step for the per-step median."""
        barrier()
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        evs[0].record(stream)
        for i in range(args.steps):
            if with_host_io:
                load_next()
            losses.append(step())
            evs[i + 1].record(stream)
        evs[-1].synchronize()
        barrier()
        ms = evs[0].elapsed_time(evs[-1])
        per = [evs[i].elapsed_time(evs[i + 1]) for i in range(args.steps)]
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms, per

    stats0 = (ctypes.c_uint64 * 11)()
    capi.check(lib.tlg_stats(h, stats0), lib, "stats")
    with ClockSampler(local) as clocks:
        ms_value, per_value = timed(with_host_io=False)
        ms_e2e, per_e2e = timed(with_host_io=True)
    stats1 = (ctypes.c_uint64 * 11)()
    capi.check(lib.tlg_stats(h, stats1), lib, "stats")
    kernels = int(stats1[3] - stats0[3]) // 2  # two timed regions of K steps each

    total_tokens = n_tok * world * args.steps
    value = total_tokens / (ms_value * 1e-3)
    e2e = total_tokens / (ms_e2e * 1e-3)

    roof = roof_hbm = None
    prof_path = args.profile or os.path.join(tempfile.gettempdir(),
                                             f"templit_gpt_profile_{os.getpid()}_rank{rank}.json")
    try:
        os.makedirs(os.path.dirname(prof_path), exist_ok=True)
        capi.check(lib.tlg_profile(h, prof_path.encode(), 1), lib, "profile")
        step()
        if rank == 0:
            peak = measure_tf32_peak(torch)
            roof, prof = gemm_roofline(prof_path, round(peak, 1),
                                       "cuBLAS TF32 8192^3 measured in this run (burst)",
                                       ms_value / args.steps)
            roof_hbm = hbm_roofline(prof)
    except Exception as exc:  # the bench line still prints
        roof = {"error": str(exc)}
    # GEMM launches by path over the whole run (eager windows and captures;
    # replays re-launch what was captured): a product the tensor-core path
    # refused would run on the CUDA cores
    g_tc, g_simt, g_refused = (ctypes.c_uint64() for _ in range(3))
    capi.cuda_lib().tl_gemm_counters(ctypes.byref(g_tc), ctypes.byref(g_simt),
                                     ctypes.byref(g_refused))

    if world > 1:
        dist.barrier()
    capi.check(lib.tlg_loader_destroy(loader), lib, "loader destroy")
    os.unlink(tok_file.name)
    capi.check(lib.tlg_destroy(h), lib, "destroy")
    if world > 1:
        dist.destroy_process_group()
    if g_simt.value:
        print(f"bench: {g_simt.value} GEMM launches ran on the CUDA cores "
              f"({g_refused.value} refused by the tensor-core path)", file=sys.stderr)
        return 1
    if rank != 0:
        return 0
    # about 10 s of CPU work: one step at batch 16
    cpu = cpu_baseline_gpt(steps=1, batch=16) if world == 1 and args.config == 4 else None
    line = {
        "metric": METRIC if args.config == 4 else
                  "GPT d768 12-block T1024 data-parallel train tokens/s (configs[4])",
        "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": round(ms_value / args.steps, 4),
        "ms_per_step_median": round(statistics.median(per_value), 4),
        "ms_per_step_p10_p90": [round(float(np.percentile(per_value, 10)), 4),
                                round(float(np.percentile(per_value, 90)), 4)],
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (Zipf(1.1) token windows; e2e draws them with the token pipeline "
                "from a Zipf(1.1) token file; N(0,0.02) weights, zero biases)",
        "config": {"workload": WORKLOAD if args.config == 4 else WORKLOAD5,
                   "model": "nn::GPT<2048,192,384,6> (4 blocks)" if args.config == 4 else
                            "12 nn::DecoderBlock<768,12> (d768, FFN 3072, vocab 2048, T 1024)",
                   "micro_batches": micro, "micro_batch": batch,
                   "global_batch": B * world, "seq_len": T, "parallelism": f"dp{world}",
                   "gemm_operands": "tf32 tensor cores, fp32 accumulate",
                   "l2": "per-step activations (GBs) exceed the 126 MB L2"},
        "e2e": {"value": round(e2e, 1), "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * n_tok * 4, "d2h_bytes_per_step": n_tok * 4,
                "ms_per_step_median": round(statistics.median(per_e2e), 4)},
        "gemm_launches_by_path": {"tensor_core": g_tc.value, "cuda_core": g_simt.value},
        "gpu_launches": kernels,
        "roofline": roof, "roofline_hbm": roof_hbm, "cpu_baseline": cpu, "clocks": clocks.summary(),
        "loss_first_last": [round(losses[0], 4), round(losses[-1], 4)],
        "runtime": {"windows": int(stats1[0]), "ops_recorded": int(stats1[1]),
                    "ops_launched": int(stats1[2]), "graph_replays": int(stats1[4]),
                    "graph_captures": int(stats1[5]), "fused_ops": int(stats1[6]),
                    "peak_device_bytes": int(stats1[7]),
                    "host_ms_per_step": round((stats1[8] + stats1[9] - stats0[8] - stats0[9])
                                              / 2e6 / args.steps, 3),
                    "optimiser_cache_hits": int(stats1[10])},
    }
    print(json.dumps(line))
    return 0


if __name__ == "__main__":
    sys.exit(main())
