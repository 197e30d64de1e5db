#!/usr/bin/env python3
"""Benchmark of the math-plus CUDA backend's GEMM / fused-attention path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

For N > 1 launch one rank per GPU with torch.distributed.run; every rank runs its own shard
(weak scaling: independent batches, no data-path collective) and rank 0 prints ONE JSON line.

A step is one pass of the hot path over one batch of synthetic input:

  batched_gemm_bf16 (default)  64 x [2048x2048]·[2048x2048] bf16 -> f32, fused +bias[2048] and
                               exact-erf GELU: math-plus Backend.matmul -> add -> gelu
                               (packages/tensor-cpu/src/index.ts:755-762, :598) as one kernel.
  causal_attention_f16         causal sdpa, Q/K/V [16, 32, 2048, 128] f16, scale 1/sqrt(128), f16 out
                               (+ f32 log-sum-exp): Backend.sdpa (index.ts:821-840) as one kernel.
  gpt2_attention_bf16          the same op at GPT-2-small's attention shape, causal bf16 [32, 12, 1024,
                               64] (a profiling case for the forward's attention launches).
  gemm_f32_1024                one f32 1024^3 GEMM (3xTF32 on the tensor cores); L2 is flushed
                               between timed steps (the inputs are 8 MiB).
  nsplit_gemm_bf16             C[16384,65536] = A[16384,8192] @ B[8192,65536] bf16 -> bf16 with B's
                               columns split over the N ranks (strong scaling: the total work is
                               fixed); each rank's GEMM epilogue stores its blocks into every rank's
                               shard-major copy of C over NVLink (the all-gather fused into the
                               GEMM), then a local permute to row-major. The line also carries the
                               blocked-view-only, GEMM-only and GEMM + NCCL all-gather + permute times.
  fused_elementwise_f32        the tensor-compile chain (x + y) * z -> sigmoid -> relu over three f32
                               inputs of 2^28 elements, fused into one kernel (WebGpuDevice.fuse,
                               packages/tensor-webgpu/src/facade.ts:137-164; the chain of
                               packages/tensor-webgpu/test/fusion.test.ts:157-163); GB/s of the
                               16 bytes each element reads and writes.

The default run (batched_gemm_bf16) also times causal_attention_f16 and reports it under
"secondary" in the same line (the metric's fused-attention half); --no-secondary skips it.
--threshold-sweep measures the host-array GEMM crossover behind tensor_cuda.caps.choose_gemm_backend.

``value`` is device-timed throughput with inputs resident in HBM (CUDA events on the launching
stream, barrier + synchronize around the timed region, max over ranks). ``e2e`` runs the same
step through the C ABI from pinned HOST buffers: the host->device copies of the inputs and the
device->host read of the result are inside its timed region. ``--impl reference`` times the
reference's CPU algorithm (the oracle's restatement of tensor-core gemmNT / attention,
packages/tensor-core/src/kernels.ts:299-362, nn-kernels.ts:179-239) on a bounded sample of the
same workload with all host threads. Inputs are seeded synthetic data with the configuration's
shapes and distributions (torch's RNG on the device).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "math-plus_b200"))

WORKLOADS = {
    "batched_gemm_bf16": dict(kind="gemm", batch=64, m=2048, n=2048, k=2048, dtype="bf16", out="f32",
                              epilogue="bias+gelu", metric="GEMM TFLOP/s (batched bf16 GEMM + bias + GELU)",
                              desc="batched GEMM bf16 in / f32 accumulate+out, 64x2048^3, +bias[2048], exact GELU"),
    "gemm_f32_1024": dict(kind="gemm", batch=1, m=1024, n=1024, k=1024, dtype="f32", out="f32", epilogue="none",
                          metric="GEMM TFLOP/s (f32, 3xTF32)", desc="single f32 GEMM 1024^3 (3xTF32 on tcgen05)"),
    "nsplit_gemm_bf16": dict(kind="nsplit", batch=1, m=16384, n=65536, k=8192, dtype="bf16", out="bf16",
                             epilogue="none", metric="GEMM TFLOP/s (column-split bf16 GEMM + all-gather)",
                             desc="C[16384,65536] = A[16384,8192] @ B[8192,65536] bf16, B's columns split over "
                                  "the ranks, every rank ends with the whole C (GEMM fused with its all-gather)"),
    "gpt2_forward_bf16": dict(kind="gpt2", batch=32, seq=1024, dtype="bf16",
                              metric="GPT-2-small forward TFLOP/s (bf16)",
                              desc="GPT-2-small-shaped forward (12 layers, d 768, 12 heads, d_ff 3072, vocab 50257), "
                                   "batch 32 x 1024 tokens, random-init bf16 weights ~ N(0, 0.02), logits bf16"),
    "fused_elementwise_f32": dict(kind="fusion", n=1 << 28, dtype="f32", unit="GB/s",
                                  metric="fused element-wise GB/s ((x + y) * z -> sigmoid -> relu, f32)",
                                  desc="one fused kernel over three f32 inputs of 2^28 elements: "
                                       "relu(sigmoid((x + y) * z)), f64 evaluation, f32 out (16 bytes per element)"),
    "causal_attention_f16": dict(kind="attention", batch=16, heads=32, seq=2048, head_dim=128, dtype="f16",
                                 causal=True, metric="fused attention TFLOP/s (causal f16)",
                                 desc="causal sdpa f16 [16,32,2048,128], scale 1/sqrt(128), f16 out + f32 LSE"),
    "gpt2_attention_bf16": dict(kind="attention", batch=32, heads=12, seq=1024, head_dim=64, dtype="bf16",
                                causal=True, metric="fused attention TFLOP/s (causal bf16, GPT-2 shape)",
                                desc="causal sdpa bf16 [32,12,1024,64] (one GPT-2-small layer's attention at "
                                     "batch 32 x 1024 tokens), scale 1/8, bf16 out + f32 LSE"),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="batched_gemm_bf16", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20,
                    help="streamed end-to-end steps (the pipeline fills and drains once per region)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-secondary", action="store_true",
                    help="time only --workload (the default run also times the causal attention configuration)")
    ap.add_argument("--threshold-sweep", action="store_true",
                    help="measure the host-array GEMM crossover (device end to end vs one CPU thread) and exit")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU work for the baseline sample")
    ap.add_argument("--batch", type=int, default=None, help="override the per-rank batch (small profiling cases)")
    ap.add_argument("--elements", type=int, default=None,
                    help="override the element count of the fused element-wise workload (small profiling cases)")
    ap.add_argument("--expression", default="sigmoid_chain", choices=sorted(EXPRESSIONS),
                    help="the fused element-wise workload's expression")
    ap.add_argument("--precision", default="f64", choices=["f64", "f32"],
                    help="the fused element-wise workload's evaluation precision (f64: the CPU evaluator's "
                         "numbers; f32: the WebGPU backend's)")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profiled_traffic(key: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/*<key>*.txt)."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for fn in sorted(os.listdir(pdir)):
        if key in fn and fn.endswith(".txt"):
            with open(os.path.join(pdir, fn)) as f:
                for line in f:
                    if line.startswith("traffic_bytes_per_launch:"):
                        try:
                            return float(line.split(":", 1)[1].split()[0])
                        except ValueError:
                            return None
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, bus_id):
        self.bus_id, self.proc, self.lines, self.t = bus_id, None, [], None

    def _read(self):
        for x in self.proc.stdout:
            self.lines.append(x.strip())

    def start(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.bus_id:
            cmd += ["-i", self.bus_id]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.t:
            self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def dist_env():
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


def unit_of(w):
    """(unit, scale): throughput is work per second / scale."""
    return (w["unit"], 1e9) if w.get("unit") == "GB/s" else ("TFLOP/s", 1e12)


# The fused element-wise workload's expressions over inputs x, y, z: the reference's fused chain
# (fusion.test.ts:157-163), and an exact-GELU chain whose cost is the erf evaluation.
EXPRESSIONS = {
    "sigmoid_chain": ("relu(sigmoid((x + y) * z))", lambda x, y, z: x.add(y).mul(z).sigmoid().relu()),
    "gelu_chain": ("gelu(x * y + 1) + z", lambda x, y, z: x.mul(y).add(1).gelu().add(z)),
}


def fusion_expr(w=None):
    sys.path.insert(0, os.path.join(ROOT, "math-plus_b200"))
    from tensor_cuda.fusion import Traced
    name = (w or {}).get("expression", "sigmoid_chain")
    return EXPRESSIONS[name][1](Traced.input(0), Traced.input(1), Traced.input(2))


def flop_per_step(w):
    """Work per step: FLOP, or bytes for the HBM-bound fused element-wise workload."""
    if w["kind"] == "fusion":
        return 16.0 * w["n"]
    if w["kind"] == "gpt2":
        sys.path.insert(0, os.path.join(ROOT, "math-plus_b200"))
        from tensor_cuda.gpt2 import GPT2Config
        return GPT2Config().forward_flop(w["batch"], w["seq"])
    if w["kind"] in ("gemm", "nsplit"):
        return 2.0 * w["batch"] * w["m"] * w["n"] * w["k"]
    f = 4.0 * w["batch"] * w["heads"] * w["seq"] * w["seq"] * w["head_dim"]
    return f / 2 if w["causal"] else f


# ---------------------------------------------------------------------------------------------
# CPU baseline: the oracle's restatement of the reference's CPU algorithm, all host threads
# ---------------------------------------------------------------------------------------------

def cpu_sample_rate(w: dict, target_s: float, threads: int):
    """Returns (flop/s, sample text, seconds) of the oracle on a sample of the workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    rng = np.random.default_rng(7)
    if w["kind"] == "fusion":
        node = fusion_expr(w).node
        n = 1 << 16
        while True:
            xs = [rng.standard_normal(n).astype(np.float32) for _ in range(3)]
            t0 = time.perf_counter()
            O.eval_ir(node, xs, w.get("precision", "f64"))
            dt = time.perf_counter() - t0
            if dt >= target_s / 4 or n >= w["n"]:
                break
            n = min(w["n"], n * 4)
        return 16.0 * n / dt, (f"{n} of the {w['n']} elements through the oracle's restatement of "
                               f"tensor-compile's evaluator (evalValue, {w.get('precision', 'f64')}, one thread)"), dt
    if w["kind"] == "gpt2":
        sys.path.insert(0, os.path.join(ROOT, "math-plus_b200"))
        from tensor_cuda.gpt2 import GPT2Config, random_weights
        full = GPT2Config()
        wts = random_weights(GPT2Config(n_layer=1), seed=3)
        f = {k: ((v.astype(np.uint32) << 16).view(np.float32).reshape(v.shape) if v.dtype == np.uint16 else v)
             for k, v in wts.items()}
        L = 64
        while True:
            ids = rng.integers(0, full.vocab, (1, L), dtype=np.int32)
            t0 = time.perf_counter()
            O.gpt2_forward(f, ids, 1, full.n_head, full.eps, threads=threads)
            dt = time.perf_counter() - t0
            if dt >= target_s / 4 or L >= w["seq"]:
                break
            L = min(w["seq"], L * 2)
        flop = GPT2Config(n_layer=1).forward_flop(1, L)
        return flop / dt, (f"a 1-layer full-width forward (embedding, block, LN, LM head over the 50257-token "
                           f"vocabulary) of one {L}-token sequence, f64 accumulate"), dt
    if w["kind"] == "attention":
        L, D = w["seq"], w["head_dim"]
        mask = np.tril(np.ones((L, L), np.bool_)).reshape(1, 1, L, L) if w["causal"] else None
        heads_total = w["batch"] * w["heads"]

        def run(nh):
            q, k, v = (rng.standard_normal((1, nh, L, D)).astype(np.float16).astype(np.float32) for _ in range(3))
            t0 = time.perf_counter()
            O.sdpa(q, k, v, mask, 1 / math.sqrt(D), threads=threads)
            return time.perf_counter() - t0

        nh = max(1, min(threads, heads_total))
        per_round = run(nh)  # one head per thread
        rounds = max(1, int(target_s / max(per_round, 1e-3)))
        nh = max(1, min(heads_total, rounds * threads))
        dt = run(nh)
        # the reference's CPU attention does the full Lq x Lk work per head (a causal mask is
        # applied element-wise); the rate is reported against the same causal FLOP count as the GPU
        flop = flop_per_step(w) / heads_total * nh
        return flop / dt, f"{nh} of the {heads_total} (b,h) heads [{L}x{D}], f64 accumulate", dt
    m, n_all, k = w["m"], w["n"], w["k"]
    n = min(n_all, 4096)  # a column block of a very wide B has the same per-FLOP cost
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)

    def run(rows):
        a = (rng.standard_normal((rows, k)) / np.sqrt(k)).astype(np.float32)
        t0 = time.perf_counter()
        c = O.matmul(a, b, threads=threads)
        if w["epilogue"] == "bias+gelu":
            O.gelu(O.add_f32(c, bias))
        return time.perf_counter() - t0

    rows = 16
    dt = run(rows)
    while dt < 0.5 and rows < m:
        rows = min(m, rows * 4)
        dt = run(rows)
    want_rows = max(16, int(rows / dt * target_s))
    rows = min(m, want_rows)
    reps = max(1, min(w["batch"], want_rows // m)) if want_rows > m else 1
    t = sum(run(rows) for _ in range(reps))
    flop = 2.0 * reps * rows * n * k
    cols = f"{k}x{n}" if n == n_all else f"{k}x{n} column block of the {k}x{n_all}"
    what = (f"{reps} of the {w['batch']} products {m}x{k} @ {cols}" if rows == m else
            f"{rows} of the {m} rows of one {m}x{k} @ {cols} product")
    return flop / t, what + (" (+bias, GELU), f64 accumulate" if w["epilogue"] == "bias+gelu"
                             else ", f64 accumulate"), t


# ---------------------------------------------------------------------------------------------
# The host-array GEMM crossover (chooseGemmBackend, packages/tensor-webgpu/src/threshold.ts:67-85)
# ---------------------------------------------------------------------------------------------

THRESHOLD_SHAPES = ([(n, n, n) for n in (8, 16, 24, 32, 48, 64, 96, 128, 160, 192, 256, 384, 512)] +
                    [(mn, kk, mn) for mn in (32, 64, 128, 256) for kk in (16, 64, 256, 1024, 4096)] +
                    [(16, 1024, 3072), (1, 768, 50257)])


def run_threshold_sweep(args):
    """Per (m, k, n): the device end to end from host f32 arrays (pageable A and B copied up, the f32
    GEMM, C copied back, wall clock, median) against the reference's CPU algorithm (the oracle's
    restatement of tensor-core gemmNT, one host thread). Prints one JSON line with every shape and
    the (m·n, m·n·k) thresholds that send the most shapes to the device without sending any that
    measured slower there."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import Device, gemm_desc
    dev = Device.shared(0)
    rng = np.random.default_rng(11)
    rows = []

    def timed(fn, budget_s):
        fn()
        ts = []
        t_end = time.perf_counter() + budget_s
        while len(ts) < 5 or (time.perf_counter() < t_end and len(ts) < 200):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)

    for m, k, n in THRESHOLD_SHAPES:
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        c = np.empty((m, n), np.float32)
        desc = gemm_desc(m, n, k, F.F32, F.F32, F.B_KN)

        def device_call():
            da, db, dc = dev.alloc(a.nbytes), dev.alloc(b.nbytes), dev.alloc(c.nbytes)
            dev.copy_h2d(da.ptr, a)
            dev.copy_h2d(db.ptr, b)
            dev.gemm(desc, da.ptr, db.ptr, dc.ptr)
            dev.copy_d2h_into(c, dc.ptr)
            dev.stream_sync()
            for x in (da, db, dc):
                x.free()

        t_dev = timed(device_call, 0.2)
        t_cpu = timed(lambda: O.matmul(a, b, threads=1), 0.5)
        rows.append({"m": m, "k": k, "n": n, "device_us": t_dev * 1e6, "cpu_us": t_cpu * 1e6,
                     "speedup": t_cpu / t_dev})
    cands_e = sorted({r["m"] * r["n"] for r in rows})
    cands_w = [0] + sorted({r["m"] * r["n"] * r["k"] for r in rows})
    rule, best = None, None
    for e in cands_e:
        for wk in cands_w:
            sent = [r for r in rows if r["m"] * r["n"] >= e and r["m"] * r["n"] * r["k"] >= wk]
            if all(r["speedup"] >= 1.0 for r in sent) and (best is None or len(sent) > best):
                best = len(sent)
                rule = {"element_threshold": e, "work_threshold": wk, "shapes_sent_to_device": len(sent),
                        "shapes_faster_on_device": sum(r["speedup"] >= 1.0 for r in rows), "shapes": len(rows)}
    emit({"metric": "host-array f32 GEMM end to end: device vs one CPU thread", "unit": "us",
          "cpu": "oracle restatement of tensor-core gemmNT, 1 thread", "rows": rows, "rule": rule})


def reference_line(args, w, name, threads, budget_s=150.0):
    rates, sample, secs = [], "", []
    unit, scale = unit_of(w)
    per = max(1.0, min(args.cpu_seconds, budget_s / max(1, args.warmup + args.steps)))
    for i in range(args.warmup + args.steps):
        r, sample, s = cpu_sample_rate(w, per, threads)
        if i >= args.warmup:
            rates.append(r)
            secs.append(s)
    v = statistics.median(rates) / scale
    return {
        "impl": "reference", "metric": w["metric"], "value": v, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": flop_per_step(w) / (v * scale) * 1e3,
        "ms_per_step_basis": (f"extrapolated: one step's work / the median rate of the {args.steps} timed samples "
                              f"(each about {statistics.median(secs):.1f} s of CPU work on a part of the step)"),
        "higher_is_better": True, "scaling": "strong" if w["kind"] == "nsplit" else "weak", "vs_baseline": None,
        "dtype": "f32" if w.get("precision") == "f32" else "f64 (f32 storage)",
        "data": "synthetic", "config": {"workload": name, "description": w["desc"]},
        "cpu_baseline": {"value": v, "unit": unit, "cores": 1 if w["kind"] == "fusion" else threads, "kind": "port",
                         "sample": "per step: " + sample + ("" if w["kind"] == "fusion" else
                                   "; the oracle's restatement of tensor-core gemmNT / attention, OpenMP over "
                                   "row blocks / heads")},
        "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def run_reference(args, w):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    names = SECONDARY.get(args.workload, []) if not args.no_secondary and args.batch is None else []
    budget = 150.0 / (1 + len(names))  # the whole arm stays within a few minutes
    line = reference_line(args, w, args.workload, threads, budget)
    if names:
        line["secondary"] = [reference_line(args, dict(WORKLOADS[n]), n, threads, budget) for n in names]
    emit(line)


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------

def setup_gemm(w, dev, torch, g, local, F):
    from tensor_cuda.runtime import gemm_desc
    B_, M, N, K = w["batch"], w["m"], w["n"], w["k"]
    dt_in, dt_out = F.DTYPE_CODES[w["dtype"]], F.DTYPE_CODES[w["out"]]
    epi = F.EPI_BIAS | F.EPI_GELU if w["epilogue"] == "bias+gelu" else 0
    dvc = f"cuda:{local}"
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[w["dtype"]]
    if w["dtype"] == "f32":
        A = (torch.rand((B_, M, K), generator=g, device=dvc) * 2 - 1).to(tdt)
        Bm = (torch.rand((B_, K, N), generator=g, device=dvc) * 2 - 1).to(tdt)
    else:
        A = (torch.randn((B_, M, K), generator=g, device=dvc) / K ** 0.5).to(tdt)
        Bm = (torch.randn((B_, K, N), generator=g, device=dvc) / K ** 0.5).to(tdt)
    bias = (torch.randn((N,), generator=g, device=dvc) * 0.02).float()
    out = dev.alloc(B_ * M * N * F.DTYPE_BYTES[dt_out])
    desc = gemm_desc(M, N, K, dt_in, dt_out, F.B_KN, epi, 1.0, (B_,), (M * K,), (K * N,))
    ins = [A, Bm, bias] if epi else [A, Bm]

    def launch(ptrs, optr, stream):
        dev.gemm(desc, ptrs[0], ptrs[1], optr, ptrs[2] if epi else None, stream)

    kernel = ("gemm_kernel<kHalf, B MN-major, 256 x 256 tiles on CTA pairs (cta_group::2), 6 stages, 10 warps>"
              if w["dtype"] != "f32"
              else "gemm_kernel<kTF32x3, BN=128, 3 stages>, K split in two halves (+ one split_prologue_kernel launch: A / B hi-lo planes and the zeroing of C; the GEMM launched programmatically after it)")
    return ins, out, launch, kernel


def setup_attention(w, dev, torch, g, local, F):
    from tensor_cuda.runtime import sdpa_desc
    B_, H, L, D = w["batch"], w["heads"], w["seq"], w["head_dim"]
    dvc = f"cuda:{local}"
    tdt = torch.bfloat16 if w["dtype"] == "bf16" else torch.float16
    q, k, v = (torch.randn((B_, H, L, D), generator=g, device=dvc).to(tdt) for _ in range(3))
    out = dev.alloc(B_ * H * L * D * 2)
    lse = dev.alloc(B_ * H * L * 4)
    desc = sdpa_desc(B_, H, H, L, L, D, D, F.DTYPE_CODES[w["dtype"]], w["causal"], 1 / math.sqrt(D))

    def launch(ptrs, optr, stream):
        dev.sdpa(desc, ptrs[0], ptrs[1], ptrs[2], None, optr, lse.ptr, stream)

    return [q, k, v], out, launch, (f"attn_kernel<D={D}, {w['dtype']}> (persistent: one CTA per SM, 2 Q tiles x 128 "
                                    "rows per unit, 12 warps)")


def setup_nsplit(w, dev, torch, g, local, F, world, pg):
    from tensor_cuda import plan as P
    from tensor_cuda.parallel import ColumnSplitGemm, PeerGroup, unique_id
    from tensor_cuda.runtime import gemm_desc
    pl = P.column_split_plan(w["m"], w["n"], w["k"], world, w["out"])
    M, n, K = w["m"], pl.n_shard, w["k"]
    dvc = f"cuda:{local}"
    A = (torch.randn((M, K), generator=g, device=dvc) / K ** 0.5).to(torch.bfloat16)
    Bs = (torch.randn((K, n), generator=g, device=dvc) / K ** 0.5).to(torch.bfloat16)  # this rank's columns
    group = PeerGroup.from_torch(dev) if world > 1 else PeerGroup(dev, 0, 1, unique_id())
    fused = ColumnSplitGemm(group, M, n, K, "bf16", w["out"], F.B_KN, fused=True)

    class Out:  # this rank's whole row-major C
        ptr = fused.out_ptr
        nbytes = M * w["n"] * F.DTYPE_BYTES[F.DTYPE_CODES[w["out"]]]

    def launch(ptrs, optr, stream):
        fused(ptrs[0], ptrs[1], stream)

    extras = {"group": group, "fused": fused, "pl": pl,
              "gemm_desc": gemm_desc(M, n, K, F.BF16, F.DTYPE_CODES[w["out"]], F.B_KN)}
    return [A, Bs], Out, launch, "gemm_kernel<kHalf, B MN-major, BN=256, 4 stages, 8 output maps>", extras


def setup_fusion(w, dev, torch, g, local, F):
    from tensor_cuda.fusion import kernel_for
    n = w["n"]
    ins = [torch.randn((n,), generator=g, device=f"cuda:{local}") for _ in range(3)]
    out = dev.alloc(4 * n)
    k = kernel_for(dev, fusion_expr(w).node, ["f32"] * 3, w.get("precision", "f64"))

    def launch(ptrs, optr, stream):
        k.run(ptrs, [(n,)] * 3, (n,), optr, stream)

    return ins, out, launch, (f"mpc_fused_flat (NVRTC-compiled for sm_100a: 16-byte loads, "
                              f"{w.get('precision', 'f64')} evaluation)")


def setup_gpt2(w, dev, torch, g, local, F, rank):
    import numpy as np

    from tensor_cuda.backend import CudaBackend
    from tensor_cuda.gpt2 import GPT2, GPT2Config, random_weights
    cfg = GPT2Config()
    be = CudaBackend(dev)
    model = GPT2(be, cfg, random_weights(cfg, seed=1234))  # replicated weights
    B, L = w["batch"], w["seq"]
    ids = torch.randint(0, cfg.vocab, (B, L), generator=g, device=f"cuda:{local}", dtype=torch.int32)
    state = {}

    class Out:  # the last step's logits
        nbytes = B * L * cfg.vocab * 2

        @property
        def ptr(self):
            t = state.get("logits")
            return t.ptr if t is not None else 0

    def launch(ptrs, optr, stream):
        if "logits" in state:
            be.dispose(state.pop("logits"))
        state["logits"] = model.forward(be.external(ptrs[0], (B, L), "i32"))
        _ = state["logits"].ptr  # run the pending LM-head GEMM

    return [ids], Out(), launch, "whole forward: 12 x (LN, QKV GEMM, head split, causal attention, head merge, " \
        "out-proj GEMM, residual add, LN, fc GEMM + GELU, proj GEMM, residual add), LN, LM-head GEMM"


def time_region(dev, stream, fn, steps, barrier):
    barrier()
    dev.stream_sync(stream)
    e0, e1 = dev.event(), dev.event()
    dev.record(e0, stream)
    for _ in range(steps):
        fn()
    dev.record(e1, stream)
    dev.stream_sync(stream)
    barrier()
    return dev.elapsed_ms(e0, e1) / steps


def host_link_floor_ms(h2d_bytes, d2h_bytes, bw):
    """Least time per step for the streamed e2e leg's copies: a step's uploads and the previous
    step's read-back run at once at the rates measured for both directions together until the
    smaller transfer is done; the rest of the larger one then moves at its rate alone."""
    th = h2d_bytes / (bw["bidir_h2d_gbs"] * 1e9)
    td = d2h_bytes / (bw["bidir_d2h_gbs"] * 1e9)
    if th <= td:
        rest = d2h_bytes - th * bw["bidir_d2h_gbs"] * 1e9
        return (th + rest / (bw["d2h_gbs"] * 1e9)) * 1e3
    rest = h2d_bytes - td * bw["bidir_h2d_gbs"] * 1e9
    return (td + rest / (bw["h2d_gbs"] * 1e9)) * 1e3


def pinned_copy_gbs(dev, nbytes=256 << 20, reps=5):
    """Host<->device copy bandwidth from pinned memory (GB/s), CUDA events: each direction alone, and
    both at once on two streams (the end-to-end leg overlaps them): the roofline of its transfers."""
    import numpy as np
    h, hp = dev.pinned_array((nbytes,), np.uint8)
    h2, hp2 = dev.pinned_array((nbytes,), np.uint8)
    d, d2 = dev.alloc(nbytes), dev.alloc(nbytes)
    s2 = dev.new_stream()
    up = lambda s: dev.copy_h2d(d.ptr, h, s)
    down = lambda s: dev.copy_d2h_into(h2, d2.ptr, s)

    def timed(fns):
        for fn, s in fns:
            fn(s)
        evs = []
        for fn, s in fns:
            e0, e1 = dev.event(), dev.event()
            dev.record(e0, s)
            for _ in range(reps):
                fn(s)
            dev.record(e1, s)
            evs.append((e0, e1, s))
        for _, _, s in evs:
            dev.stream_sync(s)
        return [nbytes * reps / (dev.elapsed_ms(e0, e1) * 1e-3) / 1e9 for e0, e1, _ in evs]

    out = {"h2d_gbs": timed([(up, dev.stream)])[0], "d2h_gbs": timed([(down, dev.stream)])[0]}
    out["bidir_h2d_gbs"], out["bidir_d2h_gbs"] = timed([(up, dev.stream), (down, s2)])
    dev.destroy_stream(s2)
    d.free()
    d2.free()
    dev.host_free(hp)
    dev.host_free(hp2)
    return out


def measure_workload(args, w, name, ctx):
    """Times one workload on this rank: device value, end to end, roofline and CPU samples.
    Returns its JSON line's fields on rank 0, None on the other ranks."""
    import numpy as np
    import torch

    from tensor_cuda import _ffi as F
    dev, stream, pg, world, rank, local, barrier, bus = (ctx[k] for k in ("dev", "stream", "pg", "world", "rank",
                                                                         "local", "barrier", "bus"))
    g = torch.Generator(device=f"cuda:{local}")
    g.manual_seed(1234 + rank)
    extras = {}
    if w["kind"] == "nsplit":
        g.manual_seed(1234)  # A is the same on every rank
        ins, out, launch, kernel_name, extras = setup_nsplit(w, dev, torch, g, local, F, world, pg)
    elif w["kind"] == "gpt2":
        ins, out, launch, kernel_name = setup_gpt2(w, dev, torch, g, local, F, rank)
    elif w["kind"] == "fusion":
        ins, out, launch, kernel_name = setup_fusion(w, dev, torch, g, local, F)
    else:
        setup = setup_gemm if w["kind"] == "gemm" else setup_attention
        ins, out, launch, kernel_name = setup(w, dev, torch, g, local, F)
    strong = w["kind"] == "nsplit"
    torch.cuda.synchronize()
    ptrs = [t.data_ptr() for t in ins]
    flop_step = flop_per_step(w)
    in_bytes = sum(t.numel() * t.element_size() for t in ins)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}") if in_bytes < (200 << 20) else None

    def step():
        launch(ptrs, out.ptr, stream)

    for _ in range(args.warmup):
        step()
    dev.stream_sync(stream)

    sampler = ClockSampler(bus)
    sampler.start()
    time.sleep(0.3)
    launches0 = dev.launch_count()
    barrier()
    dev.stream_sync(stream)
    torch.cuda.synchronize()
    if flush is None:
        e0, e1 = dev.event(), dev.event()
        dev.record(e0, stream)
        for _ in range(args.steps):
            step()
        dev.record(e1, stream)
        dev.stream_sync(stream)
        ms_total = dev.elapsed_ms(e0, e1)
    else:  # L2-resident inputs: a 256 MiB write flushes L2 before each timed launch
        ev = [(dev.event(), dev.event()) for _ in range(args.steps)]
        s_torch = torch.cuda.ExternalStream(stream)
        for a, b_ in ev:
            with torch.cuda.stream(s_torch):
                flush.zero_()
            dev.record(a, stream)
            step()
            dev.record(b_, stream)
        dev.stream_sync(stream)
        ms_total = sum(dev.elapsed_ms(a, b_) for a, b_ in ev)
    barrier()
    launches = dev.launch_count() - launches0
    clocks = sampler.stop()
    def max_over_ranks(x):
        if not pg:
            return x
        t = torch.tensor([x], device=f"cuda:{local}", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        return float(t.item())

    ms_total = max_over_ranks(ms_total)
    ms_step = ms_total / args.steps
    unit, scale = unit_of(w)
    job_flop = flop_step if strong else flop_step * world
    value = job_flop / (ms_step * 1e-3) / scale

    breakdown = None
    if strong:  # the same step as GEMM alone and as GEMM + NCCL all-gather + permute
        from tensor_cuda.parallel import ColumnSplitGemm
        local_c = dev.alloc(extras["pl"].n_shard * w["m"] * F.DTYPE_BYTES[F.DTYPE_CODES[w["out"]]])
        gd = extras["gemm_desc"]
        gemm_only = lambda: dev.gemm(gd, ptrs[0], ptrs[1], local_c.ptr, None, stream)
        nccl = ColumnSplitGemm(extras["group"], w["m"], extras["pl"].n_shard, w["k"], "bf16", w["out"], F.B_KN,
                               fused=False)
        nccl_step = lambda: nccl(ptrs[0], ptrs[1], stream)
        blocks = ColumnSplitGemm(extras["group"], w["m"], extras["pl"].n_shard, w["k"], "bf16", w["out"], F.B_KN,
                                 fused=True, layout="blocks")
        blocks_step = lambda: blocks(ptrs[0], ptrs[1], stream)
        for fn in (gemm_only, nccl_step, blocks_step):
            for _ in range(max(1, args.warmup)):
                fn()
        breakdown = {"fused_gemm_allgather": ms_step,
                     "fused_gemm_allgather_blocked_layout": max_over_ranks(
                         time_region(dev, stream, blocks_step, args.steps, barrier)),
                     "gemm_only": max_over_ranks(time_region(dev, stream, gemm_only, args.steps, barrier)),
                     "gemm_then_nccl_allgather_then_permute": max_over_ranks(
                         time_region(dev, stream, nccl_step, args.steps, barrier))}
        blocks.destroy()
        nccl.destroy()
        local_c.free()

    # ---- e2e: through the C ABI from pinned host buffers, copies inside the timed region ----
    # Every step copies its inputs host -> device, runs the same step and copies its result device ->
    # host. Streaming order: uploads on one stream, the step on the device's stream, the read-back on
    # a third, device buffers double-buffered, so the uploads of step i + 1 and the read-back of step i
    # run at once on the two copy engines while step i + 1 waits only for its own uploads. The region
    # starts before the first upload and ends when the last read-back has landed in host memory.
    e2e = None
    if args.e2e_steps > 0:
        hins = []
        for t in ins:
            raw = t.contiguous().view(torch.uint8).reshape(-1)
            h, hp = dev.pinned_array((raw.numel(),), np.uint8)
            h[:] = raw.cpu().numpy()
            hins.append((h, hp, [dev.alloc(h.nbytes), dev.alloc(h.nbytes)]))
        hout, hop = dev.pinned_array((out.nbytes,), np.uint8)
        single_out = w["kind"] in ("nsplit", "gpt2")  # their output buffer is owned by the step itself
        outs = [out, out] if single_out else [out, dev.alloc(out.nbytes)]
        s_in, s_out = dev.new_stream(), dev.new_stream()
        done_up = [dev.event(), dev.event()]
        done_step = [dev.event(), dev.event()]
        done_read = [dev.event(), dev.event()]
        step_no = [0]

        def e2e_step():
            k = step_no[0] & 1
            # the uploads overwrite input buffers that the step two back read (an event never
            # recorded counts as complete)
            dev.wait_event(s_in, done_step[k])
            for h, _, dbuf in hins:
                dev.copy_h2d(dbuf[k].ptr, h, s_in)
            dev.record(done_up[k], s_in)
            dev.wait_event(stream, done_up[k])
            # the step overwrites an output buffer whose earlier read-back must have finished
            dev.wait_event(stream, done_read[k ^ 1] if single_out else done_read[k])
            launch([dbuf[k].ptr for _, _, dbuf in hins], outs[k].ptr, stream)
            dev.record(done_step[k], stream)
            dev.wait_event(s_out, done_step[k])
            dev.copy_d2h_into(hout, outs[k].ptr, s_out)
            dev.record(done_read[k], s_out)
            step_no[0] += 1

        for _ in range(2):
            e2e_step()
        for s_ in (s_in, stream, s_out):
            dev.stream_sync(s_)
        barrier()
        x0, x1 = dev.event(), dev.event()
        dev.record(x0, s_in)
        for _ in range(args.e2e_steps):
            e2e_step()
        dev.wait_event(s_out, done_step[(step_no[0] - 1) & 1])
        dev.record(x1, s_out)
        for s_ in (s_in, stream, s_out):
            dev.stream_sync(s_)
        barrier()
        ms_e2e = max_over_ranks(dev.elapsed_ms(x0, x1))
        e2e = {"value": job_flop / (ms_e2e / args.e2e_steps * 1e-3) / scale, "unit": unit,
               "h2d_bytes_per_step": int(sum(h.nbytes for h, _, _ in hins)), "d2h_bytes_per_step": int(hout.nbytes),
               "ms_per_step": ms_e2e / args.e2e_steps,
               "path": "per step: mpc_memcpy_h2d_async of every input -> the step -> mpc_memcpy_d2h_async of the "
                       "result into pinned host memory; uploads, steps and read-backs on three streams, so the "
                       "uploads of step i + 1 overlap the read-back of step i (double-buffered device buffers)"}
        for _, hp, dbuf in hins:
            dev.host_free(hp)
            for d in dbuf:
                d.free()
        dev.host_free(hop)
        if not single_out:
            outs[1].free()
        dev.destroy_stream(s_out)
        dev.destroy_stream(s_in)
        if rank == 0:
            # the host link's roofline: a step cannot end before its uploads have crossed (the
            # read-back of the previous step overlaps them on the other copy engine)
            bw = pinned_copy_gbs(dev)
            h2d_b, d2h_b = e2e["h2d_bytes_per_step"], e2e["d2h_bytes_per_step"]
            floor_ms = host_link_floor_ms(h2d_b, d2h_b, bw)
            e2e["host_link"] = dict(bw, source="measured: 256 MiB pinned copies, CUDA events, this box; the floor "
                                               "moves both directions at their concurrent rates until the smaller "
                                               "is done, then the rest of the larger at its rate alone",
                                    floor_ms_per_step=floor_ms, frac_of_floor=floor_ms / e2e["ms_per_step"])

    if extras:
        extras["fused"].destroy()
        extras["group"].destroy()
    if rank != 0:
        return None
    peaks = load_peaks()
    long_region = ms_total > 2000
    peak = peaks["bf16_tflops_sustained"] if long_region else peaks["bf16_tflops"]
    rank_flop = flop_step / world if strong else flop_step
    achieved = rank_flop / (ms_step * 1e-3) / scale  # one launch of the kernel per step and rank
    if w["kind"] == "fusion":
        roof = {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"], "peak_source": f"{peaks['source']} HBM copy",
                "traffic": profiled_traffic(name), "algorithmic_bytes_per_launch": rank_flop,
                "kernel": kernel_name}
    else:
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_source": f"{peaks['source']} bf16 dense ({'sustained' if long_region else 'burst'})",
                "traffic": profiled_traffic(name), "algorithmic_flop_per_launch": rank_flop,
                "kernel": kernel_name}
    if strong and world > 1:
        # fused GEMM + all-gather: the slower of the tensor-core time and the NVLink time of the
        # bytes every GPU must receive ((p-1)/p of C), at the measured 770 GB/s per direction
        c_bytes = out.nbytes
        nv_bytes = c_bytes * (world - 1) / world
        target_ms = max(rank_flop / (peak * 1e12), nv_bytes / 770e9) * 1e3
        roof["nvlink"] = {"bytes_in_per_gpu": nv_bytes, "achieved_gbs": nv_bytes / (ms_step * 1e-3) / 1e9,
                          "peak_gbs": 770.0, "peak_source": "measured peer copy per direction",
                          "target_ms": target_ms, "frac_of_target": target_ms / ms_step}
    if w["kind"] == "gemm" and w.get("dtype") == "f32":
        # 3xTF32 issues three tf32 products per f32 product; tf32 runs at half the bf16 rate
        tf32_roof = peak / 2 / 3
        roof["note"] = "3xTF32 issues 3 tf32 MMAs per product; tf32 dense peak is half of bf16"
        roof["tf32x3_roofline"] = {"peak": tf32_roof, "frac": achieved / tf32_roof,
                                   "source": "the bf16 peak / 2 (tf32 rate) / 3 (tf32 products per f32 product)"}
    if w["kind"] == "attention" and w["causal"]:
        roof["note"] = "FLOP = causal half of 4*B*H*L^2*D (masked tiles are skipped)"
    cpu = cpu1 = None
    if not args.no_cpu_baseline and world == 1:
        threads = len(os.sched_getaffinity(0))
        for label, nthreads, secs_target in (("all host threads", threads, args.cpu_seconds),
                                             ("restatement, 1 thread", 1, args.cpu_seconds / 2)):
            try:
                rt, sample, secs = cpu_sample_rate(w, secs_target, nthreads)
                rec = {"value": rt / scale, "unit": unit, "cores": 1 if w["kind"] == "fusion" else nthreads,
                       "kind": "port", "label": label,
                       "sample": sample + f" ({secs:.1f} s); the oracle's restatement of the reference's CPU path"}
            except Exception as ex:  # reported, never required
                rec = {"value": None, "unit": unit, "cores": None, "kind": "port", "label": label,
                       "sample": f"failed: {ex}"}
            if nthreads == threads:
                cpu = rec
            else:
                cpu1 = rec
    par = (f"column split over {world} GPUs, all-gather fused into the GEMM epilogue (peer stores into the "
           "shard-major view), then a local permute to row-major" if strong
           else f"dp{world} (shards, no collective)")
    cfg = {"workload": name, "description": w["desc"], "parallelism": par}
    if breakdown:
        cfg["breakdown_ms_per_step"] = breakdown
    cfg.update({k: w[k] for k in ("batch", "m", "n", "k", "heads", "seq", "head_dim", "out") if k in w})
    if w["kind"] == "fusion":
        cfg["expression"] = EXPRESSIONS[w.get("expression", "sigmoid_chain")][0]
        cfg["precision"] = w.get("precision", "f64")
    cfg["l2"] = "flushed between steps (256 MiB write)" if flush is not None else "inputs larger than L2 (126 MB)"
    line = {
        "metric": w["metric"], "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": w["dtype"],
        "data": "synthetic (seeded torch RNG on device; configuration shapes and distributions)",
        "config": cfg, "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
        "clocks": clocks,
    }
    if cpu1 is not None:
        line["cpu_baseline_1thread"] = cpu1
    return line


# The default run also measures the fused-attention configuration, so the metric's second half
# (fused-attention TFLOP/s) is in the same line.
SECONDARY = {"batched_gemm_bf16": ["causal_attention_f16"]}


def run_ours(args, w):
    import torch

    from tensor_cuda.runtime import Device

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        pg = dist

    def barrier():
        if pg:
            pg.barrier()

    dev = Device.shared(local)
    bus = None
    try:
        p = torch.cuda.get_device_properties(local)
        bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        pass
    ctx = {"dev": dev, "stream": dev.stream, "pg": pg, "world": world, "rank": rank, "local": local,
           "barrier": barrier, "bus": bus}
    line = measure_workload(args, w, args.workload, ctx)
    extra = []
    if not args.no_secondary and args.batch is None:
        for sub_name in SECONDARY.get(args.workload, []):
            sub = measure_workload(args, dict(WORKLOADS[sub_name]), sub_name, ctx)
            if sub is not None:
                extra.append(sub)
    if rank == 0:
        if extra:
            line["secondary"] = extra
        emit(line)
    if pg:
        pg.destroy_process_group()


_RESULT = None  # the stream the JSON line goes to (the process's original stdout)


def emit(line: dict) -> None:
    out = _RESULT or sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    global _RESULT
    # Libraries print to stdout on their own (NCCL's version banner, for one): send file
    # descriptor 1 to stderr for the whole run and keep the original stdout for the one JSON line.
    sys.stdout.flush()
    _RESULT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse_args()
    if args.threshold_sweep:
        run_threshold_sweep(args)
        return
    w = dict(WORKLOADS[args.workload])
    if args.batch is not None:
        w["batch"] = args.batch
    if w["kind"] == "fusion":
        if args.elements is not None:
            w["n"] = args.elements
        w["expression"], w["precision"] = args.expression, args.precision
        if (args.expression, args.precision) != ("sigmoid_chain", "f64"):
            text = EXPRESSIONS[args.expression][0]
            w["metric"] = f"fused element-wise GB/s ({text}, f32, {args.precision} evaluation)"
            w["desc"] = (f"one fused kernel over three f32 inputs of {w['n']} elements: {text}, "
                         f"{args.precision} evaluation, f32 out (16 bytes per element)")
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
