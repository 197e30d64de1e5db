#!/usr/bin/env python3
"""Benchmark of the math-plus CUDA backend's GEMM / fused-attention path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

For N > 1 launch one rank per GPU with torch.distributed.run; every rank runs its own shard
(weak scaling: independent batches, no data-path collective) and rank 0 prints ONE JSON line.

A step is one pass of the hot path over one batch of synthetic input:

  batched_gemm_bf16 (default)  64 x [2048x2048]·[2048x2048] bf16 -> f32, fused +bias[2048] and
                               exact-erf GELU: Backend.matmul -> add -> gelu of math-plus
                               (packages/tensor-cpu/src/index.ts:755-762, :598), one kernel.
  gemm_f32_1024                one f32 1024^3 GEMM (3xTF32 on the tensor cores).

``value`` is device-timed throughput with inputs resident in HBM (CUDA events on the launching
stream, barrier + synchronize around the timed region, max over ranks). ``e2e`` runs the same
step through the C ABI with pinned HOST buffers: the host->device copies of A, B and bias and the
device->host read of C are inside its timed region. ``--impl reference`` times the reference's
CPU algorithm (the oracle's restatement of tensor-core's gemmNT, kernels.ts:299-362, with the
bias add and exact GELU) on a bounded sample of the same workload with all host threads.
Inputs are seeded synthetic data with the configuration's shapes and distributions.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "math-plus_b200"))

WORKLOADS = {
    "batched_gemm_bf16": dict(batch=64, m=2048, n=2048, k=2048, dtype="bf16", out="f32", epilogue="bias+gelu",
                              desc="batched GEMM bf16 in / f32 accumulate+out, 64x2048^3, +bias[2048], exact GELU"),
    "gemm_f32_1024": dict(batch=1, m=1024, n=1024, k=1024, dtype="f32", out="f32", epilogue="none",
                          desc="single f32 GEMM 1024^3 (3xTF32 on tcgen05)"),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="batched_gemm_bf16", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU work for the baseline sample")
    ap.add_argument("--batch", type=int, default=None, help="override the per-rank batch (small profiling cases)")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def profiled_traffic(kernel_key: str):
    """DRAM bytes per launch from the committed ncu summary (profiles/*.txt 'traffic_bytes_per_launch')."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for fn in sorted(os.listdir(pdir)):
        if kernel_key in fn and fn.endswith(".txt"):
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

    def __init__(self, bus_id: str | None):
        self.bus_id = bus_id
        self.proc = None
        self.lines: list[str] = []
        self.t = None

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

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

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


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------------------------
# reference arm: the reference's CPU algorithm (oracle restatement), all host threads
# ---------------------------------------------------------------------------------------------

def cpu_sample_rate(w: dict, target_s: float, threads: int):
    """Times the oracle (tensor-core gemmNT restatement + bias add + exact GELU, f32 out) on a
    sample of rows of one batch, sized to about target_s seconds. Returns (flop/s, sample text)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    m, n, k = w["m"], w["n"], w["k"]
    rng = np.random.default_rng(7)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    bias = (rng.standard_normal(n) * 0.02).astype(np.float32)

    def run(rows):
        a = (rng.standard_normal((rows, k)) / np.sqrt(k)).astype(np.float32)
        t0 = time.perf_counter()
        c = O.matmul(a, b, threads=threads)
        if w["epilogue"] == "bias+gelu":
            c = O.gelu(O.add_f32(c, bias))
        return time.perf_counter() - t0

    rows = 16
    dt = run(rows)
    while dt < 0.5 and rows < m:
        rows = min(m, rows * 4)
        dt = run(rows)
    rate_rows = rows / dt
    want_rows = max(16, int(rate_rows * target_s))
    rows = min(m, want_rows)
    reps = max(1, min(w["batch"], want_rows // m)) if want_rows > m else 1
    t = 0.0
    for _ in range(reps):
        t += run(rows)
    flop = 2.0 * reps * rows * n * k
    what = (f"{reps} of the {w['batch']} products ({m}x{k} @ {k}x{n}, +bias, GELU)" if rows == m else
            f"{rows} of the {m} rows of one {m}x{k} @ {k}x{n} product (+bias, GELU)")
    return flop / t, what + ", f64 accumulate", t


def run_reference(args, w):
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    rates, sample = [], ""
    for i in range(args.warmup + args.steps):
        tgt = max(1.0, min(args.cpu_seconds, 120.0 / max(1, args.warmup + args.steps)))
        r, sample, _ = cpu_sample_rate(w, tgt, threads)
        if i >= args.warmup:
            rates.append(r)
    v = statistics.median(rates) / 1e12
    flop_step = 2.0 * w["batch"] * w["m"] * w["n"] * w["k"]
    line = {
        "impl": "reference", "metric": "GEMM TFLOP/s", "value": v, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": flop_step / (v * 1e12) * 1e3 * args.gpus,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": args.workload, "description": w["desc"], "batch_per_rank": w["batch"]},
        "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": "per step: " + sample + "; oracle restatement of tensor-core gemmNT "
                                   "(packages/tensor-core/src/kernels.ts:299-362), OpenMP over row blocks"},
        "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------

def run_ours(args, w):
    import ctypes as C

    import numpy as np
    import torch

    from tensor_cuda import _ffi as F
    from tensor_cuda.runtime import Device, gemm_desc

    world, rank, local = dist_setup(args)
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
    stream = dev.stream
    B_, M, N, K = w["batch"], w["m"], w["n"], w["k"]
    dt_in = F.DTYPE_CODES[w["dtype"]]
    dt_out = F.DTYPE_CODES[w["out"]]
    epi = F.EPI_BIAS | F.EPI_GELU if w["epilogue"] == "bias+gelu" else 0

    # Seeded synthetic inputs (the configuration's distributions) generated on the device.
    g = torch.Generator(device=f"cuda:{local}")
    g.manual_seed(1234 + rank)
    tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[w["dtype"]]
    if w["dtype"] == "f32":
        A = (torch.rand((B_, M, K), generator=g, device=f"cuda:{local}") * 2 - 1).to(tdt)
        Bm = (torch.rand((B_, K, N), generator=g, device=f"cuda:{local}") * 2 - 1).to(tdt)
    else:
        A = (torch.randn((B_, M, K), generator=g, device=f"cuda:{local}") / K ** 0.5).to(tdt)
        Bm = (torch.randn((B_, K, N), generator=g, device=f"cuda:{local}") / K ** 0.5).to(tdt)
    bias = (torch.randn((N,), generator=g, device=f"cuda:{local}") * 0.02).float()
    torch.cuda.synchronize()
    out_bytes = B_ * M * N * F.DTYPE_BYTES[dt_out]
    Cbuf = dev.alloc(out_bytes)
    desc = gemm_desc(M, N, K, dt_in, dt_out, F.B_KN, epi, 1.0, (B_,), (M * K,), (K * N,))
    flop_step = 2.0 * B_ * M * N * K

    def step():
        dev.gemm(desc, A.data_ptr(), Bm.data_ptr(), Cbuf.ptr, bias.data_ptr() if epi else None, stream)

    for _ in range(args.warmup):
        step()
    dev.stream_sync(stream)

    bus = None
    try:
        p = torch.cuda.get_device_properties(local)
        bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
    except Exception:
        pass
    sampler = ClockSampler(bus)
    sampler.start()
    time.sleep(0.3)
    launches0 = dev.launch_count()
    e0, e1 = dev.event(), dev.event()
    barrier()
    dev.stream_sync(stream)
    torch.cuda.synchronize()
    dev.record(e0, stream)
    for _ in range(args.steps):
        step()
    dev.record(e1, stream)
    dev.stream_sync(stream)
    barrier()
    ms_total = dev.elapsed_ms(e0, e1)
    launches = dev.launch_count() - launches0
    clocks = sampler.stop()

    if pg:
        t = torch.tensor([ms_total], device=f"cuda:{local}", dtype=torch.float64)
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms_total = float(t.item())
    ms_step = ms_total / args.steps
    value = flop_step * world / (ms_step * 1e-3) / 1e12

    # ---- e2e: through the C ABI with pinned host buffers, copies inside the timed region ----
    e2e = None
    if args.e2e_steps > 0:
        es_in = F.DTYPE_BYTES[dt_in]
        hA, pA = dev.pinned_array((B_ * M * K * es_in,), np.uint8)
        hB, pB = dev.pinned_array((B_ * K * N * es_in,), np.uint8)
        hbias, pbias = dev.pinned_array((N,), np.float32)
        hC, pC = dev.pinned_array((out_bytes,), np.uint8)
        # host copies of the same synthetic inputs
        hA[:] = A.view(torch.uint8).reshape(-1).cpu().numpy()
        hB[:] = Bm.view(torch.uint8).reshape(-1).cpu().numpy()
        hbias[:] = bias.cpu().numpy()
        dA, dB, dbias = dev.alloc(hA.nbytes), dev.alloc(hB.nbytes), dev.alloc(hbias.nbytes)

        def e2e_step():
            dev.copy_h2d(dA.ptr, hA, stream)
            dev.copy_h2d(dB.ptr, hB, stream)
            dev.copy_h2d(dbias.ptr, hbias, stream)
            dev.gemm(desc, dA.ptr, dB.ptr, Cbuf.ptr, dbias.ptr if epi else None, stream)
            dev.copy_d2h_into(hC, Cbuf.ptr, stream)

        e2e_step()
        dev.stream_sync(stream)
        barrier()
        x0, x1 = dev.event(), dev.event()
        dev.record(x0, stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        dev.record(x1, stream)
        dev.stream_sync(stream)
        barrier()
        ms_e2e = dev.elapsed_ms(x0, x1)
        if pg:
            t = torch.tensor([ms_e2e], device=f"cuda:{local}", dtype=torch.float64)
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            ms_e2e = float(t.item())
        e2e = {"value": flop_step * world / (ms_e2e / args.e2e_steps * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": int(hA.nbytes + hB.nbytes + hbias.nbytes), "d2h_bytes_per_step": int(hC.nbytes),
               "ms_per_step": ms_e2e / args.e2e_steps, "path": "mpc_memcpy_h2d_async x3 -> mpc_gemm -> "
                                                              "mpc_memcpy_d2h_async, pinned host buffers"}
        for p_ in (pA, pB, pbias, pC):
            dev.host_free(p_)

    if rank != 0:
        if pg:
            pg.destroy_process_group()
        return

    peaks = load_peaks()
    long_region = ms_total > 2000
    peak = peaks["bf16_tflops_sustained"] if long_region else peaks["bf16_tflops"]
    kernel_ms = ms_step / max(1, launches / args.steps) if launches >= args.steps else ms_step
    achieved = flop_step / (ms_step * 1e-3) / 1e12  # one GEMM launch per step: per-launch = per-step
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "peak_source": f"{peaks['source']} bf16 dense ({'sustained' if long_region else 'burst'})",
            "traffic": profiled_traffic(args.workload), "algorithmic_flop_per_launch": flop_step,
            "kernel": "gemm_kernel<kHalf, B MN-major, BN=256, 4 stages>" if w["dtype"] != "f32"
            else "gemm_kernel<kTF32x3, BN=128, 3 stages> (+ split prologue)"}
    if w["dtype"] == "f32":
        roof["note"] = "3xTF32 issues 3 tf32 MMAs per product; tf32 dense peak is half of bf16"

    cpu = None
    if not args.no_cpu_baseline and world == 1:
        try:
            threads = len(os.sched_getaffinity(0))
            r, sample, secs = cpu_sample_rate(w, args.cpu_seconds, threads)
            cpu = {"value": r / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                   "sample": sample + f" ({secs:.1f} s); oracle restatement of tensor-core gemmNT"}
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"value": None, "unit": "TFLOP/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}

    line = {
        "metric": "GEMM TFLOP/s (batched bf16 GEMM + bias + GELU)" if w["dtype"] != "f32" else "GEMM TFLOP/s (f32)",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": w["dtype"], "data": "synthetic (seeded torch RNG on device; configuration distributions)",
        "config": {"workload": args.workload, "description": w["desc"], "batch_per_rank": B_, "m": M, "n": N, "k": K,
                   "out_dtype": w["out"], "parallelism": f"dp{world} (batch shards, no collective)",
                   "l2": "inputs larger than L2 (1 GiB of A+B per rank vs 126 MB L2)" if B_ > 1 else
                   "8 MiB inputs: L2-resident between launches",
                   "frac_of_peak": value / world / peak},
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    if pg:
        pg.destroy_process_group()


def main():
    args = parse_args()
    w = dict(WORKLOADS[args.workload])
    if args.batch is not None:
        w["batch"] = args.batch
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
