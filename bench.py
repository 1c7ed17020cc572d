"""Benchmark driver.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Prints one JSON line (rank 0).  Workloads:
  gemv_q4_0   Q4_0 block-quantized GEMV, batch 1: W 4096x4096 N(0,0.02) seed 0
              -> GGUF Q4_0, x fp32[4096] N(0,1) seed 1 quantized to Q8_0 in the
              kernel, y fp32[4096].  One step = one GEMV; consecutive steps
              rotate over 48 distinct device copies of W (453 MB > 2x the
              126 MB L2), so every step streams W from HBM.
The reference arm (--impl reference) times the CPU oracle (the reference's
CPU arithmetic restated in C) on the same workload on the host cores.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "arkantos-ai-stack-suite_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def measured_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "src": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS, "src": "fallback"}


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_init():
    """torch.distributed plumbing (gloo on the host) when launched by torchrun."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
        return dist, rank, world, local
    return None, 0, 1, 0


def dist_max(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


# ------------------------------------------------------------------------------------------
# Workload: Q4_0 GEMV (config 1)
# ------------------------------------------------------------------------------------------
GEMV_N = GEMV_K = 4096
GEMV_COPIES = 48
GEMV_BYTES = GEMV_N * GEMV_K // 32 * 18 + GEMV_K * 4 + GEMV_N * 4   # 9 469 952


def gemv_inputs(b2):
    w = b2.synth_normal(0, GEMV_N * GEMV_K, std=0.02).reshape(GEMV_N, GEMV_K)
    q = b2.quantize_weights(b2.Q4_0, w)
    x = b2.synth_normal(1, GEMV_K).reshape(1, GEMV_K)
    return q, x


def run_gemv_ours(args, dist, rank, world, local):
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    q, x = gemv_inputs(b2)
    mats = [b2.QMatrix(b2.Q4_0, q, GEMV_N, GEMV_K) for _ in range(GEMV_COPIES)]
    xd = b2.DeviceBuffer.from_array(x)
    yd = b2.DeviceBuffer(GEMV_N * 4)
    stream = b2.Stream()

    def step(i, s):
        mats[i % GEMV_COPIES].gemv_device(xd, 1, yd, s)

    for i in range(max(args.warmup, 3)):
        step(i, stream.h)
    stream.synchronize()
    # The K timed steps are one captured CUDA graph, so host launch overhead
    # does not leave the GPU idle between GEMVs.
    graph = b2.Graph(stream, lambda s: [step(i, s) for i in range(args.steps)])
    graph.launch()
    stream.synchronize()
    e0, e1 = b2.Event(), b2.Event()
    barrier(dist)
    with ClockSampler(local) as clk:
        t_end = time.time() + 0.4           # untimed load so the sampler sees the clocks under work
        while time.time() < t_end:
            graph.launch()
            stream.synchronize()
        e0.record(stream.h)
        graph.launch()
        e1.record(stream.h)
        stream.synchronize()
        t_end = time.time() + 0.2
        while time.time() < t_end:
            graph.launch()
            stream.synchronize()
    ms_total = e0.elapsed_ms(e1)
    ms_total = dist_max(dist, ms_total)
    ms_step = ms_total / args.steps
    gbs = GEMV_BYTES * world / (ms_step * 1e-3) / 1e9

    # e2e: host x in, host y out, through the C ABI call a host engine makes.
    mats_e2e = mats[:1]
    y = np.empty((1, GEMV_N), np.float32)
    for _ in range(3):
        y = mats_e2e[0].gemv(x)
    t0 = time.perf_counter()
    n_e2e = max(args.steps, 20)
    for _ in range(n_e2e):
        y = mats_e2e[0].gemv(x)
    e2e_s = (time.perf_counter() - t0) / n_e2e
    e2e_s = dist_max(dist, e2e_s)
    e2e_gbs = GEMV_BYTES * world / e2e_s / 1e9

    peaks = measured_peaks()
    out = {
        "metric": "Q4_0 GEMV HBM GB/s (4096x4096, batch 1)",
        "value": round(gbs, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "q4_0 x q8_0 -> int32 -> f32",
        "data": "synthetic: W N(0,0.02) seed 0 -> GGUF Q4_0; x N(0,1) seed 1",
        "config": {"workload": "gemv_q4_0 4096x4096 batch 1 (config 1)", "rotating_weight_copies": GEMV_COPIES,
                   "l2": "inputs larger than L2 (48 rotating W copies, 453 MB)", "replicas": world},
        "roofline": {"bound": "hbm", "achieved": round(GEMV_BYTES / (ms_step * 1e-3) / 1e9, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(GEMV_BYTES / (ms_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                     "traffic": None, "peak_src": peaks["src"],
                     "algorithmic_bytes_per_launch": GEMV_BYTES},
        "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": GEMV_K * 4,
                "d2h_bytes_per_step": GEMV_N * 4},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0:
        out["cpu_baseline"] = cpu_gemv_baseline(q, x, args.cpu_seconds)
    return out


def cpu_gemv_baseline(q, x, seconds: float) -> dict:
    from oracle import oracle as O
    nt = os.cpu_count() or 1
    xq = O.quantize_q8_0(x)[0]
    O.matmul(O.Q4_0, q, GEMV_N, GEMV_K, xq, nt)
    n = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        xq = O.quantize_q8_0(x)[0]
        O.matmul(O.Q4_0, q, GEMV_N, GEMV_K, xq, nt)
        n += 1
    dt = (time.perf_counter() - t0) / n
    return {"value": round(GEMV_BYTES / dt / 1e9, 3), "unit": "GB/s", "cores": nt, "kind": "port",
            "sample": f"{n} full GEMVs (quantize x + 4096 row dots) in {seconds:.0f} s"}


def run_gemv_reference(args, dist, rank, world, local):
    if rank != 0:
        return None
    import b2gguf as b2  # host-only helpers (quantizer, generator)
    from oracle import oracle as O
    q, x = gemv_inputs(b2)
    nt = os.cpu_count() or 1
    for _ in range(max(1, args.warmup)):
        O.matmul(O.Q4_0, q, GEMV_N, GEMV_K, O.quantize_q8_0(x)[0], nt)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.matmul(O.Q4_0, q, GEMV_N, GEMV_K, O.quantize_q8_0(x)[0], nt)
    dt = (time.perf_counter() - t0) / args.steps
    v = round(GEMV_BYTES / dt / 1e9, 3)
    return {"metric": "Q4_0 GEMV HBM GB/s (4096x4096, batch 1)", "value": v, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 x q8_0 -> int32 -> f32", "data": "synthetic",
            "config": {"workload": "gemv_q4_0 4096x4096 batch 1 (config 1)"}, "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": nt, "kind": "port",
                             "sample": f"{args.steps} full GEMVs on {nt} host threads"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


WORKLOADS = {"gemv_q4_0": (run_gemv_ours, run_gemv_reference)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemv_q4_0", choices=sorted(WORKLOADS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    dist, rank, world, local = dist_init()
    ours, ref = WORKLOADS[args.workload]
    out = (ref if args.impl == "reference" else ours)(args, dist, rank, world, local)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
