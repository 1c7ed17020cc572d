"""Benchmark driver.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Prints one JSON line (rank 0).  Workloads:
  decode_8b_q4k (default)
              Random-init Llama-architecture 8B decoder, GGUF Q4_K with a Q6_K
              head (32 layers, d 4096, FFN 14336, 32/8 heads, vocab 128256,
              theta 5e5, weights N(0,0.02) seed 6), tensor parallel over the
              torchrun ranks.  8 prompts of 2048 uniform random ids are
              prefilled, then one step = one greedy decode step of the batch
              of 8.  `value` times K steps of b2_generate (argmax fed back on
              the device); `e2e` times the same K steps as the host loop
              b2_decode + b2_get_argmax.  Every step reads all weights (4.36 GB
              / TP per rank) from HBM.  The line also carries the Q4_0 GEMV
              below as "q4_0_gemv".
  gemm_q4k    Prefill GEMM on the tensor cores: W 11008x4096 N(0,0.02)
              seed 2 -> GGUF Q4_K, X fp32 [512x4096] N(0,1) seed 3, Y fp32
              [512x11008]; one step = one b2_gemm (activation quantize +
              tcgen05 GEMM) over rotating W copies (> 2x L2).
  gemm_q8_0   The same GEMM with W -> GGUF Q8_0 (integer tcgen05 MMAs).
  gemv_q4_0   Q4_0 block-quantized GEMV, batch 1: W 4096x4096 N(0,0.02) seed 0
              -> GGUF Q4_0, x fp32[4096] N(0,1) seed 1 quantized to Q8_0 in the
              kernel, y fp32[4096].  One step = one GEMV; consecutive steps
              rotate over 48 distinct device copies of W (453 MB > 2x the
              126 MB L2), so every step streams W from HBM.  `value` runs the
              K independent GEMVs 48 per b2_gemv_multi launch; "chain" times
              the same K as one dependent b2_gemv launch each.
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


def progress(msg: str) -> None:
    """Phase marker on stderr (stdout carries only the JSON line)."""
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


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
# DRAM bytes of one Q4_K 28672x4096 batch-8 GEMV launch (the FFN gate|up at
# TP1) as ncu measured them: dram__bytes_read.sum + dram__bytes_write.sum.
GATE_UP_TRAFFIC = 66_165_248 + 117_760


def gemv_inputs(b2):
    w = b2.synth_normal(0, GEMV_N * GEMV_K, std=0.02).reshape(GEMV_N, GEMV_K)
    q = b2.quantize_weights(b2.Q4_0, w)
    x = b2.synth_normal(1, GEMV_K).reshape(1, GEMV_K)
    return q, x


def gemv_q4_0_graphs(b2, steps: int):
    """The config-1 timed region, K GEMVs over the rotating W copies with one
    shared x, in two captured forms: `streamed`, the GEMVs in launches of up to
    GEMV_COPIES independent matrices each (b2_gemv_multi: the weights stream
    back to back through one pipeline); `chain`, one launch per GEMV, each
    waiting on the previous one (b2_gemv).  Returns (graphs, stream, launches)."""
    q, x = gemv_inputs(b2)
    mats = [b2.QMatrix(b2.Q4_0, q, GEMV_N, GEMV_K) for _ in range(GEMV_COPIES)]
    xd = b2.DeviceBuffer.from_array(x)
    ys = [b2.DeviceBuffer(GEMV_N * 4) for _ in range(GEMV_COPIES)]
    stream = b2.Stream()

    def streamed(s):
        i = 0
        while i < steps:
            n = min(GEMV_COPIES, steps - i)
            b2.gemv_multi(mats[:n], xd, 1, ys[:n], s)
            i += n

    def chain(s):
        for i in range(steps):
            mats[i % GEMV_COPIES].gemv_device(xd, 1, ys[0], s)

    for f in (streamed, chain):
        f(stream.h)
    stream.synchronize()
    graphs = {"streamed": b2.Graph(stream, streamed), "chain": b2.Graph(stream, chain)}
    for g in graphs.values():
        g.launch()
    stream.synchronize()
    launches = {"streamed": -(-steps // GEMV_COPIES), "chain": steps}
    return graphs, stream, launches, (q, x, mats, xd, ys)


def time_graph(b2, g, stream) -> float:
    e0, e1 = b2.Event(), b2.Event()
    e0.record(stream.h)
    g.launch()
    e1.record(stream.h)
    stream.synchronize()
    return e0.elapsed_ms(e1)


def run_gemv_ours(args, dist, rank, world, local):
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    graphs, stream, launches, keep = gemv_q4_0_graphs(b2, args.steps)
    q, x, mats = keep[0], keep[1], keep[2]
    for _ in range(max(args.warmup, 3)):
        for g in graphs.values():
            g.launch()
    stream.synchronize()
    barrier(dist)
    with ClockSampler(local) as clk:
        t_end = time.time() + 0.4           # untimed load so the sampler sees the clocks under work
        while time.time() < t_end:
            graphs["streamed"].launch()
            stream.synchronize()
        ms_total = time_graph(b2, graphs["streamed"], stream)
        ms_chain = time_graph(b2, graphs["chain"], stream)
        t_end = time.time() + 0.2
        while time.time() < t_end:
            graphs["streamed"].launch()
            stream.synchronize()
    ms_total = dist_max(dist, ms_total)
    ms_chain = dist_max(dist, ms_chain)
    ms_step = ms_total / args.steps
    gbs = GEMV_BYTES * world / (ms_step * 1e-3) / 1e9
    chain_gbs = GEMV_BYTES * world / (ms_chain / args.steps * 1e-3) / 1e9

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
                   "l2": "inputs larger than L2 (48 rotating W copies, 453 MB)", "replicas": world,
                   "timed_region": f"K GEMVs of distinct W copies with one x, {GEMV_COPIES} per b2_gemv_multi launch"},
        "roofline": {"bound": "hbm", "achieved": round(GEMV_BYTES / (ms_step * 1e-3) / 1e9, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(GEMV_BYTES / (ms_step * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                     "traffic": None, "peak_src": peaks["src"],
                     "algorithmic_bytes_per_launch": GEMV_BYTES * GEMV_COPIES,
                     "algorithmic_bytes_per_gemv": GEMV_BYTES},
        "chain": {"value": round(chain_gbs, 1), "unit": "GB/s", "frac": round(chain_gbs / world / peaks["hbm_gbs"], 4),
                  "ms_per_gemv": ms_chain / args.steps,
                  "note": "one b2_gemv launch per GEMV, each waiting on the previous (programmatic dependent launch)"},
        "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": GEMV_K * 4,
                "d2h_bytes_per_step": GEMV_N * 4},
        "gpu_launches": launches["streamed"],
        "clocks": clk.summary(),
    }
    if rank == 0:
        out["cpu_baseline"] = cpu_gemv_baseline(q, x, args.cpu_seconds)
    return out


def gemv_q4_0_measure(b2, steps: int) -> dict:
    """Config-1 Q4_0 GEMV (the metric's second half) on the current device:
    CUDA-event time of `steps` GEMVs captured in one graph over rotating
    copies, streamed (b2_gemv_multi) and as a dependent chain (b2_gemv)."""
    graphs, stream, _, keep = gemv_q4_0_graphs(b2, steps)
    for g in graphs.values():
        g.launch()
    stream.synchronize()
    ms = time_graph(b2, graphs["streamed"], stream) / steps
    ms_chain = time_graph(b2, graphs["chain"], stream) / steps
    gbs = GEMV_BYTES / (ms * 1e-3) / 1e9
    chain_gbs = GEMV_BYTES / (ms_chain * 1e-3) / 1e9
    peaks = measured_peaks()
    return {"metric": "Q4_0 GEMV HBM GB/s (4096x4096, batch 1)", "value": round(gbs, 1), "unit": "GB/s",
            "frac": round(gbs / peaks["hbm_gbs"], 4), "peak": peaks["hbm_gbs"], "ms_per_gemv": ms,
            "algorithmic_bytes_per_gemv": GEMV_BYTES, "launches": -(-steps // GEMV_COPIES),
            "form": f"{GEMV_COPIES} independent GEMVs per b2_gemv_multi launch",
            "chain": {"value": round(chain_gbs, 1), "frac": round(chain_gbs / peaks["hbm_gbs"], 4),
                      "ms_per_gemv": ms_chain, "form": "one b2_gemv launch per GEMV"}}


def cpu_gemv_baseline(q, x, seconds: float) -> dict:
    from oracle import oracle as O
    nt = os.cpu_count() or 1
    xq = O.quantize_q8_0(x)[0]
    O.matmul(O.Q4_0, q, GEMV_N, GEMV_K, xq, nt)
    n = 0
    t0 = time.perf_counter()
    while n == 0 or time.perf_counter() - t0 < seconds:
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


# ------------------------------------------------------------------------------------------
# Workload: 8B Q4_K decode, tensor parallel (config 5)
# ------------------------------------------------------------------------------------------
LLAMA_8B = dict(n_layer=32, n_embd=4096, n_ff=14336, n_head=32, n_head_kv=8, n_vocab=128256, seed=6,
                rope_theta=500000.0, n_ctx_train=8192)
BATCH = 8
PROMPT = 2048
CLOCK_LOAD_STEPS = 32


def q_bytes(t: int, n: int, k: int) -> int:
    per = {2: 18 / 32, 8: 34 / 32, 12: 144 / 256, 14: 210 / 256}[t]
    return int(n * k * per)


def decode_weight_bytes(world: int = 1) -> int:
    """Algorithmic weight bytes one decode step reads on one rank (GGUF block bytes)."""
    c = LLAMA_8B
    d, ff, hd = c["n_embd"], c["n_ff"], c["n_embd"] // c["n_head"]
    kv = c["n_head_kv"] * hd
    layer = q_bytes(12, d + 2 * kv, d) + q_bytes(12, d, d) + q_bytes(12, 2 * ff, d) + q_bytes(12, d, ff)
    head = q_bytes(14, c["n_vocab"], d)
    return (c["n_layer"] * layer + head) // world


def decode_kv_bytes(ctx_lens, world: int = 1, row_bytes: int | None = None) -> int:
    """K and V bytes the attention of one step reads on one rank: per sequence
    and layer 2 x n_kv heads x the bytes of a cached row (fp16: 2 x head_dim;
    Q8_0: head_dim + 16) x the positions attended."""
    c = LLAMA_8B
    hd = c["n_embd"] // c["n_head"]
    rb = 2 * hd if row_bytes is None else row_bytes
    return sum(c["n_layer"] * 2 * c["n_head_kv"] * rb * int(n) for n in ctx_lens) // world


def decode_q8_0_cache(b2, dist, model, args, warm: int, world: int) -> dict:
    """The same batch-8 greedy decode (b2_generate, CUDA events, max over
    ranks) over a Q8_0 K and V cache, Milda's default cache types: the
    prompts are prefilled into a fresh context of that type first."""
    n_ctx = PROMPT + warm + args.steps + 8
    ctx = b2.Context(model, n_ctx=n_ctx, n_seq=BATCH, type_k=b2.Q8_0, type_v=b2.Q8_0)
    prompts = prompts_8b()
    first = []
    for s in range(BATCH):
        ctx.decode(prompts[s], pos=np.arange(PROMPT), seq=np.full(PROMPT, s), want_logits=2)
        first.append(int(ctx.argmax()[0][-1]))
    seqs = np.arange(BATCH, dtype=np.int32)
    ids = ctx.generate(first, warm, seq=seqs)
    e0, e1 = b2.Event(), b2.Event()
    barrier(dist)
    e0.record(ctx.stream)
    ctx.generate(ids[-1].copy(), args.steps, seq=seqs)
    e1.record(ctx.stream)
    ctx.synchronize()
    ms_total = dist_max(dist, e0.elapsed_ms(e1))
    ms_step = ms_total / args.steps
    p_start = PROMPT + warm
    ctx_lens = [p_start + k + 1 for k in range(args.steps) for _ in range(BATCH)]
    kv = decode_kv_bytes(ctx_lens, world, int(b2.lib.b2_kv_row_bytes(b2.Q8_0, LLAMA_8B["n_embd"] // LLAMA_8B["n_head"])))
    del ctx
    return {"metric": "decode tok/s (Llama-shape 8B Q4_K, batch 8, Q8_0 K and V cache)",
            "value": round(BATCH * args.steps / (ms_total * 1e-3), 1), "unit": "tok/s", "steps": args.steps,
            "ms_per_step": ms_step, "kv_bytes_per_step": int(kv / args.steps),
            "timed_region": "b2_generate: K greedy steps, device-side feedback"}


def model_path(tag: str) -> str:
    base = "/dev/shm" if os.path.isdir("/dev/shm") else "/tmp"
    try:
        st = os.statvfs(base)
        if st.f_bavail * st.f_frsize < 8 << 30:
            base = "/tmp"
    except OSError:
        base = "/tmp"
    return os.path.join(base, f"b2_bench_{tag}_{os.getpid() if tag == 'local' else 'shared'}.gguf")


def write_8b(b2, path: str) -> float:
    t0 = time.perf_counter()
    c = LLAMA_8B
    b2.write_synthetic_llama(path + ".part", c["n_layer"], c["n_embd"], c["n_ff"], c["n_head"], c["n_head_kv"],
                             c["n_vocab"], b2.Q4_K, embd_type=b2.Q4_K, out_type=b2.Q6_K, seed=c["seed"],
                             rope_theta=c["rope_theta"], n_ctx_train=c["n_ctx_train"])
    os.replace(path + ".part", path)
    return time.perf_counter() - t0


def prompts_8b() -> np.ndarray:
    rng = np.random.default_rng(LLAMA_8B["seed"])
    return rng.integers(0, LLAMA_8B["n_vocab"], (BATCH, PROMPT)).astype(np.int32)


def launches_per_step(n_layer: int, small_o: bool = False) -> int:
    """Kernels of this library one decode step launches: embed; per layer
    RMSNorm (+ Q8 image), QKV GEMV (RoPE + KV store epilogue), attention
    scores, attention exponentials, attention sum + P.V, quantize (O input;
    none when the O input is small enough for the GEMV to quantize it
    itself), O GEMV, RMSNorm (+ image), gate|up GEMV (SwiGLU epilogue),
    quantize (down input), down GEMV; then RMSNorm, head GEMV and argmax
    (the launch list of one 8B step counts 356).  No library collective runs
    in a step."""
    return 1 + (10 if small_o else 11) * n_layer + 3


def time_gemv_shape(b2, qtype: int, n: int, k: int, n_tok: int, steps: int, seed: int) -> dict:
    """CUDA-event timing of one GEMV shape over rotating weight copies (> 2x L2)."""
    w = b2.synth_normal(seed, n * k, std=0.02).reshape(n, k)
    q = b2.quantize_weights(qtype, w)
    wb = q.nbytes
    copies = max(2, -(-300_000_000 // wb))
    mats = [b2.QMatrix(qtype, q, n, k) for _ in range(copies)]
    x = b2.synth_normal(seed + 1, n_tok * k).reshape(n_tok, k)
    xd = b2.DeviceBuffer.from_array(x)
    yd = b2.DeviceBuffer(n_tok * n * 4)
    stream = b2.Stream()
    for i in range(3 * copies):
        mats[i % copies].gemv_device(xd, n_tok, yd, stream.h)
    graph = b2.Graph(stream, lambda s: [mats[i % copies].gemv_device(xd, n_tok, yd, s) for i in range(steps)])
    graph.launch()
    stream.synchronize()
    e0, e1 = b2.Event(), b2.Event()
    e0.record(stream.h)
    graph.launch()
    e1.record(stream.h)
    stream.synchronize()
    ms = e0.elapsed_ms(e1) / steps
    nbytes = wb + n_tok * k * 4 + n_tok * n * 4
    return {"ms": ms, "bytes": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9, "copies": copies}


def tp_share(dist, rank: int, world: int, make_id, path: str):
    """Rank 0's NCCL unique id (tensor parallelism) and model path, sent to every rank."""
    obj = [make_id() if rank == 0 and world > 1 else None, path]
    if dist is not None:
        dist.broadcast_object_list(obj, src=0)
    return obj[0], obj[1]


def prefill_report(c, t_prefill: float, world: int, peaks: dict) -> dict:
    """Config-5 prefill (8 prompts x 2048 tokens, one b2_decode call each):
    wall time, and the projections' FLOP rate against the tensor roofline."""
    d, ff, hd = c["n_embd"], c["n_ff"], c["n_embd"] // c["n_head"]
    per_layer = (c["n_head"] + 2 * c["n_head_kv"]) * hd * d + d * d + 3 * ff * d
    flop = 2.0 * c["n_layer"] * per_layer * BATCH * PROMPT
    tflops = flop / t_prefill / 1e12
    return {"tok_s": round(BATCH * PROMPT / t_prefill, 1), "seconds": round(t_prefill, 2),
            "projection_tflop": round(flop / 1e12, 1), "projection_tflop_s": round(tflops, 1),
            "roofline": {"bound": "tensor", "achieved": round(tflops / world, 1), "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s per GPU", "frac": round(tflops / world / peaks["bf16_tflops"], 4),
                         "peak_src": peaks["src"] + " bf16 burst"},
            "path": ("all but the last 8 tokens of each prompt through the tensor-core GEMM chunks" if world == 1
                     else "decode GEMV steps of 8 tokens (tensor-parallel)"),
            "timing": "host wall clock around the 8 b2_decode calls and their argmax reads"}


def decode_config(world: int) -> dict:
    """The config-5 workload as both arms report it."""
    return {"workload": "decode_8b_q4k: 32 layers, d 4096, ffn 14336, 32/8 heads, hd 128, vocab 128256, "
                        "theta 5e5; batch 8 x 2048-token prompts, greedy steps (config 5)",
            "global_batch": BATCH, "seq_len": PROMPT, "parallelism": f"tp{world}",
            "l2": f"inputs larger than L2 ({decode_weight_bytes(world) / 1e9:.2f} GB of weights per rank per step)"}


def run_decode_ours(args, dist, rank, world, local):
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    c = LLAMA_8B
    path = model_path("8b_q4k")
    t_write = 0.0
    if rank == 0 and not os.path.exists(path):
        progress("writing the synthetic 8B GGUF")
        t_write = write_8b(b2, path)
    nccl_id, path = tp_share(dist, rank, world, b2.nccl_unique_id, path)
    progress("loading")
    barrier(dist)
    t0 = time.perf_counter()
    model = b2.Model(path, device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    t_load = time.perf_counter() - t0
    load = {"seconds": round(t_load, 3), "file_bytes": os.path.getsize(path), "device_bytes": model.device_bytes(),
            "file_gb_per_s": round(os.path.getsize(path) / t_load / 1e9, 2),
            "path": "mmap (sequential read-ahead) -> multithreaded repack into two pinned slabs -> async H2D; "
                    "page cache released after the upload"}
    warm = max(args.warmup, 3)
    n_ctx = PROMPT + warm + CLOCK_LOAD_STEPS + args.steps + 8
    ctx = b2.Context(model, n_ctx=n_ctx, n_seq=BATCH)
    prompts = prompts_8b()
    progress("prefill")
    # Prefill: each prompt through b2_decode (8-token steps), last logits -> first greedy token.
    barrier(dist)
    t0 = time.perf_counter()
    first = []
    for s in range(BATCH):
        ctx.decode(prompts[s], pos=np.arange(PROMPT), seq=np.full(PROMPT, s), want_logits=2)
        first.append(int(ctx.argmax()[0][-1]))
    t_prefill = dist_max(dist, time.perf_counter() - t0)
    seqs = np.arange(BATCH, dtype=np.int32)
    progress(f"prefill done in {t_prefill:.1f} s; warm-up")
    # Warm-up steps (graph capture on the first), then the state the timed steps start from.
    ids = ctx.generate(first, warm, seq=seqs)
    start_tok = ids[-1].copy()
    p_start = PROMPT + warm

    def rewind():
        for s in range(BATCH):
            ctx.kv_seq_rm(s, p_start, -1)

    e0, e1 = b2.Event(), b2.Event()
    barrier(dist)
    progress("timed steps")
    with ClockSampler(local) as clk:
        ctx.generate(start_tok, CLOCK_LOAD_STEPS, seq=seqs)     # untimed load: clocks seen under work
        rewind()
        ctx.exchange_wait_ns(reset=True)
        barrier(dist)
        if args.profile_range:
            b2.check(b2.lib.b2_profiler_range(1), "profiler_range")
        e0.record(ctx.stream)
        gen = ctx.generate(start_tok, args.steps, seq=seqs)
        e1.record(ctx.stream)
        ctx.synchronize()
        wait_us = ctx.exchange_wait_ns() / 1e3 / args.steps
        if args.profile_range:
            b2.check(b2.lib.b2_profiler_range(0), "profiler_range")
    ms_total = dist_max(dist, e0.elapsed_ms(e1))
    ms_step = ms_total / args.steps
    tok_s = BATCH * args.steps / (ms_total * 1e-3)
    exchange = None
    if world > 1:
        # each waiting kernel's first CTA adds the wall time of its wait for
        # the peers' partials (attention-out, FFN-down, the head shards)
        exchange = {"wait_us_per_step_max_rank": round(dist_max(dist, wait_us), 1),
                    "wait_us_per_step_rank0": round(wait_us, 1), "step_us": round(ms_step * 1e3, 1),
                    "waits_per_step": 2 * c["n_layer"] + 1,
                    "note": "wall time of the exchange waits (globaltimer, 256 ns resolution) against the step"}

    # The same steps with Milda's sampler chain drawing every row on the
    # device (penalties, top-k 40, top-p 0.9, min-p 0.05, temperature 0.75,
    # dist; one chain per row, seeds 42 + row) instead of the greedy argmax.
    progress("sampled steps")
    samplers = [b2.Sampler(ctx, seed=42 + i) for i in range(BATCH)]
    rewind()
    ctx.generate_sampled(samplers, start_tok, 2, seq=seqs)    # untimed: the sampled step's graph is captured
    rewind()
    for sm in samplers:
        sm.reset()
    barrier(dist)
    e0.record(ctx.stream)
    ctx.generate_sampled(samplers, start_tok, args.steps, seq=seqs)
    e1.record(ctx.stream)
    ctx.synchronize()
    ms_sampled = dist_max(dist, e0.elapsed_ms(e1)) / args.steps
    del samplers

    # e2e: the llama-style host loop through the C ABI (b2_decode with host
    # token/pos/seq arrays, b2_get_argmax back to the host) from the same state.
    progress("e2e host loop")
    rewind()
    tok = start_tok.copy()
    e2e_ids = np.empty_like(gen)
    barrier(dist)
    t0 = time.perf_counter()
    for k in range(args.steps):
        ctx.decode(tok, pos=np.full(BATCH, p_start + k, np.int32), seq=seqs, want_logits=1)
        tok = ctx.argmax(BATCH)[0].copy()
        e2e_ids[k] = tok
    e2e_s = dist_max(dist, time.perf_counter() - t0)
    e2e_tok_s = BATCH * args.steps / e2e_s

    # Roofline of the whole step (weights + KV this rank reads) and of the
    # dominant kernel measured alone: the gate|up Q4_K GEMV at batch 8.
    peaks = measured_peaks()
    ctx_lens = [p_start + k + 1 for k in range(args.steps) for _ in range(BATCH)]
    step_bytes = decode_weight_bytes(world) + decode_kv_bytes(ctx_lens, world) / args.steps
    step_gbs = step_bytes / (ms_step * 1e-3) / 1e9
    ff_l = c["n_ff"] // world
    progress("kernel roofline")
    g = time_gemv_shape(b2, b2.Q4_K, 2 * ff_l, c["n_embd"], BATCH, 64, 7)
    del ctx
    progress("decode over a Q8_0 KV cache")
    q8kv = decode_q8_0_cache(b2, dist, model, args, warm, world)
    del model
    q40 = gemv_q4_0_measure(b2, 200) if rank == 0 else None
    out = {
        "metric": "decode tok/s (Llama-shape 8B Q4_K, batch 8)",
        "value": round(tok_s, 1),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": warm,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q4_k/q6_k x q8_k -> int32 -> f32, fp16 KV",
        "data": "synthetic: random-init Llama 8B (N(0,0.02) seed 6) GGUF Q4_K + Q6_K head; uniform random prompt ids",
        "config": decode_config(world),
        "roofline": {"bound": "hbm", "kernel": f"gemv Q4_K batch 8, {2 * ff_l}x{c['n_embd']} (ffn gate|up)",
                     "achieved": round(g["gbs"], 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(g["gbs"] / peaks["hbm_gbs"], 4),
                     "traffic": GATE_UP_TRAFFIC if world == 1 else None,
                     "traffic_src": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                                    "(profiles/gemv_kernel_q4k_28672x4096_b8.md); the TP shards are other shapes",
                     "peak_src": peaks["src"],
                     "algorithmic_bytes_per_launch": g["bytes"], "ms_per_launch": g["ms"]},
        "step_roofline": {"achieved": round(step_gbs, 1), "unit": "GB/s", "frac": round(step_gbs / peaks["hbm_gbs"], 4),
                          "algorithmic_bytes_per_step": int(step_bytes),
                          "note": "weights + fp16 KV read per rank per step / device time per step"},
        "e2e": {"value": round(e2e_tok_s, 1), "unit": "tok/s", "h2d_bytes_per_step": 3 * BATCH * 4,
                "d2h_bytes_per_step": 32 * 4, "greedy_ids_equal_device_loop": bool(np.array_equal(e2e_ids, gen))},
        "timed_region": "b2_generate: K greedy steps, device-side feedback",
        "context_at_start": p_start,
        "gpu_launches": launches_per_step(c["n_layer"]) * args.steps,
        "clocks": clk.summary(),
        "setup_s": {"write_gguf": round(t_write, 1), "load": round(t_load, 1), "prefill": round(t_prefill, 1)},
        "load": load,
        "exchange": exchange,
        "decode_sampled": {"value": round(BATCH / (ms_sampled * 1e-3), 1), "unit": "tok/s",
                           "ms_per_step": ms_sampled, "steps": args.steps,
                           "chain": "Milda's defaults on the device: penalties over 64 tokens (1.08), top-k 40, "
                                    "top-p 0.90, min-p 0.05, temperature 0.75, dist (mt19937, seed 42 + row)"},
        "prefill_tok_s": round(BATCH * PROMPT / t_prefill, 1),
        "prefill": prefill_report(c, t_prefill, world, peaks),
    }
    out["decode_q8_0_kv"] = q8kv
    if q40 is not None:
        out["q4_0_gemv"] = q40
    if world == 1 and not args.skip_1b:
        progress("config-4 decode (1.1B Q4_0, batch 1)")
        sub = argparse.Namespace(**vars(args))
        sub.steps = min(args.steps, GEN_1B)
        sub.cpu_seconds = min(args.cpu_seconds, 5.0)
        d1 = run_decode1b_ours(sub, None, 0, 1, local)
        out["decode_1b_q4_0"] = {k: d1[k] for k in ("metric", "value", "unit", "steps", "ms_per_step", "roofline",
                                                     "e2e", "gpu_launches", "clocks") if k in d1}
        if "cpu_baseline" in d1:
            out["decode_1b_q4_0"]["cpu_baseline"] = d1["cpu_baseline"]
    if rank == 0:
        progress("cpu baseline")
        out["cpu_baseline"] = cpu_decode_baseline(path, args.cpu_seconds)
    barrier(dist)
    if rank == 0 and not args.keep_model:
        try:
            os.remove(path)
        except OSError:
            pass
    return out


def cpu_decode_samples(path: str, n_samples: int | None, seconds: float | None, warm: int, layers: int | None = None,
                       ctx_len: int = PROMPT, with_time: bool = False):
    """Oracle decode of one token of a model at context ctx_len, timed as
    samples: one decoder layer per sample (cycling over all layers, so every
    layer's weights come from DRAM), plus embed+final norm+head samples.
    Returns (seconds per token extrapolated, samples, threads)."""
    from oracle import oracle as O
    nt = os.cpu_count() or 1
    m = O.Model(path)
    m.init_cache(1, ctx_len + 8)
    m.cache_fill(0x3C00)
    nl = m.n_layers
    tok, pos = 17, ctx_len
    t_layer, t_head = [], []

    def sample(i):
        j = (i + nl) % (nl + 1)      # the head first, then layers 0..nl-1, cycling
        t0 = time.perf_counter()
        if j == nl:
            m.forward_range(0, tok, pos, 0, 0, logits=True, n_threads=nt)
            t_head.append(time.perf_counter() - t0)
        else:
            m.forward_range(0, tok, pos, j, j + 1, logits=False, n_threads=nt)
            t_layer.append(time.perf_counter() - t0)

    for i in range(warm):
        sample(0 if i % 2 == 0 else nl)   # head and last layer: page the mapping in
    t_layer.clear()
    t_head.clear()
    i, t_start = 0, time.perf_counter()
    while True:
        if n_samples is not None and i >= n_samples:
            break
        if seconds is not None and time.perf_counter() - t_start >= seconds and t_head and t_layer:
            break
        sample(i)
        i += 1
    if not t_layer:
        sample(1)
        i += 1
    timed = float(np.sum(t_layer) + np.sum(t_head))
    per_tok = nl * float(np.mean(t_layer)) + float(np.mean(t_head))
    return (per_tok, i, nt, timed) if with_time else (per_tok, i, nt)


def cpu_decode_baseline(path: str, seconds: float) -> dict:
    per_tok, n, nt = cpu_decode_samples(path, None, seconds, 2)
    return {"value": round(1.0 / per_tok, 4), "unit": "tok/s", "cores": nt, "kind": "port",
            "sample": f"{n} samples of one token at context {PROMPT}: single decoder layers cycling over all 32 "
                      f"plus embed+norm+head; tok/s = 1 / (32 x mean layer + head) (the CPU path decodes the batch "
                      f"token by token, so batch 8 does not change tok/s)"}


def write_8b_cpu_arm(path: str) -> None:
    """The config-5 model file for the CPU reference arm, written by the
    oracle's numpy GGUF writer (same shapes and block types; random valid
    blocks), so the arm's process loads no product library."""
    from oracle import synth_gguf as S
    c = LLAMA_8B
    S.write_llama(path + ".part", c["n_layer"], c["n_embd"], c["n_ff"], c["n_head"], c["n_head_kv"], c["n_vocab"],
                  S.Q4_K, S.Q4_K, S.Q6_K, c["seed"], rope_theta=c["rope_theta"], n_ctx_train=c["n_ctx_train"])
    os.replace(path + ".part", path)


def run_decode_reference(args, dist, rank, world, local):
    """The reference's CPU decode path (the oracle port) on the host cores.
    A step is one timed sample: one decoder layer of one token (cycling over
    all 32) or embed + norm + head.  ms_per_step is the mean sample time the
    run measured; value is the tok/s those samples extrapolate to (one token
    = 32 layer samples + 1 head sample)."""
    if rank != 0:
        return None
    path = model_path("8b_q4k_cpu")
    if not os.path.exists(path):
        write_8b_cpu_arm(path)
    t0 = time.perf_counter()
    per_tok, n, nt, timed_s = cpu_decode_samples(path, args.steps, None, args.warmup, with_time=True)
    wall = time.perf_counter() - t0
    if not args.keep_model:
        try:
            os.remove(path)
        except OSError:
            pass
    v = round(1.0 / per_tok, 4)
    return {"metric": "decode tok/s (Llama-shape 8B Q4_K, batch 8)", "value": v, "unit": "tok/s", "n_gpus": world,
            "steps": n, "warmup": args.warmup, "ms_per_step": timed_s / n * 1e3,
            "value_kind": "extrapolated: 1 / (32 x mean layer sample + mean head sample) per token",
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "q4_k/q6_k x q8_k -> int32 -> f32, fp16 KV",
            "data": "synthetic: Llama 8B shapes, Q4_K layers + Q6_K head with random valid blocks (oracle writer)",
            "config": decode_config(world),
            "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "tok/s", "cores": nt, "kind": "port",
                             "sample": f"each step one sample: a single decoder layer (cycling over all 32) or "
                                       f"embed+norm+head of one token at context {PROMPT}; {n} samples timed in "
                                       f"{timed_s:.1f} s ({wall:.0f} s with warm-up)"},
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------------------------------------
# Workload: 1.1B Q4_0 decode, batch 1 (config 4)
# ------------------------------------------------------------------------------------------
LLAMA_1B = dict(n_layer=22, n_embd=2048, n_ff=5632, n_head=32, n_head_kv=4, n_vocab=32000, seed=5,
                rope_theta=10000.0, n_ctx_train=2048)
PROMPT_1B, GEN_1B = 128, 256


def write_1b(b2, path: str) -> float:
    t0 = time.perf_counter()
    c = LLAMA_1B
    b2.write_synthetic_llama(path + ".part", c["n_layer"], c["n_embd"], c["n_ff"], c["n_head"], c["n_head_kv"],
                             c["n_vocab"], b2.Q4_0, embd_type=b2.Q4_0, out_type=b2.Q4_0, seed=c["seed"],
                             rope_theta=c["rope_theta"], n_ctx_train=c["n_ctx_train"])
    os.replace(path + ".part", path)
    return time.perf_counter() - t0


def weight_bytes_1b() -> int:
    c = LLAMA_1B
    d, ff, hd = c["n_embd"], c["n_ff"], c["n_embd"] // c["n_head"]
    qkv = (c["n_head"] + 2 * c["n_head_kv"]) * hd
    per_layer = q_bytes(2, qkv, d) + q_bytes(2, d, d) + q_bytes(2, 2 * ff, d) + q_bytes(2, d, ff)
    return c["n_layer"] * per_layer + q_bytes(2, c["n_vocab"], d)


def run_decode1b_ours(args, dist, rank, world, local):
    """Config 4: 128-token prompt, then GEN_1B greedy steps of one sequence,
    timed as one b2_generate call (device-side feedback) with CUDA events;
    e2e is the host loop b2_decode + b2_get_argmax over the same steps."""
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    c = LLAMA_1B
    path = model_path("1b_q4_0")
    t_write = write_1b(b2, path) if rank == 0 and not os.path.exists(path) else 0.0
    nccl_id, path = tp_share(dist, rank, world, b2.nccl_unique_id, path)
    model = b2.Model(path, device=local, tp_rank=rank, tp_size=world, nccl_id=nccl_id)
    n_ctx = PROMPT_1B + 2 * GEN_1B + 16
    ctx = b2.Context(model, n_ctx=n_ctx, n_seq=1)
    prompt = np.random.default_rng(c["seed"]).integers(0, c["n_vocab"], PROMPT_1B).astype(np.int32)
    ctx.decode(prompt, want_logits=2)
    first = int(ctx.argmax()[0][-1])
    steps = min(args.steps, GEN_1B)
    warm = max(args.warmup, 3)
    ctx.generate([first], warm, seq=[0])          # graph capture + warm-up
    ctx.kv_seq_rm(0, PROMPT_1B, -1)
    e0, e1 = b2.Event(), b2.Event()
    barrier(dist)
    with ClockSampler(local) as clk:
        e0.record(ctx.stream)
        gen = ctx.generate([first], steps, seq=[0])
        e1.record(ctx.stream)
        ctx.synchronize()
    ms = dist_max(dist, e0.elapsed_ms(e1))
    tok_s = steps / (ms * 1e-3)
    ctx.kv_seq_rm(0, PROMPT_1B, -1)
    tok, ids = first, []
    barrier(dist)
    t0 = time.perf_counter()
    for k in range(steps):
        ctx.decode([tok], pos=[PROMPT_1B + k], seq=[0], want_logits=1)
        tok = int(ctx.argmax()[0][0])
        ids.append(tok)
    e2e_s = dist_max(dist, time.perf_counter() - t0)
    peaks = measured_peaks()
    hd = c["n_embd"] // c["n_head"]
    kv_step = sum(c["n_layer"] * 2 * c["n_head_kv"] * hd * 2 * (PROMPT_1B + k + 1) for k in range(steps)) / steps
    step_bytes = (weight_bytes_1b() + kv_step) / world
    step_gbs = step_bytes / (ms / steps * 1e-3) / 1e9
    out = {"metric": "decode tok/s (Llama-shape 1.1B Q4_0, batch 1)", "value": round(tok_s, 1), "unit": "tok/s",
           "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": ms / steps, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "q4_0 x q8_0 -> int32 -> f32, fp16 KV",
           "data": "synthetic: random-init Llama 1.1B (N(0,0.02) seed 5) GGUF Q4_0; uniform random prompt ids",
           "config": {"workload": "decode_1b_q4_0: 22 layers, d 2048, ffn 5632, 32/4 heads, hd 64, vocab 32000; "
                                  "128-token prompt, greedy steps, batch 1 (config 4)",
                      "global_batch": 1, "seq_len": PROMPT_1B, "parallelism": f"tp{world}",
                      "l2": "inputs larger than L2 (0.62 GB of weights per step)"},
           "roofline": {"bound": "hbm", "kernel": "decode step (weights + KV per token)",
                        "achieved": round(step_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": round(step_gbs / peaks["hbm_gbs"], 4), "traffic": None, "peak_src": peaks["src"],
                        "algorithmic_bytes_per_launch": int(step_bytes)},
           "e2e": {"value": round(steps / e2e_s, 1), "unit": "tok/s", "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 128,
                   "greedy_ids_equal_device_loop": bool(np.array_equal(np.array(ids), gen.ravel()[:steps]))},
           "gpu_launches": launches_per_step(c["n_layer"], small_o=True) * steps, "clocks": clk.summary(),
           "setup_s": {"write_gguf": round(t_write, 1)}}
    del ctx, model
    if rank == 0 and args.cpu_seconds > 0:
        per_tok, n, nt = cpu_decode_samples(path, None, args.cpu_seconds, 2, layers=c["n_layer"], ctx_len=PROMPT_1B)
        out["cpu_baseline"] = {"value": round(1.0 / per_tok, 3), "unit": "tok/s", "cores": nt, "kind": "port",
                               "sample": f"{n} samples of one token at context {PROMPT_1B}: single decoder layers "
                                         f"cycling over all {c['n_layer']} plus embed+norm+head"}
    barrier(dist)
    if rank == 0 and not args.keep_model:
        try:
            os.remove(path)
        except OSError:
            pass
    return out


# ------------------------------------------------------------------------------------------
# Workload: decode attention over an fp16 KV cache + in-place KV shift (config 3)
# ------------------------------------------------------------------------------------------
ATTN_HEADS, ATTN_KV, ATTN_HD, ATTN_CTX = 32, 8, 128, 4096


def attn_measure(b2, n_seq: int, steps: int, kv_type: int = 1) -> dict:
    """CUDA-event time of b2_attn_decode_typed (one query per sequence at
    position ctx-1, all ctx positions attended) over rotating KV copies
    larger than L2, and of the shift that drops the first 1024 positions and
    re-ropes K.  kv_type: B2_F16 (1) or B2_Q8_0 (8) for both caches; Q8_0
    rows hold random codes and a fixed block scale."""
    rng = np.random.default_rng(4)
    rb = int(b2.lib.b2_kv_row_bytes(kv_type, ATTN_HD))   # bytes per cached row (one kv head, one position)
    rows = ATTN_KV * ATTN_CTX * n_seq
    kv_bytes = 2 * rows * rb
    copies = max(1, -(-300_000_000 // kv_bytes))
    if kv_type == b2.F16:
        kv = rng.standard_normal(rows * ATTN_HD, dtype=np.float32).astype(np.float16).view(np.uint8)
    else:
        cb = ATTN_HD if kv_type == b2.Q8_0 else ATTN_HD // 2      # code bytes of a row
        kv = np.zeros((rows, rb), np.uint8)
        kv[:, :cb] = rng.integers(0, 256, (rows, cb), dtype=np.uint8)
        kv[:, cb:cb + ATTN_HD // 16] = np.frombuffer(np.float16(0.01).tobytes() * (ATTN_HD // 32), np.uint8)
        kv = kv.ravel()
    ks = [b2.DeviceBuffer.from_array(kv) for _ in range(copies)]
    vs = [b2.DeviceBuffer.from_array(kv[::-1].copy()) for _ in range(copies)]
    q = b2.DeviceBuffer.from_array(rng.standard_normal((n_seq, ATTN_HEADS * ATTN_HD), dtype=np.float32))
    out = b2.DeviceBuffer(n_seq * ATTN_HEADS * ATTN_HD * 4)
    pos = b2.DeviceBuffer.from_array(np.full(n_seq, ATTN_CTX - 1, np.int32))
    seq = b2.DeviceBuffer.from_array(np.arange(n_seq, dtype=np.int32))
    stream = b2.Stream()

    def one(i, s):
        b2.check(b2.lib.b2_attn_decode_typed(q.ptr, ks[i % copies].ptr, kv_type, vs[i % copies].ptr, kv_type, pos.ptr,
                                             seq.ptr, n_seq, n_seq, ATTN_HEADS, ATTN_KV, ATTN_HD, ATTN_CTX, out.ptr, s),
                 "attn_decode")

    for i in range(2 * copies):
        one(i, stream.h)
    graph = b2.Graph(stream, lambda s: [one(i, s) for i in range(steps)])
    graph.launch()
    stream.synchronize()
    e0, e1 = b2.Event(), b2.Event()
    e0.record(stream.h)
    graph.launch()
    e1.record(stream.h)
    stream.synchronize()
    ms = e0.elapsed_ms(e1) / steps
    nbytes = kv_bytes + n_seq * ATTN_HEADS * ATTN_HD * 8
    # KV shift: positions [1024, 4096) of every sequence rotated by -1024 (K read + write)
    def shift(i, s):
        for sq in range(n_seq):
            b2.check(b2.lib.b2_kv_shift_k_typed(ks[i % copies].ptr, kv_type, sq, ATTN_KV, ATTN_HD, ATTN_CTX, 1024,
                                                ATTN_CTX, -1024, 10000.0, s), "kv_shift_k")
    shift(0, stream.h)
    sg = b2.Graph(stream, lambda s: [shift(i, s) for i in range(max(1, steps // 4))])
    sg.launch()
    stream.synchronize()
    e0.record(stream.h)
    sg.launch()
    e1.record(stream.h)
    stream.synchronize()
    ms_shift = e0.elapsed_ms(e1) / max(1, steps // 4)
    shift_bytes = n_seq * 2 * (ATTN_CTX - 1024) * ATTN_KV * rb
    return {"batch": n_seq, "kv_type": {b2.Q8_0: "q8_0", b2.Q4_0: "q4_0"}.get(kv_type, "f16"), "ms": ms, "gbs": nbytes / (ms * 1e-3) / 1e9, "bytes": nbytes, "copies": copies,
            "shift_ms": ms_shift, "shift_gbs": shift_bytes / (ms_shift * 1e-3) / 1e9, "shift_bytes": shift_bytes}


def run_attn_ours(args, dist, rank, world, local):
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    batches = (1, 4, 16) if args.attn_batch is None else (args.attn_batch,)
    want = lambda t: args.attn_kv in ("all", t) or (args.attn_kv == "both" and t in ("f16", "q8_0"))
    res = [attn_measure(b2, n, args.steps) for n in batches] if want("f16") else []
    # Milda's default cache type (Q8_0 K and V) and its other one (Q4_0), the same batches
    res_q8 = [attn_measure(b2, n, args.steps, b2.Q8_0) for n in batches] if want("q8_0") else []
    res_q4 = [attn_measure(b2, n, args.steps, b2.Q4_0) for n in batches] if want("q4_0") else []
    peaks = measured_peaks()
    big = (res or res_q8 or res_q4)[-1]
    kvn = {"f16": "fp16", "q8_0": "Q8_0", "q4_0": "Q4_0"}[big["kv_type"]]
    return {"metric": f"decode attention HBM GB/s (32 q / 8 kv heads, hd 128, ctx 4096, {kvn} KV)",
            "value": round(big["gbs"] * world, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": 2,
            "ms_per_step": big["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"{kvn} KV, fp32 math",
            "data": "synthetic, seed 4: q N(0,1); fp16 K, V N(0,1); Q8_0 K, V uniform codes, block scale 0.01",
            "config": {"workload": f"attn_decode batch {big['batch']}, ctx 4096 (config 3); all batches in 'batches'",
                       "l2": "inputs larger than L2 (rotating KV copies)"},
            "roofline": {"bound": "hbm", "achieved": round(big["gbs"], 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(big["gbs"] / peaks["hbm_gbs"], 4), "traffic": None, "peak_src": peaks["src"],
                         "algorithmic_bytes_per_launch": big["bytes"]},
            "batches": [{k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()} for r in res],
            "batches_q8_0": [{k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()} for r in res_q8],
            "batches_q4_0": [{k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()} for r in res_q4],
            "gpu_launches": args.steps * 3}


# ------------------------------------------------------------------------------------------
# Workload: quantized prefill GEMM on the tensor cores (config 2)
# ------------------------------------------------------------------------------------------
GEMM_N, GEMM_K, GEMM_T = 11008, 4096, 512
GEMM_FLOP = 2 * GEMM_N * GEMM_K * GEMM_T
GEMM_REF_TOKENS = 8          # tokens per reference-arm step (a bounded sample of the 512)


GEMM_QTYPE = {"gemm_q4k": (12, "Q4_K", "q4_k x q8_k -> f16 exact integers -> f32 (TMEM)"),
              "gemm_q8_0": (8, "Q8_0", "q8_0 x q8_0 -> s32 (TMEM) -> f32")}


def gemm_inputs(b2, qt):
    w = b2.synth_normal(2, GEMM_N * GEMM_K, std=0.02).reshape(GEMM_N, GEMM_K)
    q = b2.quantize_weights(qt, w)
    x = b2.synth_normal(3, GEMM_T * GEMM_K).reshape(GEMM_T, GEMM_K)
    return q, x


def cpu_gemm_rate(q, x, seconds: float | None, n_tok: int | None, nt: int, qt: int) -> tuple[float, int]:
    """Oracle (reference-order) matmul of whole tokens on nt host threads:
    returns (seconds per token, tokens done)."""
    from oracle import oracle as O
    xq = O.quantize_act(qt, x[:1])
    O.matmul(qt, q, GEMM_N, GEMM_K, xq[0], nt)
    n, t0 = 0, time.perf_counter()
    while (n_tok is not None and n < n_tok) or (seconds is not None and time.perf_counter() - t0 < seconds):
        xq = O.quantize_act(qt, x[n % GEMM_T:n % GEMM_T + 1])
        O.matmul(qt, q, GEMM_N, GEMM_K, xq[0], nt)
        n += 1
    return (time.perf_counter() - t0) / n, n


def run_gemm_ours(args, dist, rank, world, local):
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    qt, qname, qdtype = GEMM_QTYPE[args.workload]
    q, x = gemm_inputs(b2, qt)
    wb = q.nbytes
    copies = max(2, -(-300_000_000 // wb))               # rotating W copies, > 2x L2
    mats = [b2.QMatrix(qt, q, GEMM_N, GEMM_K) for _ in range(copies)]
    xd = b2.DeviceBuffer.from_array(x)
    yd = b2.DeviceBuffer(GEMM_T * GEMM_N * 4)
    st = b2.DeviceBuffer.from_array(np.zeros(1, np.int32))
    ws = b2.DeviceBuffer(mats[0].gemm_workspace_bytes(GEMM_T))
    stream = b2.Stream()

    def step(i, s):
        mats[i % copies].gemm_device(xd, GEMM_T, yd, st, s, ws)

    for i in range(max(args.warmup, 3)):
        step(i, stream.h)
    stream.synchronize()
    graph = b2.Graph(stream, lambda s: [step(i, s) for i in range(args.steps)])
    graph.launch()
    stream.synchronize()
    e0, e1 = b2.Event(), b2.Event()
    barrier(dist)
    with ClockSampler(local) as clk:
        t_end = time.time() + 0.4
        while time.time() < t_end:
            graph.launch()
            stream.synchronize()
        e0.record(stream.h)
        graph.launch()
        e1.record(stream.h)
        stream.synchronize()
    ms_step = dist_max(dist, e0.elapsed_ms(e1) / args.steps)
    code = int(st.download(np.int32)[0])
    if code:
        raise RuntimeError(f"gemm pipeline wait expired (code {code})")
    tflops = GEMM_FLOP / (ms_step * 1e-3) / 1e12

    # e2e: X from pinned host memory, Y back to pinned host memory, inside the timed region
    xh = b2.PinnedArray.from_array(x)
    yh = b2.PinnedArray((GEMM_T, GEMM_N))
    n_e2e = max(5, min(args.steps, 50))
    for _ in range(2):
        mats[0].gemm(xh.array, yh.array)
    t0 = time.perf_counter()
    for _ in range(n_e2e):
        mats[0].gemm(xh.array, yh.array)
    e2e_s = dist_max(dist, (time.perf_counter() - t0) / n_e2e)
    peaks = measured_peaks()
    out = {
        "metric": f"{qname} prefill GEMM TFLOP/s (W 11008x4096, X 512x4096)",
        "value": round(tflops * world, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": qdtype,
        "data": f"synthetic: W N(0,0.02) seed 2 -> GGUF {qname}; X N(0,1) seed 3",
        "config": {"workload": f"{args.workload} 11008x4096 x 512 tokens (config 2)", "rotating_weight_copies": copies,
                   "l2": f"inputs larger than L2 ({copies} rotating W copies, {copies * wb / 1e6:.0f} MB)",
                   "replicas": world},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 2), "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": round(tflops / peaks["bf16_tflops"], 4), "traffic": None,
                     "peak_src": peaks["src"] + " bf16 burst", "algorithmic_flop_per_launch": GEMM_FLOP},
        "e2e": {"value": round(GEMM_FLOP * world / e2e_s / 1e12, 3), "unit": "TFLOP/s",
                "h2d_bytes_per_step": GEMM_T * GEMM_K * 4, "d2h_bytes_per_step": GEMM_T * GEMM_N * 4},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and args.cpu_seconds > 0:
        nt = os.cpu_count() or 1
        per_tok, n = cpu_gemm_rate(q, x, args.cpu_seconds, None, nt, qt)
        out["cpu_baseline"] = {"value": round(2 * GEMM_N * GEMM_K / per_tok / 1e12, 5), "unit": "TFLOP/s",
                               "cores": nt, "kind": "port",
                               "sample": f"{n} tokens (activation quantize + 11008 row vec_dots) in {args.cpu_seconds:.0f} s"}
    return out


def run_gemm_reference(args, dist, rank, world, local):
    if rank != 0:
        return None
    import b2gguf as b2  # host-only helpers (quantizer, generator)
    qt, qname, _ = GEMM_QTYPE[args.workload]
    q, x = gemm_inputs(b2, qt)
    nt = os.cpu_count() or 1
    cpu_gemm_rate(q, x, None, max(1, args.warmup), nt, qt)
    per_tok, n = cpu_gemm_rate(q, x, None, GEMM_REF_TOKENS * args.steps, nt, qt)
    v = round(2 * GEMM_N * GEMM_K / per_tok / 1e12, 5)
    return {"metric": f"{qname} prefill GEMM TFLOP/s (W 11008x4096, X 512x4096)", "value": v, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": per_tok * GEMM_REF_TOKENS * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": f"{qname.lower()} x q8 -> int32 -> f32", "data": "synthetic",
            "config": {"workload": f"{args.workload} 11008x4096 x 512 tokens (config 2)"}, "impl": "reference",
            "cpu_baseline": {"value": v, "unit": "TFLOP/s", "cores": nt, "kind": "port",
                             "sample": f"{n} of the 512 tokens ({GEMM_REF_TOKENS} per step) on {nt} host threads"},
            "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


TYPE_NAMES = {"q4_0": 2, "q8_0": 8, "q4_k": 12, "q6_k": 14}


def run_gemv_op(args, dist, rank, world, local):
    """One GEMV shape (--qtype/--rows/--cols/--batch) timed alone: the
    profiling target for a projection of the decode step."""
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    r = time_gemv_shape(b2, TYPE_NAMES[args.qtype], args.rows, args.cols, args.batch, args.steps, 7)
    peaks = measured_peaks()
    gbs = dist_max(dist, r["ms"])
    gbs = r["bytes"] * world / (gbs * 1e-3) / 1e9
    return {"metric": f"{args.qtype} GEMV HBM GB/s ({args.rows}x{args.cols}, batch {args.batch})",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": 3,
            "ms_per_step": r["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": f"{args.qtype} x q8 -> int32 -> f32", "data": "synthetic: W N(0,0.02) seed 7, x N(0,1) seed 8",
            "config": {"workload": f"gemv_op {args.qtype} {args.rows}x{args.cols} batch {args.batch}",
                       "rotating_weight_copies": r["copies"], "l2": "inputs larger than L2 (rotating copies)"},
            "roofline": {"bound": "hbm", "achieved": round(r["gbs"], 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(r["gbs"] / peaks["hbm_gbs"], 4), "traffic": None, "peak_src": peaks["src"],
                         "algorithmic_bytes_per_launch": r["bytes"]},
            "gpu_launches": args.steps}


# MoE FFN layers of the MoE GGUFs the engines load (their ffn_*_exps tensors):
# name -> (n_embd, expert FFN, experts, experts used)
MOE_SHAPES = {"qwen3_moe_30b_a3b": (2048, 768, 128, 8), "mixtral_8x7b": (4096, 14336, 8, 2)}


def moe_measure(b2, name: str, steps: int) -> dict:
    """One token through one routed FFN layer, batch 1 (the decode case):
    router GEMV (Q8_0), routing, gate and up grouped expert GEMVs (Q4_K), the
    down grouped GEMV over per-expert inputs, and the weighted combination;
    CUDA events over a graph of `steps` tokens.  Each token has its own
    input (its own experts), and the layer's expert stacks are rotated over
    copies larger than L2.  (The SiLU·mul between up and down is left out:
    the down GEMV reads the gate outputs, same bytes.)"""
    d, ff, ne, nu = MOE_SHAPES[name]
    stack_bytes = 3 * ne * ff * (d // 256) * 144
    copies = max(2, -(-300_000_000 // stack_bytes))
    def mk(seed, rows, k):   # one expert's weights, repeated for every expert of the stack (timing only)
        one = b2.quantize_weights(b2.Q4_K, b2.synth_normal(seed, rows * k, std=0.02).reshape(rows, k))
        return np.tile(one, (ne, 1))

    g, u, dn = mk(31, ff, d), mk(32, ff, d), mk(33, d, ff)
    router = b2.quantize_weights(b2.Q8_0, b2.synth_normal(34, ne * d, std=0.05).reshape(ne, d))
    layers = [(b2.QMatrix(b2.Q4_K, g, ne * ff, d), b2.QMatrix(b2.Q4_K, u, ne * ff, d),
               b2.QMatrix(b2.Q4_K, dn, ne * d, ff), b2.QMatrix(b2.Q8_0, router, ne, d)) for _ in range(copies)]
    n_x = 64
    xs = b2.DeviceBuffer.from_array(b2.synth_normal(35, n_x * d).reshape(n_x, d))
    lg, ids, wts = b2.DeviceBuffer(ne * 4), b2.DeviceBuffer(nu * 4), b2.DeviceBuffer(nu * 4)
    gy, uy = b2.DeviceBuffer(nu * ff * 4), b2.DeviceBuffer(nu * ff * 4)
    dy, out = b2.DeviceBuffer(nu * d * 4), b2.DeviceBuffer(d * 4)
    stream = b2.Stream()

    def one(i, s):
        mg, mu, md, mr = layers[i % copies]
        x = xs.ptr + (i % n_x) * d * 4
        b2.check(b2.lib.b2_gemv(mr.h, x, 1, lg.ptr, s), "router gemv")
        b2.check(b2.lib.b2_moe_route(lg.ptr, 1, ne, nu, 1, ids.ptr, wts.ptr, s), "moe_route")
        b2.check(b2.lib.b2_moe_gemv(mg.h, ne, x, 0, 1, ids.ptr, nu, gy.ptr, s), "moe gate")
        b2.check(b2.lib.b2_moe_gemv(mu.h, ne, x, 0, 1, ids.ptr, nu, uy.ptr, s), "moe up")
        b2.check(b2.lib.b2_moe_gemv(md.h, ne, gy.ptr, 1, 1, ids.ptr, nu, dy.ptr, s), "moe down")
        b2.check(b2.lib.b2_moe_combine(dy.ptr, wts.ptr, 1, nu, d, out.ptr, s), "moe_combine")

    for i in range(2 * copies):
        one(i, stream.h)
    graph = b2.Graph(stream, lambda s: [one(i, s) for i in range(steps)])
    graph.launch()
    stream.synchronize()
    e0, e1 = b2.Event(), b2.Event()
    e0.record(stream.h)
    graph.launch()
    e1.record(stream.h)
    stream.synchronize()
    ms = e0.elapsed_ms(e1) / steps
    expert_bytes = nu * 3 * ff * (d // 256) * 144
    nbytes = expert_bytes + ne * (d // 32) * 34
    return {"layer": name, "n_embd": d, "expert_ffn": ff, "experts": ne, "used": nu, "us_per_token": ms * 1e3,
            "bytes_per_token": nbytes, "gbs": nbytes / (ms * 1e-3) / 1e9, "copies": copies,
            "launches_per_token": 5 + (2 * nu if ff * 4 > 32 * 1024 else 1)}


def run_moe_ours(args, dist, rank, world, local):
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    res = [moe_measure(b2, n, args.steps) for n in MOE_SHAPES]
    peaks = measured_peaks()
    q = res[0]
    return {"metric": "MoE FFN layer decode HBM GB/s (Qwen3-MoE-like: d 2048, 128 experts of 768, top-8, Q4_K)",
            "value": round(q["gbs"] * world, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": 3,
            "ms_per_step": q["us_per_token"] / 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q4_k experts, q8_0 router x q8 -> int32 -> f32",
            "data": "synthetic: W N(0,0.02) seeds 31-34, x N(0,1) seed 35 (64 inputs, their own experts)",
            "config": {"workload": "moe: one routed FFN layer per token, batch 1; all shapes in 'layers'",
                       "l2": "inputs larger than L2 (rotating expert stacks)"},
            "roofline": {"bound": "hbm", "achieved": round(q["gbs"], 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": round(q["gbs"] / peaks["hbm_gbs"], 4), "traffic": None, "peak_src": peaks["src"],
                         "algorithmic_bytes_per_launch": q["bytes_per_token"]},
            "layers": [{k: (round(v, 4) if isinstance(v, float) else v) for k, v in r.items()} for r in res],
            "gpu_launches": args.steps * q["launches_per_token"]}


def run_sampler_ours(args, dist, rank, world, local):
    """One draw of Milda's sampler chain (penalties over 64, top-k 40, top-p
    0.9, min-p 0.05, temperature 0.75, dist) over a 128256-entry logits row
    on the device: b2_sampler_sample_logits per step (two kernels, the token
    read back), the penalty window full, host wall clock per draw."""
    import b2gguf as b2
    b2.check(b2.lib.b2_set_device(local), "set_device")
    path = model_path("sampler_tiny")
    b2.write_synthetic_llama(path, 1, 256, 512, 4, 2, 512, b2.Q8_0, embd_type=b2.Q8_0, out_type=b2.Q8_0, seed=3)
    m = b2.Model(path)
    ctx = b2.Context(m, n_ctx=32, n_seq=1)
    sm = b2.Sampler(ctx)
    nv = 128256
    rng = np.random.default_rng(5)
    rows = [b2.DeviceBuffer.from_array((rng.standard_normal(nv) * 3).astype(np.float32)) for _ in range(8)]
    for i in range(max(args.warmup, 3) + 64):
        sm.accept(sm.sample_logits(rows[i % 8].ptr, nv))
    t0 = time.perf_counter()
    for i in range(args.steps):
        sm.sample_logits(rows[i % 8].ptr, nv)
    us = (time.perf_counter() - t0) / args.steps * 1e6
    del sm, ctx, m
    os.remove(path)
    return {"metric": "sampler chain draw latency (128256-entry logits, Milda's chain)", "value": round(us, 2),
            "unit": "us", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": us / 1e3,
            "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "f32 logits",
            "data": "synthetic: logits N(0,3) seed 5, 8 rows rotating", "config": {"workload": "sampler"},
            "gpu_launches": 2 * args.steps, "timing": "host wall clock per b2_sampler_sample_logits (synchronous)"}


WORKLOADS = {"decode_8b_q4k": (run_decode_ours, run_decode_reference),
             "gemv_q4_0": (run_gemv_ours, run_gemv_reference),
             "decode_1b_q4_0": (run_decode1b_ours, None),
             "gemv_op": (run_gemv_op, None),
             "gemm_q4k": (run_gemm_ours, run_gemm_reference),
             "gemm_q8_0": (run_gemm_ours, run_gemm_reference),
             "attn": (run_attn_ours, None),
             "moe": (run_moe_ours, None),
             "sampler": (run_sampler_ours, None)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default 512 decode / 200 GEMV)")
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode_8b_q4k", choices=sorted(WORKLOADS))
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--keep-model", action="store_true", help="keep the synthetic GGUF file after the run")
    ap.add_argument("--skip-1b", action="store_true", help="decode_8b_q4k: leave out the 1.1B Q4_0 (config 4) line")
    ap.add_argument("--attn-batch", type=int, default=None, help="attn: one batch size (default 1, 4 and 16)")
    ap.add_argument("--attn-kv", default="all", choices=["all", "both", "f16", "q8_0", "q4_0"],
                    help="attn: KV cache types to time (default all; both = f16 and q8_0)")
    ap.add_argument("--profile-range", action="store_true",
                    help="open the profiler range around the timed decode steps only")
    ap.add_argument("--qtype", default="q4_k", choices=sorted(TYPE_NAMES), help="gemv_op weight type")
    ap.add_argument("--rows", type=int, default=28672, help="gemv_op output rows")
    ap.add_argument("--cols", type=int, default=4096, help="gemv_op input columns")
    ap.add_argument("--batch", type=int, default=8, help="gemv_op tokens per GEMV (1..8)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 512 if args.workload == "decode_8b_q4k" else 200
    dist, rank, world, local = dist_init()
    ours, ref = WORKLOADS[args.workload]
    if args.impl == "reference" and ref is None:
        out = {"impl": "reference", "unavailable": f"workload {args.workload} has no CPU reference arm"}
    else:
        out = (ref if args.impl == "reference" else ours)(args, dist, rank, world, local)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
