#!/usr/bin/env python
"""Benchmark of the Q4 decode hot path.

Workload: a 12B-class FFN stack, batch-1 decode -- 48 layers, hidden 3840,
intermediate 15360, GeGLU, Q4 group-32 weights quantized from N(0, 0.02)
(synthetic, seeded; generated and quantized on the GPU).  One step = one
decode token through all 48 FFN half-blocks (rmsnorm -> fused FFN ->
rmsnorm -> residual).  With --gpus N (torchrun) each rank holds 1/N of the
intermediate dimension; the step is still one kernel launch per GPU, which
pushes each layer's partial down projection to the peer GPUs over NVLink and
sums the ranks' partials in rank order (no collective between layers).

Metric: achieved HBM GB/s of algorithmic bytes -- 18 B per
32 weights, activations counted once -- for the whole job; tokens/s is
reported beside it.  The 4.78 GB of weights exceed the 126 MB L2 by ~38x, so
no L2 flush is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
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
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "Q4 GEMV/FFN achieved HBM GB/s (% of peak); decode tokens/s at 1/2/4/8 GPUs"
H, I, LAYERS = 3840, 15360, 48
WEIGHT_BYTES_PER_LAYER = 3 * H * I // 32 * 18           # 99,532,800
ACT_BYTES_PER_LAYER = H * 2 + H * 4 + H * 4 + H * 2      # x in/out bf16, down in/out fp32
BYTES_PER_LAYER = WEIGHT_BYTES_PER_LAYER + ACT_BYTES_PER_LAYER


def workload_config(n_gpus: int, layers: int = LAYERS) -> dict:
    return {"workload": "12B-class FFN stack decode (BASELINE config 4)", "layers": layers, "hidden": H,
            "intermediate": I, "activation": "GeGLU", "quant": "Q4 group-32, 18 B/32 weights",
            "global_batch": 1, "tensor_parallel": n_gpus, "l2": "inputs > L2 (4.78 GB weights vs 126 MB L2)"}


def load_peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "source": "fallback"}


def profiled_traffic(kernel: str) -> float | None:
    """DRAM bytes per layer of `kernel` from its committed ncu summary
    (dram__bytes_read.sum + dram__bytes_write.sum of one captured launch
    divided by the layers that launch processed)."""
    p = os.path.join(ROOT, "profiles", f"{kernel}_12b_stack.md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("traffic_bytes_per_layer:"):
            return float(line.split(":", 1)[1].strip())
    return None


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline (the C restatement of the reference's CPU path)
# ---------------------------------------------------------------------------
def synthetic_cpu_layer(seed: int):
    """Random but well-formed packed Q4 matrices of the config-4 shapes (the
    CPU cost does not depend on the values)."""
    import numpy as np

    from oracle import q4
    rng = np.random.default_rng(seed)
    mats = []
    for rows, cols in ((I, H), (I, H), (H, I)):
        b = rng.integers(0, 256, size=(rows, cols // 32, 20), dtype=np.uint8)
        b[:, :, 16:18] = np.frombuffer(q4.bf16_bits(np.float32(0.004)).tobytes(), np.uint8)
        b[:, :, 18:] = 0
        mats.append(b.reshape(rows, cols // 32 * 20))
    return mats


def cpu_baseline(budget_s: float = 10.0) -> dict:
    """Time the C oracle's FFN half-block on all host threads over a bounded
    sample (about `budget_s` seconds of layers); GB/s of the same algorithmic
    bytes.  One layer's packed weights (110 MB) exceed the host's last-level
    cache, so repeating a layer costs what distinct layers would."""
    import numpy as np

    from oracle import cpu
    threads = cpu.max_threads()
    g, u, d = synthetic_cpu_layer(0)
    x = np.random.default_rng(1).normal(0, 1, H).astype(np.float32)
    cpu.ffn_block(g, u, d, x, threads)  # warm-up
    t0 = time.perf_counter()
    n = 0
    while True:
        x = cpu.ffn_block(g, u, d, x, threads)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    return {"value": round(BYTES_PER_LAYER * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"{n} FFN half-blocks (H=3840, I=15360, GeGLU; {n / LAYERS:.1f} decode steps of the 48-layer "
                      f"stack) through the C port of the reference CPU path, OpenMP over {threads} threads, "
                      f"{dt:.2f} s",
            "s_per_layer": dt / n}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    from oracle import cpu
    threads = cpu.max_threads()
    g, u, d = synthetic_cpu_layer(0)
    x = np.random.default_rng(1).normal(0, 1, H).astype(np.float32)
    layers_per_step = args.layers   # a whole decode step: every FFN half-block of the stack
    for _ in range(args.warmup):
        x = cpu.ffn_block(g, u, d, x, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _ in range(layers_per_step):
            x = cpu.ffn_block(g, u, d, x, threads)
    dt = time.perf_counter() - t0
    value = BYTES_PER_LAYER * layers_per_step * args.steps / dt / 1e9
    sample = (f"each step = all {layers_per_step} FFN half-blocks (H=3840, I=15360, GeGLU) of one decode token "
              f"through the C port of the reference CPU path, OpenMP over {threads} threads")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "q4/bf16/f32",
            "data": "synthetic", "config": workload_config(1, args.layers),
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "tokens_per_s": round(args.steps / dt, 4)}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def build_stack(stack, layers: int, seed: int = 1234):
    import torch

    from alveare_b200 import q4_quantize
    dev = torch.device("cuda", stack.device)
    g = torch.Generator(device=dev)
    for l in range(layers):
        mats = []
        for m, (rows, cols) in enumerate(((I, H), (I, H), (H, I))):
            g.manual_seed(seed + 3 * l + m)
            w = torch.randn((rows, cols), generator=g, device=dev, dtype=torch.float32).mul_(0.02)
            mats.append(q4_quantize(w))
            del w
        stack.add_layer(*mats)
        del mats
    torch.cuda.synchronize(dev)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from alveare_b200.stack import FFNStack

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    stack = FFNStack(H, I, device=local, rank=rank, world=world)
    build_stack(stack, args.layers)
    if world > 1:
        t = torch.ones(1, device="cuda")
        dist.all_reduce(t)  # warm the communicator before graph capture
        torch.cuda.synchronize()

    # ---- steady-state device throughput (graph replay) ----
    stack.prepare()
    step_launches = stack.launches
    s = stack.stream
    for _ in range(args.warmup):
        stack.replay()
    s.synchronize()
    # start the clock sampler before the barrier: no rank may be held up
    # inside the timed region by another rank's host-side work
    clocks = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(args.steps):
            stack.replay()
        e1.record(s)
    s.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    clock_info = clocks.stop() if clocks else None
    t = torch.tensor([ms], device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    ms_step = ms_total / args.steps
    stack.ctx.sync_status(s.cuda_stream)

    # ---- dominant kernel alone ----
    if stack.fused:
        # one ffn_stack_kernel launch is the whole step
        kernel, kernel_layers, kernel_us = "ffn_stack_kernel", args.layers, ms_step * 1e3
    else:
        # the per-layer ffn_kernel launches of a step, without the all-reduces
        g_layers = stack.capture(layers_only=True)
        for _ in range(2):
            g_layers.replay()
        s.synchronize()
        reps = max(2, args.steps)
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            k0.record(s)
            for _ in range(reps):
                g_layers.replay()
            k1.record(s)
        s.synchronize()
        kernel, kernel_layers = "ffn_kernel", 1
        kernel_us = k0.elapsed_time(k1) * 1e3 / (reps * args.layers)
        del g_layers

    # ---- end to end through the public API with host buffers ----
    x_host = torch.zeros(H, dtype=torch.bfloat16).pin_memory()
    x_host.normal_()
    y_host = torch.empty(H, dtype=torch.bfloat16).pin_memory()
    for _ in range(2):
        stack.forward(x_host, y_host)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        stack.forward(x_host, y_host)
    e2e_s = (time.perf_counter() - t0) / args.steps
    te = torch.tensor([e2e_s], device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_s = float(te.item())

    total_bytes = BYTES_PER_LAYER * args.layers           # one token, all ranks together
    value = total_bytes / (ms_step * 1e-3) / 1e9
    peaks = load_peaks()
    per_launch_bytes = ((WEIGHT_BYTES_PER_LAYER // world) + ACT_BYTES_PER_LAYER) * kernel_layers
    achieved = per_launch_bytes / (kernel_us * 1e-6) / 1e9
    traffic = profiled_traffic(kernel)
    if traffic is not None:
        traffic = round(traffic * kernel_layers / world)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "q4 weights, bf16 dequant, fp32 accumulate",
        "data": "synthetic (seeded N(0,0.02) weights quantized on the GPU, random x)",
        "config": workload_config(world, args.layers),
        "tokens_per_s": round(1000.0 / ms_step, 2),
        "pct_of_hbm_peak": round(100.0 * value / (peaks["hbm_gbs"] * world), 2),
        "roofline": {"bound": "hbm", "kernel": kernel, "layers_per_launch": kernel_layers,
                     "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
                     "traffic": traffic, "launch_us": round(kernel_us, 3),
                     "bytes_per_launch": per_launch_bytes},
        "e2e": {"value": round(total_bytes / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": H * 2, "d2h_bytes_per_step": H * 2,
                "ms_per_step": round(e2e_s * 1e3, 4)},
        "gpu_launches": step_launches * args.steps,
        "clocks": clock_info,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = {k: v for k, v in cpu_baseline().items() if k != "s_per_layer"}
    stack.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="stack depth (default 48, the benchmark workload; smaller only for profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
