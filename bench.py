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
                                          "--format=csv,noheader,nounits", "-lms", "20"],
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
def host_threads() -> int:
    """Host cores this process may run on.  Set explicitly for the OpenMP C
    port: torchrun exports OMP_NUM_THREADS=1 to every rank."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


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
    threads = host_threads()
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
    threads = host_threads()
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
# the other configurations the metric names (1 GPU, rank 0)
# ---------------------------------------------------------------------------
def _time_graph(fn_launch, reps: int, calls_per_rep: int, stream) -> float:
    """Capture fn_launch() (calls_per_rep kernel calls) into a CUDA graph,
    replay it `reps` times after a warm-up; device microseconds per call."""
    import torch
    with torch.cuda.stream(stream):
        fn_launch()                       # warm-up outside capture
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn_launch()
    for _ in range(3):
        g.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    stream.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / (reps * calls_per_rep)


def _q4_on_gpu(rows: int, cols: int, seed: int, dev):
    import torch

    from alveare_b200 import q4_quantize
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = torch.randn((rows, cols), generator=g, device=dev, dtype=torch.float32).mul_(0.02)
    out = q4_quantize(w)
    del w
    return out


EXTRA_CASES = ("config1", "config2", "config5", "config3")


def extra_configs(device: int, only: str | None = None, trace: bool = False) -> dict:
    """BASELINE configs 1, 2 and 5 plus the decode-batch sweep, each through
    the library's C ABI on weights rotated over more distinct copies than L2
    holds (>= 4 x 126 MB), so every call streams its weights from HBM, and
    config 3 (Llama decode).  `only` runs one of EXTRA_CASES (config5
    includes the sweep)."""
    import torch

    from alveare_b200 import _lib
    dev = torch.device("cuda", device)
    st = torch.cuda.Stream(device=dev)
    ctx = _lib.context(device)
    peak = load_peaks()["hbm_gbs"]
    out = {}

    def want(case: str) -> bool:
        return only is None or only == case

    if want("config1"):
        out.update(_config1(ctx, dev, st, peak))
    if want("config2"):
        out.update(_config2(ctx, dev, st, peak))
    if want("config5"):
        out.update(_config5(ctx, dev, st, peak))
    torch.cuda.synchronize(dev)
    if want("config3"):
        out["config3_llama32_1b_greedy_decode"] = llama_decode(device, trace=trace)
    return out


def _config1(ctx, dev, st, peak) -> dict:
    import torch

    from alveare_b200 import Q4Weight, _lib
    # gemv 6912 x 1152, fp32 x and y, 128 weight copies (573 MB)
    lib, sp, device, out = ctx.lib, st.cuda_stream, dev.index, {}
    N1, K1, C1 = 6912, 1152, 128
    ws = [Q4Weight(_q4_on_gpu(N1, K1, 10_000 + i, dev), N=N1, K=K1, device=device) for i in range(C1)]
    x = torch.randn(K1, device=dev)
    y = torch.empty(N1, device=dev)

    def gemv_all():
        for w in ws:
            ctx.check(lib.alv_gemv(ctx.ptr, w.handle, 1, x.data_ptr(), _lib.F32, y.data_ptr(), _lib.F32, sp), "gemv")
    us = _time_graph(gemv_all, 10, C1, st)
    b1 = N1 * K1 // 32 * 18 + K1 * 4 + N1 * 4
    out["config1_gemv_6912x1152"] = {"us_per_call": round(us, 3), "gbs": round(b1 / us / 1e3, 1),
                                     "frac_of_hbm": round(b1 / us / 1e3 / peak, 4), "bytes_per_call": b1,
                                     "rotation": f"{C1} weight copies, {C1 * N1 * K1 // 32 * 18 / 1e6:.0f} MB"}
    for w in ws:
        w.free()
    return out


def _config2(ctx, dev, st, peak) -> dict:
    import torch

    from alveare_b200 import FusedFFNWeight, _lib
    lib, sp, device, out = ctx.lib, st.cuda_stream, dev.index, {}
    # Gemma-3-1B FFN 1152 x 6912, GeGLU, fp32 x and y, 128 copies (1.72 GB)
    H2, I2, C2 = 1152, 6912, 128
    fs = []
    for i in range(C2):
        g_, u_, d_ = (_q4_on_gpu(r, c, 20_000 + 3 * i + m, dev) for m, (r, c) in enumerate(((I2, H2), (I2, H2), (H2, I2))))
        fs.append(FusedFFNWeight(g_, u_, d_, H2, I2, "gelu", device=device))
        del g_, u_, d_
    x2 = torch.randn(H2, device=dev)
    y2 = torch.empty(H2, device=dev)

    def ffn_all():
        for f in fs:
            ctx.check(lib.alv_ffn(ctx.ptr, f.handle, 1, x2.data_ptr(), _lib.F32, y2.data_ptr(), _lib.F32, sp), "ffn")
    us = _time_graph(ffn_all, 10, C2, st)
    b2 = 3 * H2 * I2 // 32 * 18 + H2 * 8
    out["config2_ffn_1152x6912_geglu"] = {"us_per_call": round(us, 3), "gbs": round(b2 / us / 1e3, 1),
                                          "frac_of_hbm": round(b2 / us / 1e3 / peak, 4), "bytes_per_call": b2,
                                          "rotation": f"{C2} FFN copies, {C2 * b2 / 1e9:.2f} GB"}
    for f in fs:
        f.free()
    return out


def _config5(ctx, dev, st, peak) -> dict:
    import torch

    from alveare_b200 import Q4Weight, _lib
    lib, sp, device, out = ctx.lib, st.cuda_stream, dev.index, {}
    # prefill gemm 512 x 3840 x 15360 (tcgen05) and the decode-batch sweep on
    # the same shape, 8 weight copies (265 MB)
    N5, K5, B5, C5 = 15360, 3840, 512, 8
    ws = [Q4Weight(_q4_on_gpu(N5, K5, 30_000 + i, dev), N=N5, K=K5, device=device) for i in range(C5)]
    X = torch.randn((B5, K5), device=dev).to(torch.bfloat16)
    Y = torch.empty((B5, N5), device=dev)

    def gemm_all():
        for w in ws:
            ctx.check(lib.alv_gemm(ctx.ptr, w.handle, B5, X.data_ptr(), Y.data_ptr(), _lib.F32, sp), "gemm")
    us = _time_graph(gemm_all, 10, C5, st)
    flop = 2 * B5 * K5 * N5
    out["config5_prefill_gemm_512x3840x15360"] = {
        "us_per_call": round(us, 2), "tflops": round(flop / us / 1e6, 1),
        "frac_of_bf16_peak": round(flop / us / 1e6 / load_peaks_tc(), 4), "flop_per_call": flop,
        "rotation": f"{C5} weight copies, {C5 * N5 * K5 // 32 * 18 / 1e6:.0f} MB"}
    sweep = {}
    for B in (1, 2, 4, 8, 16):
        xb = torch.randn((B, K5), device=dev).to(torch.bfloat16)
        yb = torch.empty((B, N5), device=dev)

        def gemv_b(xb=xb, yb=yb, B=B):
            for w in ws:
                ctx.check(lib.alv_gemv(ctx.ptr, w.handle, B, xb.data_ptr(), _lib.BF16, yb.data_ptr(), _lib.F32, sp),
                          "gemv")
        us = _time_graph(gemv_b, 20, C5, st)
        bb = N5 * K5 // 32 * 18 + B * (K5 * 2 + N5 * 4)
        sweep[str(B)] = {"us_per_call": round(us, 2), "gbs": round(bb / us / 1e3, 1),
                         "frac_of_hbm": round(bb / us / 1e3 / peak, 4), "tokens_per_s": round(B / us * 1e6, 1)}
    out["decode_batch_sweep_15360x3840"] = sweep
    for w in ws:
        w.free()
    return out


LLAMA_PHASES = ((0, "layer start"), (1, "residual + attention norm"), (2, "qkv streamed"),
                (3, "qkv reduced + grid barrier"), (4, "rope + attention"), (5, "grid barrier after attention"),
                (6, "attention output staged"), (14, "o streamed"), (15, "o reduced"), (7, "grid barrier after o"),
                (8, "residual + ffn norm"), (9, "gate/up streamed"), (10, "gate/up reduced + grid barrier"),
                (11, "act staged"), (12, "down streamed"), (13, "down reduced + grid barrier"))


def llama_decode(device: int, steps: int = 256, n_prompt: int = 128, trace: bool = False) -> dict:
    """Llama-3.2-1B shape, random-init Q4 weights (N(0,
    0.02), quantized on the GPU; K/V padding rows zero as on disk), a
    128-token random prompt, then `steps` greedy tokens; tokens/s of the
    device-side greedy loop (one CUDA graph per step) and the Q4 bytes a
    token streams."""
    import torch

    from alveare_b200.llama import LlamaConfig, LlamaDecoder
    dev = torch.device("cuda", device)
    cfg = LlamaConfig.llama32_1b(max_seq=n_prompt + steps)
    H, Iw, V = cfg.hidden, cfg.intermediate, cfg.vocab
    kv = cfg.kv_heads * cfg.head_dim
    Vp = (V + 2047) // 2048 * 2048
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    emb = torch.randn((V, H), generator=g, device=dev).mul_(0.02).half()
    lm = torch.zeros((Vp, H), device=dev)
    lm[:V] = emb.float()
    w = {"token_embd": emb, "output_norm.weight": torch.ones(H, device=dev), "lm_head_packed": q4_quantize_dev(lm)}
    del lm
    shapes = {"attn_q": (H, H, H), "attn_k": (H, H, kv), "attn_v": (H, H, kv), "attn_output": (H, H, H),
              "ffn_gate": (Iw, H, Iw), "ffn_up": (Iw, H, Iw), "ffn_down": (H, Iw, H)}
    weight_bytes = Vp * H // 32 * 18
    for l in range(cfg.layers):
        w[f"blk.{l}.attn_norm.weight"] = torch.ones(H, device=dev)
        w[f"blk.{l}.ffn_norm.weight"] = torch.ones(H, device=dev)
        for p, (rows, cols, real) in shapes.items():
            m = torch.zeros((rows, cols), device=dev)
            m[:real] = torch.randn((real, cols), generator=g, device=dev).mul_(0.02)
            w[f"blk.{l}.{p}.weight_packed"] = q4_quantize_dev(m)
            weight_bytes += real * cols // 32 * 18   # the padding rows are not streamed
            del m
    prompt = torch.randint(0, V, (n_prompt,), generator=torch.Generator().manual_seed(78)).tolist()
    st = torch.cuda.current_stream(dev)

    def timed(per_kernel_step: int):
        cfg.per_kernel_step = per_kernel_step
        dec = LlamaDecoder(w, cfg, device=device)
        for _ in range(2):   # warm-up (graph capture on the first)
            dec.start(prompt)
            dec.run(n_prompt - 1, 8)
        dec.start(prompt)
        dec.run(n_prompt - 1, 0)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        st.synchronize()
        e0.record(st)
        dec.run(0, steps)
        e1.record(st)
        st.synchronize()
        us_tok = e0.elapsed_time(e1) * 1e3 / steps
        toks = dec.tokens(n_prompt, steps)
        one = dec.one_launch()
        # batched prefill of the prompt's first n_prompt - 1 positions
        dec.start(prompt)
        dec.prefill(0, n_prompt - 1)
        dec.start(prompt)
        st.synchronize()
        e0.record(st)
        dec.prefill(0, n_prompt - 1)
        e1.record(st)
        st.synchronize()
        prefill_ms = e0.elapsed_time(e1)
        phases = None
        if trace and one:  # the stamps of layer 1 of one step at position n_prompt + steps / 2
            ctx = dec.ctx
            tr = torch.zeros((ctx.info()["num_sms"], 16), dtype=torch.int64, device=dev)
            ctx.check(ctx.lib.alv_set_trace(ctx.ptr, tr.data_ptr()), "alv_set_trace")
            dec.forward(toks[steps // 2], n_prompt + steps // 2, return_logits=True)
            ctx.check(ctx.lib.alv_set_trace(ctx.ptr, None), "alv_set_trace")
            phases = trace_summary(tr.cpu().numpy().astype("float64"), LLAMA_PHASES)
        dec.free()
        return us_tok, toks, one, phases, prefill_ms

    us, toks, one, phases, prefill_ms = timed(0)
    us_sep, toks_sep, _, _, _ = timed(1)
    del w
    return {"us_per_token": round(us, 2), "tokens_per_s": round(1e6 / us, 1),
            "q4_bytes_per_token": weight_bytes, "gbs": round(weight_bytes / us / 1e3, 1),
            "frac_of_hbm": round(weight_bytes / us / 1e3 / load_peaks()["hbm_gbs"], 4),
            "launches_per_token": 1 if one else 7 * cfg.layers + 3,
            "separate_kernels_us_per_token": round(us_sep, 2), "same_tokens_as_separate_kernels": toks == toks_sep,
            "batched_prefill_ms": round(prefill_ms, 3), "batched_prefill_tokens_per_s": round((n_prompt - 1) / prefill_ms * 1e3, 1),
            "steps": steps, "prompt": n_prompt, "distinct_tokens": len(set(toks)),
            "l2": "695 MB of weights per token vs 126 MB L2",
            **({"phase_trace_us": phases} if phases else {})}


def q4_quantize_dev(w):
    from alveare_b200 import q4_quantize
    return q4_quantize(w)


def load_peaks_tc() -> float:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"])
    return 1590.0

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
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
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
    if args.trace:
        line["phase_trace_us"] = stack_phase_trace(stack, rank)
    if rank == 0 and world == 1 and not args.no_extras:
        line["other_configs"] = extra_configs(local)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = {k: v for k, v in cpu_baseline().items() if k != "s_per_layer"}
    stack.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


STACK_PHASES = ((0, "glue start"), (9, "down loaded"), (10, "down norm reduced"), (11, "x norm reduced"),
                (12, "xn written"), (1, "glue done"), (7, "gate/up streamed"), (2, "gate/up reduced + act"),
                (3, "grid barrier"), (4, "act staged"), (8, "down streamed"), (5, "down reduced (+ pushed)"),
                (6, "grid barrier (+ peer exchange)"))


def trace_summary(t, phases) -> dict:
    """Per-phase deltas (us) of the median over CTAs of alv_set_trace stamps."""
    import numpy as np
    base = float(np.median(t[:, phases[0][0]]))
    out, prev = {}, 0.0
    for i, name in phases:
        v = (float(np.median(t[:, i])) - base) / 1e3
        out[name] = round(v - prev, 2)
        prev = v
    out["total"] = round(prev, 2)
    return out


def stack_phase_trace(stack, rank: int) -> dict | None:
    """One more step with rank 0's per-CTA phase stamps on (alv_set_trace;
    the stack kernel stamps its second layer); every rank runs the step.
    Returns rank 0's per-phase breakdown of that layer."""
    import torch
    ctx = stack.ctx
    nsm = ctx.info()["num_sms"]
    tr = torch.zeros((nsm, 16), dtype=torch.int64, device=torch.device("cuda", stack.device))
    if rank == 0:
        ctx.check(ctx.lib.alv_set_trace(ctx.ptr, tr.data_ptr()), "alv_set_trace")
    stack.release()
    x = torch.zeros(H, dtype=torch.bfloat16).pin_memory()
    y = torch.empty_like(x).pin_memory()
    stack.forward(x, y)  # captures a new graph with the trace pointer
    if rank == 0:
        ctx.check(ctx.lib.alv_set_trace(ctx.ptr, None), "alv_set_trace")
        return trace_summary(tr.cpu().numpy().astype("float64"), STACK_PHASES)
    return None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the config 1/2/5 measurements")
    ap.add_argument("--trace", action="store_true",
                    help="add the per-phase breakdown of one layer (alv_set_trace stamps, rank 0) to the line")
    ap.add_argument("--case", choices=EXTRA_CASES, default=None,
                    help="run only this extra configuration (one GPU; for profiling captures) and print its JSON")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="stack depth (default 48, the benchmark workload; smaller only for profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps({"case": args.case, **extra_configs(0, args.case, args.trace)}), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
