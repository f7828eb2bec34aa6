#!/usr/bin/env python
"""Benchmark of the AWQ hot path on B200 (one JSON line on rank 0).

Workload (M = 1): decode of one token through every
AWQ linear of a Llama-2-7B-shaped model -- 32 layers x {qkv 4096->12288,
o 4096->4096, gate_up 4096->22016, down 11008->4096}, group 128, f16
activations ~ N(0,1), f16 scales ~ U(0.001, 0.02), uniform random nibbles.
Every layer has its own weights (3.4 GB in total, far above the 126 MB L2),
so each step reads all weights cold from HBM. One step = the 128 fused GEMM
launches of one token, replayed as a CUDA graph.

  value  = weight bytes (packed + zeros + scales) of all linears / time, GB/s
  e2e    = the same through the public API (AWQGEMMLinear.forward) per step,
           with the step's activations copied host->device from pinned memory
           and the step's outputs copied back, inside the timed region
  roofline: the decode kernel's algorithmic bytes per launch / its average
           launch duration over the timed region (CUDA events on the stream
           the graph runs on; every launch in it is a decode kernel), against
           the measured HBM copy bandwidth of MEASURED_PEAKS.json
  cpu_baseline: the C restatement of the reference's arithmetic with F = f32
           (native float, vectorised, every host thread) on a bounded sample of
           the same workload; the same sample and threads as --impl reference

Keys at the end of the line (single-GPU runs):
  cfg0_decode: BASELINE configs[0], M = 1, 4096 x 4096, g 128, f32 x and f32
           scales, 24 rotated weight copies (L2 cold): us per launch, GB/s
  dequantize: the standalone dequantize kernel (natural order) on configs[0]
           (4096 x 4096 -> f32) and configs[4] (8192 x 57344 -> f16)
  prefill: BASELINE configs[2], the Llama-2-7B layer at M = 512 / 2048 / 8192
           (f16) and M = 2048 with f32 activations: us per layer, TFLOP/s,
           fraction of the measured dense bf16 peak
  tp_llama3_70b_mlp: BASELINE configs[4], the Llama-3-70B MLP sharded over
           the job's GPUs (gate_up 8192->57344 column-parallel, down
           28672->8192 row-parallel with an fp32 NCCL all-reduce) at M in
           {1, 8, 2048}: us per MLP (max over ranks), the same MLP unsharded on
           one GPU of the job, and the strong-scaling efficiency between them
Earlier keys: the decode M sweep, per-linear launch times, the Qwen2-7B M
sweep, the fused neighbours and the fused tensor-parallel
collectives against NCCL.

--workload prefill prints one line for the prefill measurement alone (for
profiling), --no-autotune uses the planner's default plans.

--impl reference runs the CPU restatement of the reference's arithmetic (the
reference itself is Rust/CubeCL on wgpu and cannot run on this machine) on the
host cores, on a bounded sample of the same workload.

With N GPUs (torchrun) every rank decodes its own model replica (weak
scaling, no data-path collective); ranks meet for the barrier and the
max-over-ranks timing, and then run the tensor-parallel configs[4] MLP
together (the layers' own collectives).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

LLAMA2_7B = [("qkv", 4096, 12288), ("o_proj", 4096, 4096), ("gate_up", 4096, 22016),
             ("down", 11008, 4096)]
GROUP = 128
METRIC = "AWQ GEMM decode M=1 HBM GB/s (Llama-2-7B AWQ linears, f16)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--rows", type=int, default=1)
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the M sweep, the prefill numbers and the CPU baseline")
    ap.add_argument("--no-autotune", action="store_true", help="use the default plans")
    ap.add_argument("--workload", choices=["decode", "prefill"], default="decode")
    ap.add_argument("--prefill-rows", type=int, default=2048)
    return ap.parse_args()


# ------------------------------------------------------------------ helpers
def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def weight_bytes(k, n, dtype_bytes=2):
    return k * n // 2 + (k // GROUP) * (n // 8) * 4 + (k // GROUP) * n * dtype_bytes


def measured_peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def profile_traffic():
    """dram bytes per decode launch from the committed ncu summary, if present."""
    path = os.path.join(REPO, "profiles", "decode_traffic.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap"}

    def __init__(self, index: int, period_s: float = 0.02):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], set()
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def run():
                while not self._stop.is_set():
                    try:
                        self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                        r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        for bit, name in self.REASONS.items():
                            if r & bit:
                                self.reasons.add(name)
                    except Exception:
                        pass
                    time.sleep(self.period)

            self._thread = threading.Thread(target=run, daemon=True)
            self._thread.start()
        except Exception:
            self._thread = None
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": sorted(self.reasons)}


# ------------------------------------------------------------- our arm
def run_ours(a, rank, local_rank, world):
    import torch
    import torch.distributed as dist

    import cube_awq_b200 as cawq
    from cube_awq_b200 import synth

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    rows, dt = a.rows, torch.float16
    layers = []
    for li in range(a.layers):
        lin = []
        for j, (name, k, n) in enumerate(LLAMA2_7B):
            w = synth.make_weights(k, n, GROUP, dt, dev, seed=(rank * 1000 + li) * 10 + j)
            layer = cawq.AWQGEMMLinear(w.qweight, w.qzeros, w.scales)
            lin.append((name, k, n, layer))
        layers.append(lin)
    xs = {name: synth.make_input(rows, k, dt, dev, seed=17 + j)
          for j, (name, k, n) in enumerate(LLAMA2_7B)}
    ys = {name: torch.empty(rows, n, dtype=dt, device=dev) for name, k, n in LLAMA2_7B}
    step_bytes = sum(weight_bytes(k, n) for _, k, n in LLAMA2_7B) * a.layers

    # one autotune per distinct shape (setup, untimed); plans are then cached
    plans = {}
    for name, k, n, layer in layers[0]:
        if a.no_autotune:
            plans[name] = cawq.plan_get(rows, k, n, GROUP, dt)
        else:
            plans[name] = cawq.autotune(xs[name], layer.qweight, layer.qzeros, layer.scales,
                                        GROUP, out=ys[name])

    def step():
        for lin in layers:
            for name, k, n, layer in lin:
                cawq.gemm(xs[name], layer.qweight, layer.qzeros, layer.scales, GROUP, out=ys[name])

    stream = torch.cuda.Stream(dev)
    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(graph, stream=stream):
            step()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(a.warmup):
        graph.replay()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches_per_step = a.layers * len(LLAMA2_7B)
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.nvtx.range_push("cawq_timed")
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(a.steps):
                graph.replay()
            e1.record(stream)
        e1.synchronize()
        torch.cuda.nvtx.range_pop()
        barrier()
    ms_local = e0.elapsed_time(e1) / a.steps
    ms = max_over_ranks(ms_local)
    value = step_bytes * world / (ms * 1e-3) / 1e9
    # roofline: every launch of the timed region is a decode kernel; its
    # average duration there (launches overlap only by their prologues)
    achieved = (step_bytes / launches_per_step) / (ms_local * 1e-3 / launches_per_step) / 1e9

    # ---- per-linear launches, each bracketed by events (diagnostic only)
    n_prof = max(1, min(a.steps, 20))
    evs = []
    cur = torch.cuda.current_stream(dev)
    for _ in range(n_prof):
        for lin in layers:
            for name, k, n, layer in lin:
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record(cur)
                cawq.gemm(xs[name], layer.qweight, layer.qzeros, layer.scales, GROUP, out=ys[name])
                s1.record(cur)
                evs.append((weight_bytes(k, n), s0, s1, name))
    torch.cuda.synchronize()
    per_name = {}
    for b, s0, s1, name in evs:
        per_name.setdefault(name, []).append(s0.elapsed_time(s1))
    peaks, peaks_kind = measured_peaks()
    traffic = profile_traffic()

    # ---- e2e: public API, host buffers, copies inside the timed region
    pin_x = {name: xs[name].cpu().pin_memory() for name in xs}
    pin_y = {name: torch.empty(rows, n, dtype=dt).pin_memory() for name, k, n in LLAMA2_7B}
    h2d = sum(t.numel() * t.element_size() for t in pin_x.values())
    d2h = sum(t.numel() * t.element_size() for t in pin_y.values())
    dx = {name: torch.empty_like(xs[name]) for name in xs}
    e2e_steps = max(1, min(a.steps, 50))

    def e2e_step():
        for name in dx:
            dx[name].copy_(pin_x[name], non_blocking=True)
        outs = {}
        for lin in layers:
            for name, k, n, layer in lin:
                outs[name] = layer.forward(dx[name])
        for name in pin_y:
            pin_y[name].copy_(outs[name], non_blocking=True)

    for _ in range(min(a.warmup, 3)):
        e2e_step()
    barrier()
    e0.record()
    for _ in range(e2e_steps):
        e2e_step()
    e1.record()
    e1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    e2e_val = step_bytes * world / (e2e_ms * 1e-3) / 1e9

    # ---- extras (single-GPU measurements only at N = 1; at N > 1 every rank
    # joins the tensor-parallel configs[4] measurement)
    extras = {}
    if not a.no_extras and world == 1:
        sweep = {}
        for m in (1, 2, 4, 8):
            xm = {name: synth.make_input(m, k, dt, dev, seed=5) for name, k, n in LLAMA2_7B}
            ym = {name: torch.empty(m, n, dtype=dt, device=dev) for name, k, n in LLAMA2_7B}
            g2 = torch.cuda.CUDAGraph()
            for lin in layers[:1]:
                for name, k, n, layer in lin:
                    cawq.autotune(xm[name], layer.qweight, layer.qzeros, layer.scales, GROUP, out=ym[name])
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g2, stream=stream):
                    for lin in layers:
                        for name, k, n, layer in lin:
                            cawq.gemm(xm[name], layer.qweight, layer.qzeros, layer.scales, GROUP,
                                      out=ym[name])
            for _ in range(3):
                g2.replay()
            torch.cuda.synchronize()
            reps = 20
            e0.record()
            for _ in range(reps):
                g2.replay()
            e1.record()
            e1.synchronize()
            t = e0.elapsed_time(e1) / reps
            sweep[str(m)] = {"us_per_token_step": round(t * 1e3, 2),
                             "gb_per_s": round(step_bytes / (t * 1e-3) / 1e9, 1)}
            del g2
        del layers
        torch.cuda.empty_cache()
        extras["fused_neighbours"] = fused_neighbour_numbers(dev)
        extras["qwen2_m_sweep"] = qwen2_sweep(dev)
        extras["crossover_sweep"] = crossover_sweep(dev)
        extras["decode_sweep_m"] = sweep
        extras["us_per_linear_isolated"] = {k: round(statistics.median(v) * 1e3, 2)
                                            for k, v in per_name.items()}
        extras["cfg0_decode"] = cfg0_decode_numbers(dev, peaks)
        extras["dequantize"] = dequant_numbers(dev, peaks)
        extras["prefill"] = prefill_sweep(dev, peaks)
    tp_keys = {}
    if not a.no_extras:
        if world > 1:
            del layers
            torch.cuda.empty_cache()
        try:  # every rank fails the same way (same calls, same sizes)
            tp_keys["tp_fused_collectives"] = tp_fused_numbers(dev, world, max_over_ranks)
        except Exception as exc:
            tp_keys["tp_fused_collectives"] = {"error": f"{type(exc).__name__}: {exc}"[:300]}
        tp_keys["tp_llama3_70b_mlp"] = tp_mlp_numbers(dev, world, max_over_ranks)

    if world > 1:
        # Every rank's work is done. The process group is left to process exit
        # (main() ends every rank with os._exit): NCCL logs its teardown on
        # stdout, and other ranks' lines would land after rank 0's JSON line.
        del graph
        torch.cuda.synchronize()
        dist.barrier()
    if rank != 0:
        return

    cpu = None if (a.no_extras or world > 1) else cpu_baseline()
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded; uniform nibbles, scales U(0.001,0.02), x N(0,1))",
        "config": workload_config(a, world),
        "tokens_per_s": round(world * 1e3 / ms, 1),
        "gpu_launches": a.steps * launches_per_step,
        "graph": "one CUDA graph per step (128 launches)",
        "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "api": "AWQGEMMLinear.forward x 128, no graph"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic, "peak_kind": peaks_kind,
                     "algorithmic_bytes_per_launch": step_bytes // launches_per_step,
                     "kernel": "cawq::decode_kernel, average over the timed region "
                               f"({launches_per_step} launches per step)"},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "plans": plans,
    }
    # bulky diagnostics first, the compact key numbers last (the end of the
    # line is what a truncated log keeps)
    for key in ("fused_neighbours", "qwen2_m_sweep", "crossover_sweep", "decode_sweep_m",
                "us_per_linear_isolated"):
        if key in extras:
            line[key] = extras.pop(key)
    if "tp_fused_collectives" in tp_keys:
        line["tp_fused_collectives"] = tp_keys.pop("tp_fused_collectives")
    line.update(extras)
    line.update(tp_keys)
    print(json.dumps(line), flush=True)


def workload_config(a, world):
    """The `config` of both arms' lines (the reference arm prints the same)."""
    return {"workload": "configs[1] decode M=1: Llama-2-7B AWQ linears x 32 layers, g128",
            "rows_m": a.rows, "layers": a.layers, "group_size": GROUP,
            "step_weight_bytes": sum(weight_bytes(k, n) for _, k, n in LLAMA2_7B) * a.layers,
            "l2": "cold (3.4 GB of distinct weights per step)",
            "parallelism": f"replica x{world} (weak, no data-path collective)"}


def cfg0_decode_numbers(dev, peaks, copies=24, reps=20):
    """BASELINE configs[0] as its own number: M = 1, K = N = 4096, g = 128,
    f32 x and f32 scales, no bias; `copies` seeded weight sets (24 x 9 MB,
    above the 126 MB L2) launched back to back from one graph, so each launch
    reads its weights from HBM. us per launch, weight bytes / us."""
    import torch

    import cube_awq_b200 as cawq
    from cube_awq_b200 import synth
    k = n = 4096
    dt = torch.float32
    ws = [synth.make_weights(k, n, GROUP, dt, dev, seed=600 + c) for c in range(copies)]
    x = synth.make_input(1, k, dt, dev, seed=601)
    y = torch.empty(1, n, dtype=dt, device=dev)
    stream = torch.cuda.Stream(dev)

    def run():
        for w in ws:
            cawq.gemm(x, w.qweight, w.qzeros, w.scales, GROUP, out=y)
    us = _graph_us(run, reps, stream) / copies
    nbytes = ws[0].nbytes()
    gbs = nbytes / (us * 1e-6) / 1e9
    plan = cawq.plan_get(1, k, n, GROUP, dt)
    del ws
    return {"us": round(us, 3), "gb_per_s": round(gbs, 1),
            "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4), "bytes": nbytes,
            "path": plan["path"], "l2": f"cold ({copies} rotated weight copies)"}


def prefill_sweep(dev, peaks):
    """the Llama-2-7B layer's 4 linears at M = 512, 2048,
    8192 (f16) and at M = 2048 with f32 activations and scales; per M the
    layer's us, TFLOP/s and fraction of the measured dense bf16 peak (f32:
    the same flops against the same peak), and TFLOP/s per linear."""
    import torch
    out = {}
    for m, dt, tag in ((512, torch.float16, "f16"), (2048, torch.float16, "f16"),
                       (8192, torch.float16, "f16"), (2048, torch.float32, "f32")):
        res = prefill_numbers(m, dt, dev, peaks, reps=5 if m >= 8192 or dt == torch.float32
                              else 10, copies=1 if m >= 2048 else 3)
        us = sum(r["us"] for r in res.values())
        fl = sum(2.0 * m * k * n for _, k, n in LLAMA2_7B)
        tf = fl / (us * 1e-6) / 1e12
        out[f"{tag}_M={m}"] = {"layer_us": round(us, 1), "tflops": round(tf, 1),
                               "frac": round(tf / peaks["bf16_tflops"], 4),
                               "per_linear_tflops": {nm: r["tflops"] for nm, r in res.items()},
                               "paths": sorted({r["path"] for r in res.values()})}
    return out


# ------------------------------------------------------------ prefill
def prefill_numbers(m, dt, dev, peaks, reps=10, copies=3):
    """configs[2] at M = m: TFLOP/s of each Llama-2-7B linear, graph-timed
    over `copies` distinct weight sets (flops = 2 M N K)."""
    import torch

    import cube_awq_b200 as cawq
    from cube_awq_b200 import synth
    out = {}
    stream = torch.cuda.Stream(dev)
    for j, (name, k, n) in enumerate(LLAMA2_7B):
        ws = [synth.make_weights(k, n, GROUP, dt, dev, seed=900 + 10 * j + c) for c in range(copies)]
        x = synth.make_input(m, k, dt, dev, seed=950 + j)
        y = torch.empty(m, n, dtype=dt, device=dev)
        plan = cawq.plan_get(m, k, n, GROUP, dt)

        def run():
            for w in ws:
                cawq.gemm(x, w.qweight, w.qzeros, w.scales, GROUP, out=y)
        us = _graph_us(run, reps, stream) / copies
        tflops = 2.0 * m * n * k / (us * 1e-6) / 1e12
        out[name] = {"us": round(us, 2), "tflops": round(tflops, 1),
                     "frac_of_measured_bf16_peak": round(tflops / peaks["bf16_tflops"], 4),
                     "path": plan["path"]}
        del ws, x, y
    return out


def _graph_us(fn, reps, stream):
    """Device time of one fn() replayed from a CUDA graph (us)."""
    import torch
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        with torch.cuda.graph(g, stream=stream):
            fn()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
    e1.synchronize()
    del g
    return e0.elapsed_time(e1) * 1e3 / reps


def dequant_numbers(dev, peaks, reps=20):
    """Standalone dequantize (natural order): configs[0] to f32 and configs[4]
    to f16. Bytes = packed weights + zeros + scales read + output written."""
    import torch

    import cube_awq_b200 as cawq
    from cube_awq_b200 import synth
    out = {}
    stream = torch.cuda.Stream(dev)
    for name, k, n, dt in (("cfg0_4096x4096_f32", 4096, 4096, torch.float32),
                           ("cfg4_8192x57344_f16", 8192, 57344, torch.float16)):
        w = synth.make_weights(k, n, GROUP, dt, dev, seed=700)
        o = torch.empty(k, n, dtype=dt, device=dev)
        us = _graph_us(lambda: cawq.dequantize_native(w.qweight, w.qzeros, w.scales, o, GROUP),
                       reps, stream)
        nbytes = w.nbytes() + k * n * o.element_size()
        gbs = nbytes / (us * 1e-6) / 1e9
        out[name] = {"us": round(us, 2), "gb_per_s": round(gbs, 1),
                     "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                     "bytes": nbytes, "l2": "output larger than L2" if k * n * o.element_size()
                     > 126e6 else "working set fits L2 (hot)"}
        del w, o
    return out


def qwen2_sweep(dev, reps=10):
    """Qwen2-7B AWQ linears, g = 64, f16, default plans; us per
    layer (4 launches, graph-timed, 3 weight copies rotated) per M."""
    import torch

    import cube_awq_b200 as cawq
    from cube_awq_b200 import synth
    shapes = (("qkv", 3584, 4608), ("o_proj", 3584, 3584), ("gate_up", 3584, 37888),
              ("down", 18944, 3584))
    g, dt, copies = 64, torch.float16, 3
    stream = torch.cuda.Stream(dev)
    ws = {name: [synth.make_weights(k, n, g, dt, dev, seed=800 + 10 * j + c) for c in range(copies)]
          for j, (name, k, n) in enumerate(shapes)}
    wbytes = sum(ws[name][0].nbytes() for name, _, _ in shapes)
    res = {}
    for m in (1, 2, 4, 8, 16, 64, 256, 1024, 4096):
        xs = {name: synth.make_input(m, k, dt, dev, seed=850) for name, k, n in shapes}
        ys = {name: torch.empty(m, n, dtype=dt, device=dev) for name, k, n in shapes}

        def layer_steps():
            for c in range(copies):
                for name, k, n in shapes:
                    w = ws[name][c]
                    cawq.gemm(xs[name], w.qweight, w.qzeros, w.scales, g, out=ys[name])
        us = _graph_us(layer_steps, reps, stream) / copies
        flops = sum(2.0 * m * k * n for _, k, n in shapes)
        paths = {name: cawq.plan_get(m, k, n, g, dt)["path"] for name, k, n in shapes}
        res[str(m)] = {"us_per_layer": round(us, 2),
                       "weight_gb_per_s": round(wbytes / (us * 1e-6) / 1e9, 1),
                       "tflops": round(flops / (us * 1e-6) / 1e12, 1),
                       "paths": sorted(set(paths.values()))}
        del xs, ys
    del ws
    return res


def crossover_sweep(dev, reps=10):
    """Where the decode / prefill crossover belongs: us per decoder layer
    (4 linears, f16, graph-timed, 3 weight copies rotated) of Llama-2-7B (g
    128) and Qwen2-7B (g 64) at M = 8 ... 64. Up to M = 16 both kernels run:
    the decode kernel with its default plan, and the 128-row prefill tile
    with the fastest split (1-8) per linear; above 16 only the prefill kernel
    applies (default plans). `planner` is the path the default planner takes."""
    import torch

    import cube_awq_b200 as cawq
    from cube_awq_b200 import synth
    models = {"llama2_7b": (128, (("qkv", 4096, 12288), ("o_proj", 4096, 4096),
                                  ("gate_up", 4096, 22016), ("down", 11008, 4096))),
              "qwen2_7b": (64, (("qkv", 3584, 4608), ("o_proj", 3584, 3584),
                                ("gate_up", 3584, 37888), ("down", 18944, 3584)))}
    dt, copies = torch.float16, 3
    stream = torch.cuda.Stream(dev)
    out = {}
    for model, (g, shapes) in models.items():
        ws = {name: [synth.make_weights(k, n, g, dt, dev, seed=1100 + 10 * j + c)
                     for c in range(copies)] for j, (name, k, n) in enumerate(shapes)}
        res = {}
        for m in (8, 12, 16, 24, 32, 48, 64):
            xs = {name: synth.make_input(m, k, dt, dev, seed=1150) for name, k, n in shapes}
            ys = {name: torch.empty(m, n, dtype=dt, device=dev) for name, k, n in shapes}

            def linear_us(name, plan):
                def run():
                    for c in range(copies):
                        w = ws[name][c]
                        cawq.gemm(xs[name], w.qweight, w.qzeros, w.scales, g, out=ys[name],
                                  plan=plan)
                return _graph_us(run, reps, stream) / copies

            row = {"planner": sorted({cawq.plan_get(m, k, n, g, dt)["path"]
                                      for name, k, n in shapes})}
            pre = 0.0
            for name, k, n in shapes:
                if m <= 16:
                    pre += min(linear_us(name, {"path": 2, "warps": 1, "split": sp})
                               for sp in (1, 2, 4, 8) if sp * 8 <= k // 64)
                else:
                    pre += linear_us(name, None)
            row["prefill_us"] = round(pre, 2)
            if m <= 16:
                row["decode_us"] = round(sum(linear_us(name, None) for name, _, _ in shapes), 2)
            res[f"M={m}"] = row
            del xs, ys
        out[model] = res
        del ws
    return out


def fused_neighbour_numbers(dev, reps=10):
    """The fused neighbours of the GEMM, graph-timed, us per call (weight
    copies rotated so they come from HBM at small M):
    * gate_up: cawq_gemm_silu_mul against cawq_gemm + torch silu * mul and
      against cawq_gemm alone (Llama-2-7B 4096 -> 2 x 11008, g 128; Qwen2-7B
      3584 -> 2 x 18944, g 64);
    * qkv: cawq_gemm_qkv into three outputs against three cawq_gemm calls
      (Qwen2-7B 3584 -> 3584 + 2 x 512, g 64)."""
    import torch

    import cube_awq_b200 as cawq
    from cube_awq_b200 import synth
    dt = torch.float16
    stream = torch.cuda.Stream(dev)
    res = {}
    for name, k, inter, g, copies in (("llama2_7b_gate_up", 4096, 11008, 128, 4),
                                      ("qwen2_7b_gate_up", 3584, 18944, 64, 3)):
        ws = [synth.make_weights(k, 2 * inter, g, dt, dev, seed=900 + c) for c in range(copies)]
        fz = [tuple(cawq.interleave_gate_up(t) for t in (w.qweight, w.qzeros, w.scales))
              for w in ws]
        r = {}
        for m in (1, 16, 64, 2048):
            x = synth.make_input(m, k, dt, dev, seed=950)
            y = torch.empty(m, 2 * inter, dtype=dt, device=dev)
            h = torch.empty(m, inter, dtype=dt, device=dev)

            def unfused():
                for w in ws:
                    cawq.gemm(x, w.qweight, w.qzeros, w.scales, g, out=y)
                    torch.mul(torch.nn.functional.silu(y[:, :inter]), y[:, inter:], out=h)

            def gemm_only():
                for w in ws:
                    cawq.gemm(x, w.qweight, w.qzeros, w.scales, g, out=y)

            def fused():
                for q, z, sc in fz:
                    cawq.gemm_silu_mul(x, q, z, sc, g, out=h)
            n = 2 if m >= 2048 else reps
            r[f"M={m}"] = {lab: round(_graph_us(fn, n, stream) / copies, 2) for lab, fn in
                           (("gemm_then_torch_silu_mul_us", unfused), ("gemm_only_us", gemm_only),
                            ("fused_silu_mul_us", fused))}
        res[name] = r
        del ws, fz
    k, nq, nkv, g, copies = 3584, 3584, 512, 64, 6
    ws = [synth.make_weights(k, nq + 2 * nkv, g, dt, dev, seed=960 + c) for c in range(copies)]
    parts = [[(w.qweight[:, a // 8:b // 8].contiguous(), w.qzeros[:, a // 8:b // 8].contiguous(),
               w.scales[:, a:b].contiguous())
              for a, b in ((0, nq), (nq, nq + nkv), (nq + nkv, nq + 2 * nkv))] for w in ws]
    r = {}
    for m in (1, 16, 2048):
        x = synth.make_input(m, k, dt, dev, seed=970)
        outs = [torch.empty(m, c, dtype=dt, device=dev) for c in (nq, nkv, nkv)]

        def three():
            for pw in parts:
                for (q, z, sc), o in zip(pw, outs):
                    cawq.gemm(x, q, z, sc, g, out=o)

        def split():
            for w in ws:
                cawq.gemm_qkv(x, w.qweight, w.qzeros, w.scales, g, nq, nkv, out=tuple(outs))
        n = 2 if m >= 2048 else reps
        r[f"M={m}"] = {lab: round(_graph_us(fn, n, stream) / copies, 2) for lab, fn in
                       (("three_gemms_us", three), ("fused_qkv_split_us", split))}
    res["qwen2_7b_qkv"] = r
    del ws, parts
    return res


def _timed_calls(call, n_it, max_over_ranks):
    """us per call of `call(i)` issued back to back (direct C calls, so the
    host stays ahead of the GPU), device-timed, max over ranks."""
    import torch
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(n_it):
        call(i)
    e1.record()
    e1.synchronize()
    return round(max_over_ranks(e0.elapsed_time(e1) / n_it) * 1e3, 2)


def tp_fused_numbers(dev, world, max_over_ranks, reps=20):
    """configs[4] layers with the library's own exchange over peer memory
    (cawq_gemm_colpar_p2p / _rowpar_p2p: the GEMM epilogue pushes over NVLink
    at decode sizes; above a few MiB per rank the GEMM writes only its own
    buffer and the peers read it after the flag exchange, with a
    reduce-scatter + all-gather for the row-parallel sum) against the GEMM
    followed by NCCL (cawq_gemm_colpar / _rowpar): gate_up
    column-parallel WITH the all-gather (full [M, 57344] on every rank) and
    down row-parallel (all-reduce). us per call, max over ranks."""
    import torch

    from cube_awq_b200 import _lib, synth, tp
    from cube_awq_b200.errors import check
    k1, n1, k2, n2, g, dt = 8192, 57344, 28672, 8192, GROUP, torch.float16
    comm = tp.TPComm(timeout_ms=120000)
    slot = max(2048 * n1 * 2, world * 2048 * n2 * 4)
    peers = tp.TPPeers(comm, 256 + 2 * slot + 4096, timeout_ms=10000)
    w1 = synth.make_weights(k1, n1, g, dt, dev, seed=4101)
    w2 = synth.make_weights(k2, n2, g, dt, dev, seed=4102)
    col = tp.ColumnParallelAWQLinear(w1.qweight, w1.qzeros, w1.scales, backend="native",
                                     comm=comm)
    row = tp.RowParallelAWQLinear(w2.qweight, w2.qzeros, w2.scales, backend="native", comm=comm)
    del w1, w2
    torch.cuda.empty_cache()
    L = _lib.lib()
    f16 = _lib.CAWQ_F16
    stream = torch.cuda.current_stream(dev).cuda_stream
    res = {"n_gpus": world, "fused_p2p": "CUDA IPC peer buffers + flags: epilogue push at "
           "M <= 8, peer reads (reduce-scatter + all-gather for the sum) at M = 2048",
           "nccl": "GEMM, then NCCL all-gather + interleave / fp32 all-reduce + epilogue"}
    for m in (1, 8, 2048):
        x1 = synth.make_input(m, k1, dt, dev, seed=4103)
        x2 = synth.make_input(m, k2 // world, dt, dev, seed=4104)
        out1 = torch.empty(m, n1, dtype=dt, device=dev)
        out2 = torch.empty(m, n2, dtype=dt, device=dev)
        ws = torch.empty(m * n1, dtype=dt, device=dev)
        part = torch.empty(m * n2, dtype=torch.float32, device=dev)
        cargs = (x1.data_ptr(), col.qweight.data_ptr(), col.qzeros.data_ptr(),
                 col.scales.data_ptr(), None, out1.data_ptr())
        rargs = (x2.data_ptr(), row.qweight.data_ptr(), row.qzeros.data_ptr(),
                 row.scales.data_ptr(), None, out2.data_ptr())
        calls = {
            ("gate_up_colpar", "nccl_us"): lambda i: check(L.cawq_gemm_colpar(
                comm.handle, *cargs, ws.data_ptr(), m, k1, n1, g, f16, stream)),
            ("gate_up_colpar", "fused_p2p_us"): lambda i: check(L.cawq_gemm_colpar_p2p(
                peers.table, peers.next_epoch(), *cargs, m, k1, n1, g, f16, stream)),
            ("down_rowpar", "nccl_us"): lambda i: check(L.cawq_gemm_rowpar(
                comm.handle, *rargs, part.data_ptr(), m, k2, n2, g, f16, stream)),
            ("down_rowpar", "fused_p2p_us"): lambda i: check(L.cawq_gemm_rowpar_p2p(
                peers.table, peers.next_epoch(), *rargs, m, k2, n2, g, f16, stream)),
        }
        r = {}
        for (name, lab), call in calls.items():
            for i in range(3):
                call(i)
            r.setdefault(name, {})[lab] = _timed_calls(call, 3 if m >= 2048 else reps,
                                                       max_over_ranks)
        res[f"M={m}"] = r
        del x1, x2, out1, out2, ws, part
    torch.cuda.synchronize()
    # bit 1 set on any rank = a flag wait gave up (the fused numbers are void)
    import cube_awq_b200 as cawq
    res["device_error_word"] = int(max_over_ranks(float(cawq.device_error())))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()  # every rank's last fused call has completed
    peers.close()
    comm.close()
    del col, row
    return res


def _graph_calls_us(fn, n_rep, max_over_ranks):
    """us per fn() replayed from a CUDA graph (captured once, so the host
    stays out of the timed region), device-timed, max over ranks. fn(stream)
    issues its work on the given raw stream handle."""
    import torch
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        fn(s.cuda_stream)  # warm-up outside the graph (lazy set-up)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        fn(s.cuda_stream)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(n_rep):
            g.replay()
        e1.record(s)
    e1.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / n_rep
    del g  # a graph holding NCCL calls goes before the communicator
    torch.cuda.synchronize()
    return round(max_over_ranks(us), 2)


def tp_mlp_numbers(dev, world, max_over_ranks, reps=20):
    """configs[4] over all ranks of the job: us per MLP forward (gate_up
    column-parallel without the gather, then down row-parallel on this rank's
    share of the gate_up columns, as after the SiLU-and-mul), GEMM + NCCL
    path (the library's own communicator), each part captured in a CUDA
    graph so that the host stays out of the timed region, max over ranks.
    `one_gpu_us` is the same MLP unsharded on one GPU (each rank times it on
    its own GPU alone, max over ranks), and `efficiency` = one_gpu_us / (n_gpus
    * us), the strong-scaling efficiency of the sharded layer. `fused_us` /
    `fused_efficiency`: the same MLP with down through cawq_gemm_rowpar_p2p
    (the library's exchange over peer memory), timed from back-to-back direct
    calls (its host-side epoch keeps it out of graphs; the host stays ahead of
    the GPU), device time, max over ranks."""
    import torch

    from cube_awq_b200 import _lib, synth, tp
    from cube_awq_b200.errors import check
    k1, n1, k2, n2, g, dt = 8192, 57344, 28672, 8192, GROUP, torch.float16
    comm = tp.TPComm(timeout_ms=120000)
    w1 = synth.make_weights(k1, n1, g, dt, dev, seed=4001)
    w2 = synth.make_weights(k2, n2, g, dt, dev, seed=4002)
    col = tp.ColumnParallelAWQLinear(w1.qweight, w1.qzeros, w1.scales, gather_output=False,
                                     backend="native", comm=comm)
    row = tp.RowParallelAWQLinear(w2.qweight, w2.qzeros, w2.scales, backend="native", comm=comm)
    L = _lib.lib()
    f16 = _lib.CAWQ_F16
    nl = n1 // world
    peers = None
    if world > 1:
        plane = 2048 * n2 * 4
        slot = 2 * ((plane + 255) // 256 * 256) + 2048 * n2 * 2
        peers = tp.TPPeers(comm, 256 + 2 * slot + 4096, timeout_ms=10000)
    res = {"n_gpus": world, "backend": "native NCCL (cawq_gemm_colpar shard / cawq_gemm_rowpar)",
           "timing": "CUDA graph per part (NCCL calls captured), device time, max over ranks",
           "limit": "the down all-reduce (fp32 [M, 8192]) and per-call latency at small M"}
    for m in (1, 8, 2048):
        x = synth.make_input(m, k1, dt, dev, seed=4003)
        h = torch.empty(m, nl, dtype=dt, device=dev)
        hh = h[:, :k2 // world]  # this rank's share of the down input (row stride nl)
        hh_c = torch.empty(m, k2 // world, dtype=dt, device=dev)
        out = torch.empty(m, n2, dtype=dt, device=dev)
        part = torch.empty(m * n2, dtype=torch.float32, device=dev)
        h1 = torch.empty(m, n1, dtype=dt, device=dev)
        x2f = synth.make_input(m, k2, dt, dev, seed=4004)

        def col_call(stream):
            check(L.cawq_gemm(x.data_ptr(), col.qweight.data_ptr(), col.qzeros.data_ptr(),
                              col.scales.data_ptr(), None, h.data_ptr(), m, k1, nl, g, f16, f16,
                              _lib.CAWQ_ORDER_AWQ, nl, stream))

        def row_call(stream):
            hh_c.copy_(hh)
            check(L.cawq_gemm_rowpar(comm.handle, hh_c.data_ptr(), row.qweight.data_ptr(),
                                     row.qzeros.data_ptr(), row.scales.data_ptr(), None,
                                     out.data_ptr(), part.data_ptr(), m, k2, n2, g, f16, stream))

        def one_gpu_call(stream):  # the unsharded MLP on this GPU alone
            check(L.cawq_gemm(x.data_ptr(), w1.qweight.data_ptr(), w1.qzeros.data_ptr(),
                              w1.scales.data_ptr(), None, h1.data_ptr(), m, k1, n1, g, f16, f16,
                              _lib.CAWQ_ORDER_AWQ, n1, stream))
            check(L.cawq_gemm(x2f.data_ptr(), w2.qweight.data_ptr(), w2.qzeros.data_ptr(),
                              w2.scales.data_ptr(), None, out.data_ptr(), m, k2, n2, g, f16, f16,
                              _lib.CAWQ_ORDER_AWQ, n2, stream))
        n_rep = 3 if m >= 2048 else reps
        t_col = _graph_calls_us(col_call, n_rep, max_over_ranks)
        t_row = _graph_calls_us(row_call, n_rep, max_over_ranks)
        t_one = _graph_calls_us(one_gpu_call, n_rep, max_over_ranks)
        t = t_col + t_row
        res[f"M={m}"] = {"us": round(t, 2), "gate_up_colpar_us": t_col,
                         "down_rowpar_allreduce_us": t_row, "one_gpu_us": t_one,
                         "efficiency": round(t_one / (world * t), 3)}
        if peers is not None:
            stream = torch.cuda.current_stream(dev).cuda_stream

            def fused_call(i):
                col_call(stream)
                hh_c.copy_(hh)
                check(L.cawq_gemm_rowpar_p2p(peers.table, peers.next_epoch(), hh_c.data_ptr(),
                                             row.qweight.data_ptr(), row.qzeros.data_ptr(),
                                             row.scales.data_ptr(), None, out.data_ptr(), m,
                                             k2, n2, g, f16, stream))
            for i in range(3):
                fused_call(i)
            t_f = _timed_calls(fused_call, n_rep, max_over_ranks)
            res[f"M={m}"]["fused_us"] = t_f
            res[f"M={m}"]["fused_efficiency"] = round(t_one / (world * t_f), 3)
        del x, h, hh_c, out, part, h1, x2f
    del col, row, w1, w2
    torch.cuda.synchronize()
    if peers is not None:
        import torch.distributed as dist
        dist.barrier()  # every rank's last fused call has completed
        peers.close()
    comm.close()
    torch.cuda.empty_cache()
    return res


def run_prefill_only(a, rank, local_rank, world):
    import torch
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    peaks, kind = measured_peaks()
    import torch as _t
    res = prefill_numbers(a.prefill_rows, _t.float16, dev, peaks, reps=a.steps, copies=3)
    if rank != 0:
        return
    tot_flops = sum(2.0 * a.prefill_rows * n * k for _, k, n in LLAMA2_7B)
    tot_us = sum(r["us"] for r in res.values())
    tf = tot_flops / (tot_us * 1e-6) / 1e12
    print(json.dumps({"metric": "AWQ GEMM prefill TFLOP/s (Llama-2-7B AWQ linears, f16)",
                      "value": round(tf, 1), "unit": "TFLOP/s", "n_gpus": 1,
                      "higher_is_better": True, "dtype": "f16", "data": "synthetic",
                      "config": {"workload": f"configs[2] prefill M={a.prefill_rows}, g128",
                                 "rows_m": a.prefill_rows},
                      "per_linear": res, "peak": peaks["bf16_tflops"], "peak_kind": kind,
                      "frac": round(tf / peaks["bf16_tflops"], 4)}), flush=True)


# ------------------------------------------------------- CPU baseline
class CpuSample:
    """A bounded sample of the workload for the CPU restatement of the
    reference's arithmetic: CPU_SAMPLE_LAYERS seeded Llama-2-7B layers (the 4
    linears of configs[1] at full size, M = 1), computed with F = f32 (the
    reference's native-float path, the precision its own tests use). One step
    = one layer's 4 linears; bytes are counted as for the GPU metric (packed
    weights + zeros + f16-sized scales)."""

    LAYERS = 2

    def __init__(self):
        import numpy as np
        rng = np.random.default_rng(1)
        words = lambda shape: np.frombuffer(rng.bytes(4 * int(np.prod(shape))),
                                            dtype=np.uint32).reshape(shape)
        self.layers = []
        for _ in range(self.LAYERS):
            lin = []
            for name, k, n in LLAMA2_7B:
                lin.append((k, n, words((k, n // 8)), words((k // GROUP, n // 8)),
                            rng.uniform(0.001, 0.02, (k // GROUP, n)).astype(np.float32),
                            rng.standard_normal((1, k)).astype(np.float32)))
            self.layers.append(lin)

    def step(self, i: int, threads: int):
        import oracle
        t0 = time.perf_counter()
        nbytes = 0
        for k, n, qw, qz, s, x in self.layers[i % self.LAYERS]:
            oracle.gemm_ref(x, qw, qz, s, GROUP, dtype="f32", threads=threads)
            nbytes += weight_bytes(k, n)
        return nbytes, time.perf_counter() - t0


def cpu_f16_emulated(threads: int):
    """Second figure: the same restatement with F = f16, every operation
    rounded to f16 in software (a double computation plus a rounding routine
    per operation), on the o_proj shape restricted to 256 output columns."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(2)
    k, nc = 4096, 256
    qw = rng.integers(0, 2**32, (k, nc // 8), dtype=np.uint64).astype(np.uint32)
    qz = rng.integers(0, 2**32, (k // GROUP, nc // 8), dtype=np.uint64).astype(np.uint32)
    s = rng.uniform(0.001, 0.02, (k // GROUP, nc)).astype(np.float16)
    x = rng.standard_normal((1, k)).astype(np.float16)
    t0 = time.perf_counter()
    oracle.gemm_ref(x, qw, qz, s, GROUP, dtype="f16", threads=threads)
    return weight_bytes(k, nc) / (time.perf_counter() - t0) / 1e9


def cpu_run(steps: int, warmup: int, threads: int):
    sample = CpuSample()
    for i in range(warmup):
        sample.step(i, threads)
    tb, ts = 0, 0.0
    for i in range(steps):
        b, t = sample.step(warmup + i, threads)
        tb += b
        ts += t
    return tb, ts


CPU_SAMPLE_TEXT = ("C restatement of the reference's gemm_awq arithmetic with F = f32 (native "
                   "float, vectorised, -O3 AVX2, no FMA contraction): per step one Llama-2-7B "
                   "layer's 4 AWQ linears at full size, M = 1, rotating over 2 seeded layers "
                   "(~210 MB); bytes counted as for the GPU metric")


def cpu_baseline(steps: int = 20, warmup: int = 2):
    import oracle
    threads = oracle.max_threads()
    b, s = cpu_run(steps, warmup, threads)
    return {"value": round(b / s / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{CPU_SAMPLE_TEXT}; {steps} steps, {s:.2f} s",
            "f16_emulated_gbs": round(cpu_f16_emulated(threads), 4)}


def run_reference(a, rank, world):
    if rank != 0:
        return
    import oracle
    threads = oracle.max_threads()
    b, s = cpu_run(a.steps, max(0, min(a.warmup, 3)), threads)
    v = b / s / 1e9
    line = {
        "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(s / a.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "impl": "reference",
        "data": "synthetic (seeded)",
        "config": workload_config(a, world),
        "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{CPU_SAMPLE_TEXT}; {a.steps} steps, {s:.2f} s (the "
                                   "Rust/CubeCL reference cannot run on this machine)"},
        "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    rank, local_rank, world = dist_env()
    if world > 1:
        # NCCL's communicator lines (rank, nranks, device: "Init COMPLETE")
        # show that every rank joined an N-rank communicator. NCCL reads this
        # once, at its first call, so it is set before torch is imported; a
        # quieter level from the environment (VERSION, WARN) is raised.
        if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION", "WARN"):
            os.environ["NCCL_DEBUG"] = "INFO"
            os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
    if a.impl == "reference":
        run_reference(a, rank, world)
    elif a.workload == "prefill":
        run_prefill_only(a, rank, local_rank, world)
    else:
        run_ours(a, rank, local_rank, world)
        if world > 1:
            # All device work is done; leave without the libraries' exit-time
            # teardown, whose NCCL log lines would otherwise follow the JSON
            # line on stdout.
            sys.stdout.flush()
            sys.stderr.flush()
            os._exit(0)


if __name__ == "__main__":
    main()
