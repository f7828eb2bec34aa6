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
           launch duration (CUDA events on the launching stream), against the
           measured HBM copy bandwidth of MEASURED_PEAKS.json

--impl reference runs the CPU restatement of the reference's arithmetic (the
reference itself is Rust/CubeCL on wgpu and cannot run on this machine) on the
host cores, on a bounded sample of the same workload.

With N GPUs (torchrun) every rank decodes its own model replica (weak
scaling); ranks only meet for the barrier and the max-over-ranks timing.
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
    ap.add_argument("--no-extras", action="store_true", help="skip the M sweep and CPU baseline")
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
        plans[name] = cawq.autotune(xs[name], layer.qweight, layer.qzeros, layer.scales, GROUP,
                                    out=ys[name])

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
    with ClockSampler(local_rank) as clocks:
        barrier()
        e0.record()
        for _ in range(a.steps):
            graph.replay()
        e1.record()
        e1.synchronize()
        barrier()
    ms = max_over_ranks(e0.elapsed_time(e1)) / a.steps
    value = step_bytes * world / (ms * 1e-3) / 1e9

    # ---- roofline: per-launch CUDA events on the launching stream
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
    tot_b, tot_ms = 0, 0.0
    for b, s0, s1, name in evs:
        t = s0.elapsed_time(s1)
        tot_b += b
        tot_ms += t
        per_name.setdefault(name, []).append(t)
    achieved = tot_b / (tot_ms * 1e-3) / 1e9
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

    # ---- extras: M sweep of configs[1] (graph replay, cold weights)
    extras = {}
    if not a.no_extras:
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
        extras["decode_sweep_m"] = sweep

    if world > 1:
        del graph
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    cpu = None if a.no_extras else cpu_baseline(threads=1, sample_cols=512)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded; uniform nibbles, scales U(0.001,0.02), x N(0,1))",
        "config": {"workload": "configs[1] decode M=1: Llama-2-7B AWQ linears x 32 layers, g128",
                   "rows_m": rows, "layers": a.layers, "group_size": GROUP,
                   "step_weight_bytes": step_bytes, "l2": "cold (3.4 GB of distinct weights per step)",
                   "graph": "one CUDA graph per step (128 launches)",
                   "plans": plans, "parallelism": f"replica x{world} (weak, no data-path collective)"},
        "tokens_per_s": round(world * 1e3 / ms, 1),
        "us_per_linear": {k: round(statistics.median(v) * 1e3, 2) for k, v in per_name.items()},
        "e2e": {"value": round(e2e_val, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                "api": "AWQGEMMLinear.forward x 128, no graph"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": traffic, "peak_kind": peaks_kind,
                     "kernel": "cawq::decode_kernel (per-launch events, 20 steps x 128 launches)"},
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": a.steps * a.layers * len(LLAMA2_7B),
    }
    line.update(extras)
    print(json.dumps(line), flush=True)


# ------------------------------------------------------- CPU baseline
def cpu_sample(threads: int, sample_cols: int):
    """Time the oracle (reference numerics, f16) on one layer's 4 linears at
    M = 1, restricted to the first `sample_cols` output columns of each."""
    import numpy as np

    import oracle
    rng = np.random.default_rng(1)
    total_bytes, total_s = 0, 0.0
    for name, k, n in LLAMA2_7B:
        nc = min(n, sample_cols)
        qw = rng.integers(0, 2**32, (k, nc // 8), dtype=np.uint64).astype(np.uint32)
        qz = rng.integers(0, 2**32, (k // GROUP, nc // 8), dtype=np.uint64).astype(np.uint32)
        s = rng.uniform(0.001, 0.02, (k // GROUP, nc)).astype(np.float16)
        x = rng.standard_normal((1, k)).astype(np.float16)
        t0 = time.perf_counter()
        oracle.gemm_ref(x, qw, qz, s, GROUP, dtype="f16", threads=threads)
        total_s += time.perf_counter() - t0
        total_bytes += weight_bytes(k, nc)
    return total_bytes, total_s


def cpu_baseline(threads: int, sample_cols: int):
    import oracle
    if threads <= 0:
        threads = oracle.max_threads()
    b, s = cpu_sample(threads, sample_cols)
    return {"value": round(b / s / 1e9, 4), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle reference numerics (f16 ops), M=1, 4 Llama-2-7B linears x "
                      f"{sample_cols} output columns ({b} weight bytes), {s:.2f} s"}


def run_reference(a, rank, world):
    if rank != 0:
        return
    import oracle
    threads = oracle.max_threads()
    sample_cols = 256
    for _ in range(max(0, min(a.warmup, 3))):
        cpu_sample(threads, sample_cols)
    tb, ts = 0, 0.0
    for _ in range(a.steps):
        b, s = cpu_sample(threads, sample_cols)
        tb += b
        ts += s
    v = tb / ts / 1e9
    line = {
        "metric": METRIC, "value": round(v, 4), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": round(ts / a.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f16", "impl": "reference",
        "data": "synthetic (seeded)",
        "config": {"workload": "configs[1] decode M=1: Llama-2-7B AWQ linears, g128",
                   "rows_m": 1, "group_size": GROUP},
        "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"per step: 4 linears x {sample_cols} output columns, M=1, "
                                   "oracle restating the reference's F arithmetic (Rust/CubeCL "
                                   "reference not runnable here)"},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    rank, local_rank, world = dist_env()
    if a.impl == "reference":
        run_reference(a, rank, world)
    else:
        run_ours(a, rank, local_rank, world)


if __name__ == "__main__":
    main()
