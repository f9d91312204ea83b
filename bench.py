#!/usr/bin/env python
"""Benchmark of the B200 G1 step: world-steps/s of the forward control step at B = 4096 worlds per GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0. A "step" is one control step (4 x 5 ms substeps, Newton capped at 10 iterations) of the
4096 worlds of BASELINE configuration 2 (seeded synthetic states of the benchmark distribution; rank r uses seed
1 + r). `value` is device-timed (CUDA events on the launching stream, inputs resident in HBM, an L2 flush between
steps outside the timed events, max over ranks); `e2e` is the same metric through the public torch API with the
inputs copied from pinned host memory and the outputs copied back inside the timed region. `roofline` counts the
step's algorithmic FP32 FLOPs from the kernel's own work counters (nablaengine_b200/flops.py) over the measured kernel
time; `cpu_baseline` times the float64 CPU oracle (the reference's CPU path, MuJoCo C, is not installed on the box) on
a bounded sample with all host threads. Under torchrun every rank runs its own 4096 worlds (weak scaling, no
collective inside the step).

--impl reference: the reference's CPU implementation of the path on the box's host cores (MuJoCo is not installed, so
the float64 oracle port stands in), rank 0 only, each step a bounded sample of the same workload.
"""
import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))
B_PER_GPU = 4096
ITERATIONS, SUBSTEPS = 10, 4
FP32_PEAK_TFLOPS_NOMINAL = 148 * 128 * 2 * 1.965e9 / 1e12  # 74.4: 148 SMs x 128 FP32 lanes x FMA at 1965 MHz
METRIC = "world-steps/sec fwd at B=4096/GPU"


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except Exception:  # noqa: BLE001
        return {}


class Clocks:
    """nvidia-smi samples (every 200 ms) while the timed region runs."""

    def __init__(self, index):
        self.index, self.rows, self.proc = index, [], None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:  # noqa: BLE001
            self.proc = None
        time.sleep(0.3)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        time.sleep(0.3)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:  # noqa: BLE001
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in self.rows for n, v in zip(names, r[4:8]) if v.lower() == "active"})
        loaded = [x for x in sm if x > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": float(self.rows[0][1]) if self.rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(self.rows)}


def traffic_per_world():
    """DRAM bytes per world of one forward launch from the committed ncu summary (None if absent)."""
    p = ROOT / "profiles" / "k_forward.md"
    if not p.exists():
        return None
    m = re.search(r"dram_bytes_per_world:\s*([0-9.eE+-]+)", p.read_text())
    return float(m.group(1)) if m else None


def cpu_baseline(seconds=12.0):
    """The float64 oracle (all host threads) on BASELINE configuration 1 (256 seeded worlds), repeated ~12 s."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    from nablaengine_b200 import synthetic
    s = synthetic.config_states("cpu_reference")
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    B = args[0].shape[0]
    threads = oracle.threads_available()
    oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)  # warm-up
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)
        n += 1
    dt = time.perf_counter() - t0
    return {"value": B * n / dt, "unit": "world-steps/s", "cores": threads, "kind": "port",
            "sample": f"{n} calls x {B} worlds of configuration 1 (seed 0), float64 oracle, {ITERATIONS} iterations "
                      f"x {SUBSTEPS} substeps, {dt:.1f} s; MuJoCo C (the reference's CPU path) is not installed"}


def measure_fwd_grad(dev, rank, steps, warmup, flush):
    """forward + analytic VJP of one step (4096 worlds, 10 % lowered into multi-contact),
    loss = sum(qvel'^2), exact gradient mode (clamp_kv=1, normal=0), through torch autograd (torch_ffi.step then
    loss.backward()). Device time per step (CUDA events, L2 flushed between steps); the forward-with-tape and the
    adjoint kernels also timed alone."""
    import torch
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("vjp", seed_offset=rank)
    keys = ("qpos", "qvel", "warm", "ctrl", "friction", "com")
    x = [torch.from_numpy(s[k]).to(dev) for k in keys]
    B = x[0].shape[0]
    leaves = [x[0].clone().requires_grad_(True), x[1].clone().requires_grad_(True), x[3].clone().requires_grad_(True)]

    def one():
        q, v, u = leaves
        for t in leaves:
            t.grad = None
        q1, v1, w1 = torch_ffi.step(q, v, x[2], u, x[4], x[5], iterations=ITERATIONS, substeps=SUBSTEPS, clamp_kv=1,
                                    normal=0)
        (v1 * v1).sum().backward()

    st = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in ev:
            flush.zero_()
            e0.record(st)
            fn()
            e1.record(st)
        torch.cuda.synchronize()
        return sum(e0.elapsed_time(e1) for e0, e1 in ev) / steps

    ms = timed(one)
    ms_fwd_tape = timed(lambda: torch_ffi.forward(*x, iterations=ITERATIONS, substeps=SUBSTEPS, tape=True))
    q1, v1, w1, info, tape = torch_ffi.forward(*x, iterations=ITERATIONS, substeps=SUBSTEPS, tape=True)
    gq, gv = torch.zeros_like(q1), 2 * v1
    ms_bwd = timed(lambda: torch_ffi.backward(tape, x[4], x[5], gq, gv, clamp_kv=1, normal=0))
    return {"B": B, "ms": ms, "ms_fwd_tape": ms_fwd_tape, "ms_adjoint": ms_bwd}


def measure_jacobian(dev, rank, steps, warmup, flush):
    """the full 71 x 99 step Jacobian of 4096 worlds (forward with tape, then the Jacobian
    kernel, exact mode), device time per step with the L2 flushed between steps; us per world."""
    import torch
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("jacobian", seed_offset=rank)
    x = [torch.from_numpy(s[k]).to(dev) for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    B = x[0].shape[0]
    st = torch.cuda.current_stream(dev)

    def one():
        tape = torch_ffi.forward(*x, iterations=ITERATIONS, substeps=SUBSTEPS, tape=True)[4]
        return torch_ffi.jacobian(tape, x[4], x[5], substeps=SUBSTEPS)

    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    tot = 0.0
    for _ in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        one()
        e1.record(st)
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    return {"B": B, "ms": tot / steps}


def run_reference(a, rank):
    """--impl reference: rank 0 times the reference's CPU path substitute (the float64 oracle port) per step on a
    bounded sample of the configuration-2 workload."""
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    from nablaengine_b200 import synthetic
    s = synthetic.config_states("forward")
    sample = 512  # worlds per timed step (a bounded slice of the 4096)
    args = [s[k][:sample] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    threads = oracle.threads_available()
    for _ in range(a.warmup):
        oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)
    times = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)
        times.append(time.perf_counter() - t0)
    value = sample * len(times) / sum(times)
    out = {"metric": METRIC, "value": value, "unit": "world-steps/s", "impl": "reference", "n_gpus": a.gpus,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * B_PER_GPU / value,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
           "config": {"workload": "forward control step, BASELINE configuration 2 (B=4096 seeded synthetic G1 "
                                  "states; the timed sample: the first 512 worlds per step)",
                      "iterations": ITERATIONS, "substeps": SUBSTEPS, "cpu_threads": threads},
           "cpu_baseline": {"value": value, "unit": "world-steps/s", "cores": threads, "kind": "port",
                            "sample": f"{sample} of the 4096 worlds per step, float64 oracle; MuJoCo C (the "
                                      "reference's CPU path) is not installed on the box"},
           "e2e": {"value": value, "unit": "world-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    a = ap.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if a.impl == "reference":
        return run_reference(a, rank)
    a.warmup = max(a.warmup, 3)

    import torch
    import torch.distributed as dist
    from nablaengine_b200 import capi, flops, synthetic, torch_ffi
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    torch_ffi.init(local)
    s = synthetic.config_states("forward", seed_offset=rank)
    keys = ("qpos", "qvel", "warm", "ctrl", "friction", "com")
    x = [torch.from_numpy(s[k]).to(dev) for k in keys]
    B = x[0].shape[0]
    lib = capi.load()
    st = torch.cuda.current_stream(dev)

    # work counters of this workload (untimed; the outputs are bitwise the timed call's)
    stats = torch.zeros((B, SUBSTEPS, 8), dtype=torch.int32, device=dev)
    outs = [torch.empty((B, 36), device=dev), torch.empty((B, 35), device=dev), torch.empty((B, 35), device=dev),
            torch.empty((B, 4), dtype=torch.int32, device=dev)]
    import ctypes
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.nb_g1_forward_stats(ctypes.c_void_p(st.cuda_stream), B, *map(P, x), ITERATIONS, SUBSTEPS,
                                 *map(P, outs), P(stats))
    assert rc == 0, rc
    flop_step = flops.per_step(stats.cpu().numpy())
    counters = stats.cpu().numpy().reshape(-1, 8).mean(0)

    flush = torch.empty(256 * 2 ** 20 // 4, dtype=torch.float32, device=dev)  # > 126 MB L2
    for _ in range(a.warmup):
        torch_ffi.forward(*x, iterations=ITERATIONS, substeps=SUBSTEPS)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    with Clocks(local) as clk:
        for e0, e1 in ev:
            flush.zero_()
            e0.record(st)
            torch_ffi.forward(*x, iterations=ITERATIONS, substeps=SUBSTEPS)
            e1.record(st)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    kern_ms = [e0.elapsed_time(e1) for e0, e1 in ev]
    total = torch.tensor([sum(kern_ms)], dtype=torch.float64, device=dev)
    fg = measure_fwd_grad(dev, rank, a.steps, a.warmup, flush)
    jac = measure_jacobian(dev, rank, max(1, min(a.steps, 3)), 1, flush)
    fg_ms = torch.tensor([fg["ms"], fg["ms_fwd_tape"], fg["ms_adjoint"], jac["ms"]], dtype=torch.float64,
                         device=dev)

    # end to end through the public API: pinned host inputs in, host outputs back, every step
    host = [t.cpu().pin_memory() for t in x]
    hout = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs]
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = sum(t.numel() * t.element_size() for t in hout)

    def e2e_step():
        dx = [h.to(dev, non_blocking=True) for h in host]
        r = torch_ffi.forward(*dx, iterations=ITERATIONS, substeps=SUBSTEPS)
        for h, o in zip(hout, r):
            h.copy_(o, non_blocking=True)

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(a.steps):
        e2e_step()
    e1.record(st)
    torch.cuda.synchronize()
    e2e_total = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
        dist.all_reduce(e2e_total, op=dist.ReduceOp.MAX)
        dist.all_reduce(fg_ms, op=dist.ReduceOp.MAX)
    t_s, e2e_s = total.item() / 1e3, e2e_total.item() / 1e3
    value = world * B * a.steps / t_s
    e2e_value = world * B * a.steps / e2e_s
    clocks = clk.summary()
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    ms = 1e3 * t_s / a.steps
    achieved = flop_step / (ms / 1e3) / 1e12
    tpw = traffic_per_world()
    peaks = load_peaks()
    out = {
        "metric": METRIC, "value": value, "unit": "world-steps/s", "n_gpus": world, "steps": a.steps,
        "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "forward control step, BASELINE configuration 2: B=4096 worlds per GPU of seeded "
                               "synthetic G1 states (home keyframe, joint noise, root height U(0.70, 0.80) m)",
                   "worlds_per_gpu": B, "iterations": ITERATIONS, "substeps": SUBSTEPS,
                   "l2": "flushed between timed steps (256 MB write outside the events)",
                   "parallelism": f"data-parallel worlds, {world} GPU(s), no collective in the step",
                   "mean_counts_per_substep": {"contacts": float(counters[0]), "rows": float(counters[1]),
                                               "newton_iterations": float(counters[2]),
                                               "line_search_evals": float(counters[3]),
                                               "factorisations": float(counters[4])}},
        "roofline": {"bound": "fp32", "achieved": achieved,
                     "peak": FP32_PEAK_TFLOPS_NOMINAL, "unit": "TFLOP/s",
                     "frac": achieved / FP32_PEAK_TFLOPS_NOMINAL,
                     "peak_note": "FP32 CUDA-core peak at the measured max SM clock (148 SMs x 128 lanes x 2 x "
                                  f"{peaks.get('sm_max_mhz', 1965.0):.0f} MHz; MEASURED_PEAKS.json has no FP32 "
                                  "figure); the path has no GEMM or HBM-bound kernel",
                     "flop_per_step": flop_step,
                     "traffic": None if tpw is None else tpw * B,
                     "hbm_achieved_gbs": (B * (556 + 440) / (ms / 1e3)) / 1e9,
                     "hbm_peak_gbs": peaks.get("hbm_gbs")},
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": "world-steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": a.steps * (3 if torch_ffi._DIAG_ON[0] else 2),  # k_order, k_forward (+ diagnostics)
        "fwd_grad": {"metric": "world-steps/sec fwd+grad at B=4096/GPU (BASELINE configuration 3: loss sum(qvel'^2), "
                               "VJP w.r.t. qpos, qvel, ctrl, exact mode clamp_kv=1 normal=0, torch autograd)",
                     "value": world * fg["B"] / (fg_ms[0].item() / 1e3), "unit": "world-steps/s",
                     "ms_per_step": fg_ms[0].item(), "ms_forward_with_tape": fg_ms[1].item(),
                     "ms_adjoint": fg_ms[2].item(), "worlds_per_gpu": fg["B"],
                     "gpu_launches_per_step": 3, "l2": "flushed between timed steps"},
        "jacobian": {"metric": "full 71 x 99 step Jacobian (forward with tape + Jacobian kernel, exact mode), us per "
                               "world at B=4096/GPU (BASELINE configuration 4)",
                     "value": fg_ms[3].item() * 1e3 / jac["B"], "unit": "us/world", "higher_is_better": False,
                     "ms_per_step": fg_ms[3].item(), "worlds_per_gpu": jac["B"], "gpu_launches_per_step": 3,
                     "l2": "flushed between timed steps"},
        "kernel_ms": {"median": statistics.median(kern_ms), "min": min(kern_ms), "max": max(kern_ms)},
    }
    if world == 1 and not a.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline()
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
