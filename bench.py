#!/usr/bin/env python
"""Benchmark of the B200 G1 step: world-steps/s of the forward control step at B = 4096 worlds per GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One JSON line on rank 0. A "step" is one control step (4 x 5 ms substeps, Newton capped at 10 iterations) of the
4096 worlds of BASELINE configuration 2 (seeded synthetic states of the benchmark distribution; rank r uses seed
1 + r). `value` is device-timed (CUDA events on the launching stream, inputs resident in HBM, an L2 flush between
steps outside the timed events, max over ranks); `e2e` is the same metric through the public torch API with the
inputs copied from pinned host memory and the outputs copied back inside the timed region (double-buffered copy
streams overlapping the copies with the neighbouring steps' compute). `roofline` counts the step's algorithmic FP32
FLOPs from the kernel's own work counters (nablaengine_b200/flops.py) over the measured kernel time; `cpu_baseline`
times the float64 CPU oracle (the reference's CPU path, MuJoCo C, is not installed on the box) on a bounded sample
with all host threads. Under torchrun every rank runs its own 4096 worlds (weak scaling, no
collective inside the step).

--impl reference: the reference's CPU implementation of the path on the box's host cores (MuJoCo is not installed, so
the float64 oracle port stands in), rank 0 only, each step a bounded sample of the same workload.
"""
import argparse
import json
import os
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


# DRAM bytes (read + write) per world of one forward launch: ncu `dram__bytes_read.sum + dram__bytes_write.sum` of
# k_forward on 2220 configuration-2 worlds with the world order (one wave, captured by `ncu --set full
# --clock-control none -k regex:k_forward -s 2 -c 1 python bench.py --profile-case forward --worlds 2220`), divided by
# the worlds; the inputs and outputs of the step, nothing re-read
FORWARD_DRAM_BYTES_PER_WORLD = 702


def cpu_baseline(seconds=10.0, corpus_seconds=6.0):
    """The float64 oracle (all host threads) on BASELINE configuration 1 (256 seeded worlds, repeated ~10 s) and on
    the reference's corpus mf_s0 (its first 1024 states, ~6 s), beside the reference's published MuJoCo C numbers on
    the same corpus (MuJoCo C itself is not installed on the box)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    from nablaengine_b200 import synthetic
    threads = oracle.threads_available()

    def rate(args, secs):
        oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)  # warm-up
        n, t0 = 0, time.perf_counter()
        while time.perf_counter() - t0 < secs:
            oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)
            n += 1
        dt = time.perf_counter() - t0
        return args[0].shape[0] * n / dt, n, dt

    s = synthetic.config_states("cpu_reference")
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    value, n, dt = rate(args, seconds)
    cx, _ = corpus_inputs()
    cval, cn, cdt = rate([a[:1024] for a in cx], corpus_seconds)
    return {"value": value, "unit": "world-steps/s", "cores": threads, "kind": "port",
            "sample": f"{n} calls x {args[0].shape[0]} worlds of configuration 1 (seed 0), float64 oracle, "
                      f"{ITERATIONS} iterations x {SUBSTEPS} substeps, {dt:.1f} s; MuJoCo C (the reference's CPU path) "
                      "is not installed on the box",
            "corpus_mf_s0": {"value": cval, "unit": "world-steps/s", "cores": threads,
                             "sample": f"{cn} calls x the first 1024 states of mf_s0, float64 oracle, {cdt:.1f} s",
                             "published_mujoco_c": {cpu: {"ms_per_4096_worlds": ms, "threads": th,
                                                          "world_steps_per_s": 4096 / (ms / 1e3)}
                                                    for cpu, (ms, th) in PUBLISHED_CPU.items()}}}


CORPUS = ROOT / "tests" / "golden" / "corpus_mf_s0.npz"
# the reference's published numbers on this corpus at B = 4096 (docs/results/paper_<gpu>/paper_bench.md:91 forward,
# :92 vjp, :35 backward, :50 Jacobian; 3-process medians for forward and vjp), ms per step (Jacobian: us per world)
PUBLISHED = {"H100 80GB HBM3 (sm_90)": {"fwd": 1.700, "vjp": 2.728, "bwd": 0.930, "jacobian_us_per_world": 16.74},
             "RTX PRO 6000 Blackwell Server (sm_120)": {"fwd": 1.214, "vjp": 1.784, "bwd": 0.563,
                                                         "jacobian_us_per_world": 9.74}}
# MuJoCo C float64 on the same corpus, 4096 worlds per step (paper_<gpu>/paper_bench.md:28), ms per step and threads
PUBLISHED_CPU = {"AMD EPYC 9555": (34.746, 16), "Xeon Platinum 8462Y+": (57.374, 13)}


def corpus_inputs(dev=None):
    """The 4096 input states of the reference's benchmark corpus mf_s0 and its stored cotangent 0."""
    with np.load(CORPUS) as z:
        keys = ("qpos", "qvel", "qacc_warmstart", "ctrl", "friction", "com")
        x = [np.ascontiguousarray(z[k]) for k in keys]
        cot = [np.ascontiguousarray(z["cot_qpos"]), np.ascontiguousarray(z["cot_qvel"])]
    if dev is None:
        return x, cot
    import torch
    return [torch.from_numpy(a).to(dev) for a in x], [torch.from_numpy(a).to(dev) for a in cot]


def paper_timeit(call, sync, rounds=6, warm_calls=5, warm_s=1.0, target_s=0.25):
    """The reference's timing protocol (scripts/paper_bench/common.py:154-193): warm-up of at least warm_calls calls
    and warm_s seconds (each call synchronised), then rounds + 1 rounds of n back-to-back calls with one
    synchronisation each (n sized so a round lasts about target_s), the first round dropped; wall-clock ms per call:
    median, p10, p90 over the kept rounds."""
    t0, k = time.perf_counter(), 0
    while k < warm_calls or time.perf_counter() - t0 < warm_s:
        call()
        sync()
        k += 1
    per_call = (time.perf_counter() - t0) / k
    n = int(min(200, max(1, round(target_s / max(per_call, 1e-6)))))
    per = []
    for _ in range(rounds + 1):
        t = time.perf_counter()
        for _ in range(n):
            call()
        sync()
        per.append((time.perf_counter() - t) / n)
    a = 1e3 * np.asarray(per[1:])
    return {"median": float(np.median(a)), "p10": float(np.percentile(a, 10)), "p90": float(np.percentile(a, 90)),
            "n": n, "rounds": rounds}


def measure_corpus(dev):
    """The reference's own benchmark workload: the 4096 states of its corpus mf_s0, 10 iterations, 4 substeps, timed
    with its protocol (paper_timeit), for the legs it publishes: fwd (forward without tape), fwd_tape, bwd (the
    adjoint alone on one tape, the stored cotangent 0), vjp (forward with tape + adjoint) in the exact gradient mode
    (clamp_kv=1, normal=0), and the full 71 x 99 Jacobian (forward with tape + the Jacobian kernel)."""
    import torch
    from nablaengine_b200 import torch_ffi
    x, (cq, cv) = corpus_inputs(dev)
    B = x[0].shape[0]
    sync = torch.cuda.synchronize
    kw = dict(iterations=ITERATIONS, substeps=SUBSTEPS)
    q1, v1, w1, info, tape = torch_ffi.forward(*x, tape=True, **kw)
    inf = info.cpu().numpy()
    legs = {
        "fwd": lambda: torch_ffi.forward(*x, **kw),
        "fwd_tape": lambda: torch_ffi.forward(*x, tape=True, **kw),
        "bwd": lambda: torch_ffi.backward(tape, x[4], x[5], cq, cv, clamp_kv=1, normal=0),
        "vjp": lambda: torch_ffi.backward(torch_ffi.forward(*x, tape=True, **kw)[4], x[4], x[5], cq, cv, clamp_kv=1,
                                          normal=0),
        "jacobian": lambda: torch_ffi.jacobian(torch_ffi.forward(*x, tape=True, **kw)[4], x[4], x[5]),
    }
    out = {"workload": "the reference's corpus mf_s0 (4096 states, tests/golden/corpus_mf_s0.npz), 10 iterations x "
                       "4 substeps, exact gradient mode; the reference's timing protocol (wall clock, back-to-back "
                       "calls, one sync per round, median of 6 rounds after a dropped one)",
           "worlds": B, "mean_newton_iterations_last_substep": float(inf[:, 0].mean()),
           "mean_contacts_last_substep": float(inf[:, 1].mean()), "max_rows_last_substep": int(inf[:, 2].max())}
    for name, fn in legs.items():
        r = paper_timeit(fn, sync)
        r["world_steps_per_s"] = B / (r["median"] / 1e3)
        out[name] = r
    out["jacobian"]["us_per_world"] = out["jacobian"]["median"] * 1e3 / B
    out["published"] = PUBLISHED
    return out


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
    """--impl reference: rank 0 times the reference's CPU path substitute (the float64 oracle port, all host threads)
    per step on the whole configuration-2 workload (4096 worlds per step)."""
    if rank != 0:
        return
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    from nablaengine_b200 import synthetic
    s = synthetic.config_states("forward")
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    B = args[0].shape[0]
    threads = oracle.threads_available()
    for _ in range(a.warmup):
        oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)
    times = []
    for _ in range(a.steps):
        t0 = time.perf_counter()
        oracle.step(*args, iterations=ITERATIONS, substeps=SUBSTEPS, threads=threads)
        times.append(time.perf_counter() - t0)
    value = B * len(times) / sum(times)
    out = {"metric": METRIC, "value": value, "unit": "world-steps/s", "impl": "reference", "n_gpus": a.gpus,
           "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1e3 * B / value,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
           "config": {"workload": "forward control step, BASELINE configuration 2 (B=4096 seeded synthetic G1 "
                                  "states, all 4096 per timed step)",
                      "iterations": ITERATIONS, "substeps": SUBSTEPS, "cpu_threads": threads},
           "cpu_baseline": {"value": value, "unit": "world-steps/s", "cores": threads, "kind": "port",
                            "sample": f"all {B} worlds per step, float64 oracle; MuJoCo C (the reference's CPU path) "
                                      "is not installed on the box"},
           "e2e": {"value": value, "unit": "world-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def profile_case(a):
    """--profile-case K: a small case for ncu captures, the kernel K (forward: configuration-2 states; adjoint: one
    forward with tape, then the adjoint, configuration-3 states, exact mode; jacobian: configuration-4 states)
    launched --launches times on --worlds seeded worlds (default 1480: one wave of the forward). Capture the last
    launch with ncu (-k regex:k_<K> -s <launches - 1> -c 1); no timing is printed."""
    import torch
    from nablaengine_b200 import synthetic, torch_ffi
    cfg = {"forward": "forward", "adjoint": "vjp", "jacobian": "jacobian", "corpus": None}[a.profile_case]
    if cfg is None:
        x, _ = corpus_inputs("cuda")
        x = [t[:a.worlds] for t in x]
    else:
        s = synthetic.config_states(cfg, B=a.worlds)
        x = [torch.from_numpy(s[k]).cuda() for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    if a.profile_case in ("forward", "corpus"):
        for _ in range(a.launches):
            out = torch_ffi.forward(*x)
        torch.cuda.synchronize()
        print("ok forward, mean Newton iterations of the last substep", out[3][:, 0].float().mean().item())
        return
    q1, v1, w1, info, tape = torch_ffi.forward(*x, tape=True)
    if a.profile_case == "adjoint":
        gq, gv = torch.zeros_like(q1), 2 * v1
        for _ in range(a.launches):
            r = torch_ffi.backward(tape, x[4], x[5], gq, gv, clamp_kv=1, normal=0)
        torch.cuda.synchronize()
        print("ok adjoint, |g_ctrl| =", r[2].norm().item())
    else:
        for _ in range(a.launches):
            J, jinfo = torch_ffi.jacobian(tape, x[4], x[5])
        torch.cuda.synchronize()
        print("ok jacobian, |J| =", J.norm().item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-corpus", action="store_true", help="skip the corpus leg")
    ap.add_argument("--profile-case", choices=("forward", "adjoint", "jacobian", "corpus"), default=None,
                    help="run a small case of one kernel for an ncu capture instead of the benchmark")
    ap.add_argument("--worlds", type=int, default=1480, help="--profile-case: worlds")
    ap.add_argument("--launches", type=int, default=3, help="--profile-case: launches of the kernel")
    a = ap.parse_args()
    if a.profile_case:
        return profile_case(a)
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
    corpus = measure_corpus(dev) if world == 1 and not a.no_corpus else None

    # end to end through the public API: pinned host inputs in, host outputs back, every step; the copies run on
    # their own streams, double-buffered, so step i + 1's inputs cross while step i computes and step i's outputs
    # come back while step i + 1 computes (every byte of every step still crosses inside the timed region)
    host = [t.cpu().pin_memory() for t in x]
    hout = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs]
    h2d = sum(t.numel() * t.element_size() for t in host)
    d2h = sum(t.numel() * t.element_size() for t in hout)
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    dbuf = [[torch.empty_like(t) for t in x] for _ in range(2)]

    def e2e_run(n):
        h2d_stream.wait_stream(st)
        freed = [None, None]  # per input buffer: the step that read it is done
        for i in range(n):
            b = i % 2
            with torch.cuda.stream(h2d_stream):
                if freed[b] is not None:
                    h2d_stream.wait_event(freed[b])
                for d, h in zip(dbuf[b], host):
                    d.copy_(h, non_blocking=True)
                arrived = torch.cuda.Event()
                arrived.record(h2d_stream)
            st.wait_event(arrived)
            r = torch_ffi.forward(*dbuf[b], iterations=ITERATIONS, substeps=SUBSTEPS)
            freed[b] = torch.cuda.Event()
            freed[b].record(st)
            with torch.cuda.stream(d2h_stream):
                d2h_stream.wait_event(freed[b])
                for h, o in zip(hout, r):
                    h.copy_(o, non_blocking=True)
                    o.record_stream(d2h_stream)
        st.wait_stream(d2h_stream)
        st.wait_stream(h2d_stream)

    e2e_run(2)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    h0 = time.perf_counter()
    e2e_run(a.steps)
    e2e_host_ms = (time.perf_counter() - h0) * 1e3 / a.steps  # the host's time to enqueue a step (not the metric)
    e1.record(st)
    torch.cuda.synchronize()
    e2e_total = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    per_rank = [total.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(per_rank, total)
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
        dist.all_reduce(e2e_total, op=dist.ReduceOp.MAX)
        dist.all_reduce(fg_ms, op=dist.ReduceOp.MAX)
    per_rank_ms = [t.item() / a.steps for t in per_rank]
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
    tpw = FORWARD_DRAM_BYTES_PER_WORLD
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
                     "traffic": tpw * B,
                     "hbm_achieved_gbs": (B * (556 + 440) / (ms / 1e3)) / 1e9,
                     "hbm_peak_gbs": peaks.get("hbm_gbs")},
        "clocks": clocks,
        "e2e": {"value": e2e_value, "unit": "world-steps/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_s * 1e3 / a.steps, "host_enqueue_ms_per_step": e2e_host_ms},
        # k_order, k_forward (+ the diagnostics counters and the last-forward record)
        "gpu_launches": a.steps * (4 if torch_ffi.diagnostics_enabled() else 2),
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
        "per_rank_ms_per_step": per_rank_ms,
    }
    if corpus is not None:
        out["corpus"] = corpus
    if world == 1 and not a.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline()
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
