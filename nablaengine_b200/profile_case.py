"""A small profiling case: `python -m nablaengine_b200.profile_case [--worlds B] [--launches N] [--kernel K]` runs one
of the kernels N times (default 3) on B (default 1480: one wave of the forward) seeded worlds of the benchmark
configurations and prints a summary. K = forward (k_forward, configuration 2 states), adjoint (k_adjoint after one
forward with tape, configuration 3 states, exact mode) or jacobian (k_jacobian, configuration 4 states). For ncu:
capture the last launch (-k regex:k_<K> -s N-1 -c 1)."""
import argparse

import torch

from nablaengine_b200 import synthetic, torch_ffi

KEYS = ("qpos", "qvel", "warm", "ctrl", "friction", "com")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--worlds", type=int, default=1480)
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--kernel", default="forward", choices=("forward", "adjoint", "jacobian"))
    a = ap.parse_args()
    cfg = {"forward": "forward", "adjoint": "vjp", "jacobian": "jacobian"}[a.kernel]
    s = synthetic.config_states(cfg, B=a.worlds)
    x = [torch.from_numpy(s[k]).cuda() for k in KEYS]
    if a.kernel == "forward":
        for _ in range(a.launches):
            out = torch_ffi.forward(*x)
        torch.cuda.synchronize()
        print("ok forward, mean Newton iterations of the last substep", out[3][:, 0].float().mean().item())
        return
    q1, v1, w1, info, tape = torch_ffi.forward(*x, tape=True)
    if a.kernel == "adjoint":
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


if __name__ == "__main__":
    main()
