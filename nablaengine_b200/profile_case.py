"""A small profiling case: `python -m nablaengine_b200.profile_case [--worlds B] [--launches N]` runs the forward
step N times (default 3) on B (default 1024) seeded worlds of the benchmark configuration and prints the mean
iteration count. For ncu: capture the last launch (-k regex:k_forward -s N-1 -c 1)."""
import argparse

import torch

from nablaengine_b200 import synthetic, torch_ffi


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--worlds", type=int, default=1024)
    ap.add_argument("--launches", type=int, default=3)
    a = ap.parse_args()
    s = synthetic.config_states("forward", B=a.worlds)
    x = [torch.from_numpy(s[k]).cuda() for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    for _ in range(a.launches):
        out = torch_ffi.forward(*x)
    torch.cuda.synchronize()
    print("ok", out[3][:, 0].float().mean().item())


if __name__ == "__main__":
    main()
