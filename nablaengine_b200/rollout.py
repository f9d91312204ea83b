"""Sharded rollout with backprop through time: T control steps of B worlds per GPU,
differentiated through torch autograd (every step's forward writes its tape; the backward runs the analytic adjoint
per step in reverse), then one NCCL all-reduce of a small float64 vector [loss, sum of the squared ctrl gradients,
worlds, steps] over the ranks (NVLink / NVSwitch). The worlds shard by contiguous ranges with no collective inside
the steps; the only exchange is that all-reduce.

  python -m torch.distributed.run --nproc-per-node N -m nablaengine_b200.rollout [--worlds 32768] [--steps 32]

The loss is the mean over steps and worlds of |qvel_t|^2 (per rank its partial sum, summed over the ranks); the ctrl
gradients are d loss / d ctrl_t. `step_fn` defaults to torch_ffi.step (the CUDA path); tests of the sharding and
reduction logic on CPU pass their own step function.
"""
import json
import os

from . import synthetic

T_DEFAULT, WORLDS_DEFAULT = 32, 32768


def shard(total, rank, world):
    """(start, count) of rank's contiguous range of `total` worlds over `world` ranks (the first total % world ranks
    take one more)."""
    base, extra = divmod(int(total), int(world))
    start = rank * base + min(rank, extra)
    return start, base + (1 if rank < extra else 0)


def rollout_inputs(B, T, rank=0, device="cpu"):
    """The configuration-5 inputs of one rank: seeded synthetic states (seed 4 + rank, 5 % of worlds falling) and a
    (T, B, 29) ctrl random walk (N(0, 0.05) steps) from their ctrl, as float32 tensors on `device`."""
    import torch
    s = synthetic.config_states("rollout", B=B, seed_offset=rank)
    ctrl = synthetic.rollout_ctrl(s["ctrl"], T, seed=1000 + rank)
    t = {k: torch.from_numpy(v).to(device) for k, v in s.items()}
    t["ctrl_seq"] = torch.from_numpy(ctrl).to(device)
    return t


def bptt(inputs, step_fn=None, grad_decay=1.0, **step_kw):
    """One rollout of T steps and its backward: (loss partial sum (0-d tensor), d loss / d ctrl (T, B, 29)). The
    loss is sum_t sum_worlds |qvel_t|^2 / (T * B_total) with B_total = inputs['worlds_total'] (default: this
    rank's B)."""
    import torch
    if step_fn is None:
        from . import torch_ffi
        step_fn = torch_ffi.step
    q, v, w = inputs["qpos"], inputs["qvel"], inputs["warm"]
    ctrl = inputs["ctrl_seq"].detach().clone().requires_grad_(True)
    T, B = ctrl.shape[0], ctrl.shape[1]
    norm = 1.0 / (T * float(inputs.get("worlds_total", B)))
    loss = torch.zeros((), dtype=torch.float32, device=ctrl.device)
    for t in range(T):
        q, v, w = step_fn(q, v, w, ctrl[t], inputs["friction"], inputs["com"], grad_decay=grad_decay, **step_kw)
        loss = loss + (v * v).sum() * norm
    loss.backward()
    return loss.detach(), ctrl.grad


def reduce_stats(loss, gctrl, group=None):
    """The all-reduced float64 vector [loss, sum |g_ctrl|^2, ctrl-gradient rows, rows with a non-finite gradient]
    (one collective; torch.distributed's default group unless `group`)."""
    import torch
    import torch.distributed as dist
    g = gctrl.double()
    finite = torch.isfinite(g).all(dim=-1)
    vec = torch.stack([loss.double(), torch.where(torch.isfinite(g), g, 0.0).pow(2).sum(),
                       torch.tensor(float(finite.numel()), dtype=torch.float64, device=g.device),
                       (~finite).sum().double()])
    if dist.is_available() and dist.is_initialized():
        dist.all_reduce(vec, op=dist.ReduceOp.SUM, group=group)
    return vec


def main(argv=None):
    import argparse
    import datetime
    import torch
    import torch.distributed as dist
    from . import torch_ffi
    ap = argparse.ArgumentParser()
    ap.add_argument("--worlds", type=int, default=WORLDS_DEFAULT, help="worlds per GPU")
    ap.add_argument("--steps", type=int, default=T_DEFAULT, help="control steps T")
    ap.add_argument("--repeats", type=int, default=5)
    ap.add_argument("--compact-tape", action="store_true", help="keep compact tapes (no L_Q: 31 %% less memory)")
    a = ap.parse_args(argv)
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    torch_ffi.init(local)
    inp = rollout_inputs(a.worlds, a.steps, rank, dev)
    inp["worlds_total"] = a.worlds * world
    bptt(inp, compact_tape=a.compact_tape)  # warm-up (allocator, first launches)
    reduce_stats(*bptt(inp, compact_tape=a.compact_tape))
    times, red, vec = [], [], None
    for _ in range(a.repeats):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record()
        loss, g = bptt(inp, compact_tape=a.compact_tape)
        e1.record()
        vec = reduce_stats(loss, g)
        e2.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e2))
        red.append(e1.elapsed_time(e2))
    # per rank: the median and the slowest rollout, and the median all-reduce (with its wait for the slowest rank);
    # gathered, then the maximum over ranks of the rollout times
    mine = torch.tensor([sorted(times)[len(times) // 2], max(times), sorted(red)[len(red) // 2]], dtype=torch.float64,
                        device=dev)
    per = [mine.clone() for _ in range(world)]
    if world > 1:
        dist.all_gather(per, mine)
        dist.destroy_process_group()
    per = torch.stack(per).cpu()
    med, slow = per[:, 0].max().item(), per[:, 1].max().item()
    if rank == 0:
        v = vec.cpu().tolist()
        print(json.dumps({"metric": "BPTT rollout world-steps/s (fwd+grad)", "n_gpus": world,
                          "worlds_per_gpu": a.worlds,
                          "steps": a.steps, "repeats": a.repeats, "ms_per_rollout": med,
                          "ms_per_rollout_slowest": slow,
                          "per_rank_ms_median": per[:, 0].tolist(), "per_rank_allreduce_ms": per[:, 2].tolist(),
                          "value": world * a.worlds * a.steps / (med / 1e3), "unit": "world-steps/s",
                          "loss": v[0], "ctrl_grad_norm": v[1] ** 0.5, "rows": v[2], "nonfinite_rows": v[3],
                          "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9}), flush=True)


if __name__ == "__main__":
    main()
