"""Host logic of the sharded rollout (nablaengine_b200/rollout.py) on CPU: the world sharding, and the BPTT loss /
ctrl-gradient reduction over world_size-2 gloo ranks equal to one process over the whole batch. The step function
here is a small differentiable stand-in (the CUDA step runs in the GPU tests and bench)."""
import os
import socket

import numpy as np
import pytest
import torch

from nablaengine_b200 import rollout


def _toy_step(q, v, w, ctrl, fric, com, grad_decay=1.0):
    u = torch.nn.functional.pad(ctrl, (6, 0))
    v1 = 0.9 * v + 0.1 * u * fric[:, None] + 0.01 * com.sum(1, keepdim=True)
    q1 = q + 0.005 * torch.nn.functional.pad(v1, (0, 1))
    return q1, v1, w


def _inputs(B, T, seed):
    g = torch.Generator().manual_seed(seed)
    return dict(qpos=torch.randn(B, 36, generator=g), qvel=torch.randn(B, 35, generator=g), warm=torch.zeros(B, 35),
                friction=torch.rand(B, generator=g) + 0.5, com=0.05 * torch.randn(B, 3, generator=g),
                ctrl_seq=torch.randn(T, B, 29, generator=g))


def test_shard_covers_every_world_once():
    for total in (0, 1, 7, 32768, 262144 + 5):
        for world in (1, 2, 3, 8):
            parts = [rollout.shard(total, r, world) for r in range(world)]
            assert sum(c for _, c in parts) == total
            assert all(parts[r][0] + parts[r][1] == parts[r + 1][0] for r in range(world - 1))
            assert max(c for _, c in parts) - min(c for _, c in parts) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, B, T, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    full = _inputs(B, T, 0)
    start, n = rollout.shard(B, rank, world)
    mine = {k: (v[:, start:start + n] if k == "ctrl_seq" else v[start:start + n]) for k, v in full.items()}
    mine["worlds_total"] = B
    loss, g = rollout.bptt(mine, step_fn=_toy_step)
    vec = rollout.reduce_stats(loss, g)
    if rank == 0:
        np.save(out, vec.numpy())
    dist.destroy_process_group()


def test_two_rank_reduction_equals_one_process(tmp_path):
    import torch.multiprocessing as mp
    B, T, world = 10, 3, 2
    out = str(tmp_path / "vec.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), B, T, out), nprocs=world, join=True,
                       start_method="spawn")
    vec = np.load(out)
    full = _inputs(B, T, 0)
    loss, g = rollout.bptt(full, step_fn=_toy_step)
    ref = rollout.reduce_stats(loss, g).numpy()
    assert vec[2] == ref[2] == T * B and vec[3] == 0
    assert vec[0] == pytest.approx(ref[0], rel=1e-5)
    assert vec[1] == pytest.approx(ref[1], rel=1e-5)


def _rank_fails(rank, world, port, out):
    """Rank 1 fails after joining (an exception on the host, between steps: none of its collectives in flight); rank 0
    records what its next collective does."""
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        raise SystemExit(3)
    try:
        rollout.reduce_stats(torch.tensor(1.0), torch.ones(4, 29))
        msg = "completed"
    except Exception as e:  # the failure reaches the surviving rank as an error, not a hang
        msg = "error: " + type(e).__name__
    with open(out, "w") as f:
        f.write(msg)


def test_a_failed_rank_ends_the_other_ranks_reduction_with_an_error(tmp_path):
    import multiprocessing
    ctx = multiprocessing.get_context("spawn")
    out = str(tmp_path / "rank0.txt")
    port = _free_port()
    procs = [ctx.Process(target=_rank_fails, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung"
    assert procs[1].exitcode == 3
    with open(out) as f:
        assert f.read().startswith("error"), "the surviving rank's reduction completed without its peer"
