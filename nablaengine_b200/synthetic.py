"""Seeded synthetic G1 states: the input distribution of the benchmark configurations (they stand in for the
reference's benchmark corpora, which are not redistributed with this package).

States (numpy PCG64, float32): the `home` keyframe; hinge offsets N(0, 0.1 rad) clipped to the joint ranges; root
height U(0.70, 0.80) m; a root tilt rotation vector N(0, 0.05 rad) per axis applied to the keyframe quaternion, then
normalised; qvel N(0, 0.5); warm 0; ctrl = hinge angles + N(0, 0.2); friction U(0.4, 1.2); torso COM offset
U(-0.05, 0.05) m per axis. Variants: `lowered` (a share of worlds lowered by U(0.05, 0.15) m: multi-contact feet and
hands), `falling` (a share of worlds at root height U(0.2, 0.5) m tilted by U(0, 1) rad about a random horizontal
axis), `rollout_ctrl` (a per-step random walk of the setpoints, N(0, 0.05) per step).
"""
from pathlib import Path

import numpy as np

MODEL = Path(__file__).resolve().parent / "model" / "g1_model.npz"
NQ, NV, NU = 36, 35, 29
# the benchmark configurations 1-5 (CPU reference, forward, VJP, Jacobian, rollout): worlds per GPU, seed
CONFIGS = {
    "cpu_reference": dict(B=256, seed=0),
    "forward": dict(B=4096, seed=1),
    "vjp": dict(B=4096, seed=2, lowered=0.10),
    "jacobian": dict(B=4096, seed=3),
    "rollout": dict(B=32768, seed=4, falling=0.05, T=32),
}
_M = {}


def model():
    if not _M:
        with np.load(MODEL) as z:
            _M.update({k: z[k] for k in z.files})
    return _M


def _quat_mul(a, b):
    w1, x1, y1, z1 = a.T
    w2, x2, y2, z2 = b.T
    return np.stack([w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2, w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
                     w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2, w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2], 1)


def _rotvec_quat(v):
    ang = np.linalg.norm(v, axis=1, keepdims=True)
    axis = np.where(ang > 0, v / np.where(ang > 0, ang, 1.0), 0.0)
    return np.concatenate([np.cos(ang / 2), axis * np.sin(ang / 2)], 1)


def states(B, seed, lowered=0.0, falling=0.0, **_):
    """Dict of float32 arrays qpos, qvel, warm, ctrl, friction, com for B worlds."""
    m = model()
    rng = np.random.Generator(np.random.PCG64(seed))
    key = m["key_qpos"][0]
    rng_lo, rng_hi = m["dof_range"][6:, 0], m["dof_range"][6:, 1]
    qpos = np.tile(key, (B, 1))
    qpos[:, 7:] = np.clip(key[7:] + rng.normal(0.0, 0.1, (B, NU)), rng_lo, rng_hi)
    qpos[:, 2] = rng.uniform(0.70, 0.80, B)
    tilt = _rotvec_quat(rng.normal(0.0, 0.05, (B, 3)))
    q = _quat_mul(np.tile(key[3:7], (B, 1)), tilt)
    qpos[:, 3:7] = q / np.linalg.norm(q, axis=1, keepdims=True)
    qvel = rng.normal(0.0, 0.5, (B, NV))
    ctrl = qpos[:, 7:] + rng.normal(0.0, 0.2, (B, NU))
    friction = rng.uniform(0.4, 1.2, B)
    com = rng.uniform(-0.05, 0.05, (B, 3))
    if lowered > 0:
        sel = rng.random(B) < lowered
        qpos[sel, 2] -= rng.uniform(0.05, 0.15, int(sel.sum()))
    if falling > 0:
        sel = np.nonzero(rng.random(B) < falling)[0]
        qpos[sel, 2] = rng.uniform(0.2, 0.5, len(sel))
        phi = rng.uniform(0, 2 * np.pi, len(sel))
        axis = np.stack([np.cos(phi), np.sin(phi), np.zeros_like(phi)], 1)
        rot = _rotvec_quat(axis * rng.uniform(0.0, 1.0, (len(sel), 1)))
        q = _quat_mul(qpos[sel, 3:7], rot)
        qpos[sel, 3:7] = q / np.linalg.norm(q, axis=1, keepdims=True)
    f32 = lambda x: np.ascontiguousarray(x, np.float32)  # noqa: E731
    return dict(qpos=f32(qpos), qvel=f32(qvel), warm=np.zeros((B, NV), np.float32), ctrl=f32(ctrl),
                friction=f32(friction), com=f32(com))


def config_states(name, B=None, seed_offset=0):
    cfg = dict(CONFIGS[name])
    if B is not None:
        cfg["B"] = B
    cfg["seed"] += seed_offset
    return states(**cfg)


def rollout_ctrl(ctrl0, T, seed):
    """(T, B, 29) setpoints: a random walk from ctrl0 with N(0, 0.05) steps."""
    rng = np.random.Generator(np.random.PCG64(seed))
    steps = rng.normal(0.0, 0.05, (T,) + ctrl0.shape).astype(np.float32)
    return np.ascontiguousarray(ctrl0[None] + np.cumsum(steps, 0), np.float32)
