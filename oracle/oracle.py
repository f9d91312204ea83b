"""Python wrapper of the CPU oracle (oracle/g1_oracle.cpp). TEST INFRASTRUCTURE: the parity tests, smoke() and the
CPU-baseline leg of bench.py use it as the checker; the product package never imports it.

step(...) runs one control step of the reference's algorithm (float64 by default) on the host cores; fd_jacobian(...)
takes central differences of it in the reference's tangent basis (qpos tangent 35 = root position 3, root rotation
vector 3 in the local frame, hinge angles 29; then qvel 35 and ctrl 29), as the reference's float64 truth does
(reference `benchmarks/bench/truth/fdlib.py` fd_job: mj_integratePos for the qpos columns).
"""
import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "libg1oracle.so"
NQ, NV, NU = 36, 35, 29
_lib = None


def build():
    """Compile the oracle library (g++ with OpenMP); a no-op when it is up to date."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        _lib = ctypes.CDLL(str(LIB))
        d, i = ctypes.c_void_p, ctypes.c_int
        _lib.g1_oracle_step.argtypes = [i, d, d, d, d, d, d, i, i, ctypes.c_double, i, i, d, d, d, d, d, d]
        _lib.g1_oracle_step.restype = i
        _lib.g1_oracle_fd_jacobian_mode.argtypes = [i] + [d] * 6 + [i, i, ctypes.c_double, i, i, ctypes.c_double,
                                                                    ctypes.c_double, i, d]
        _lib.g1_oracle_fd_jacobian_mode.restype = i
        _lib.g1_oracle_core_stats.argtypes = [i] + [d] * 6 + [i, i, d, d, d]
        _lib.g1_oracle_core_stats.restype = i
        _lib.g1_oracle_matrices.argtypes = [i] + [d] * 10
        _lib.g1_oracle_matrices.restype = i
    return _lib


def _c(x, shape):
    a = np.ascontiguousarray(np.asarray(x, np.float64).reshape(shape))
    return a


def step(qpos, qvel, warm, ctrl, friction, com, iterations=10, substeps=4, tol=1e-8, precision=64, threads=0,
         stats=False, contacts=False):
    """(qpos', qvel', warm', info (B, 4) int32) of one control step, as float64 arrays; stats=True appends the
    per-substep counts (B, substeps, 4): contacts kept, rows, Newton iterations, line-search evaluations;
    contacts=True appends the last substep's kept contacts (B, 64, 3) as (pair, slot, dist), pair -1 past the count."""
    B = np.asarray(qpos).shape[0]
    args = [_c(qpos, (B, NQ)), _c(qvel, (B, NV)), _c(warm, (B, NV)), _c(ctrl, (B, NU)), _c(friction, (B,)),
            _c(com, (B, 3))]
    oq, ov, ow = np.zeros((B, NQ)), np.zeros((B, NV)), np.zeros((B, NV))
    info = np.zeros((B, 4), np.int32)
    st = np.zeros((B, int(substeps), 4), np.int32) if stats else None
    con = np.zeros((B, 64, 3)) if contacts else None
    p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    rc = lib().g1_oracle_step(B, *map(p, args), int(iterations), int(substeps), float(tol), int(precision),
                              int(threads), p(oq), p(ov), p(ow), p(info), p(st), p(con))
    if rc:
        raise ValueError(f"g1_oracle_step failed ({rc})")
    return (oq, ov, ow, info) + ((st,) if stats else ()) + ((con,) if contacts else ())


def matrices(qpos, qvel, qacc, ctrl, friction, com):
    """(M, M + h kv, H, nrow) of one substep at its input state and Newton solution qacc, float64 (B, 35, 35) each:
    the mass matrix with armature, the implicitfast matrix and the Newton Hessian at the rows active at qacc."""
    B = np.asarray(qpos).shape[0]
    args = [_c(qpos, (B, NQ)), _c(qvel, (B, NV)), _c(qacc, (B, NV)), _c(ctrl, (B, NU)), _c(friction, (B,)),
            _c(com, (B, 3))]
    M, Q, H = (np.zeros((B, NV, NV)) for _ in range(3))
    nrow = np.zeros(B, np.int32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if lib().g1_oracle_matrices(B, *map(p, args), p(M), p(Q), p(H), p(nrow)):
        raise ValueError("g1_oracle_matrices failed")
    return M, Q, H, nrow


def quat_mul(a, b):
    w1, x1, y1, z1 = np.moveaxis(a, -1, 0)
    w2, x2, y2, z2 = np.moveaxis(b, -1, 0)
    return np.stack([w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2, w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
                     w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2, w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2], -1)


def integrate_pos(qpos, dq):
    """qpos moved along the tangent dq (35): root position, root rotation vector in the local frame, hinges."""
    q = np.array(qpos, np.float64, copy=True)
    q[..., :3] += dq[..., :3]
    w = dq[..., 3:6]
    ang = np.linalg.norm(w, axis=-1, keepdims=True)
    axis = np.where(ang > 0, w / np.where(ang > 0, ang, 1), 0)
    dquat = np.concatenate([np.cos(ang / 2), axis * np.sin(ang / 2)], -1)
    quat = q[..., 3:7] / np.linalg.norm(q[..., 3:7], axis=-1, keepdims=True)
    q[..., 3:7] = quat_mul(quat, dquat)
    q[..., 7:] += dq[..., 6:]
    return q


def fd_jacobian(qpos, qvel, warm, ctrl, friction, com, h=1e-6, iterations=2000, tol=1e-13, substeps=4, threads=0):
    """Central-difference Jacobian (B, 71, 99) of (qpos' [36, qpos form], qvel' [35]) with respect to (qpos tangent
    35, qvel 35, ctrl 29), float64, on a well converged solve (defaults as the reference's truth)."""
    B = np.asarray(qpos).shape[0]
    cols = []
    for j in range(99):
        outs = []
        for s in (1.0, -1.0):
            q, v, u = np.asarray(qpos, np.float64), np.asarray(qvel, np.float64), np.asarray(ctrl, np.float64)
            if j < 35:
                dq = np.zeros((B, 35))
                dq[:, j] = s * h
                q = integrate_pos(q, dq)
            elif j < 70:
                v = v.copy()
                v[:, j - 35] += s * h
            else:
                u = u.copy()
                u[:, j - 70] += s * h
            oq, ov, _, _ = step(q, v, warm, u, friction, com, iterations, substeps, tol, 64, threads)
            outs.append(np.concatenate([oq, ov], 1))
        cols.append((outs[0] - outs[1]) / (2 * h))
    return np.stack(cols, 2)


def fd_jacobian_mode(qpos, qvel, warm, ctrl, friction, com, clamp_kv=1, normal=0, soft=0.2, h=1e-6, iterations=2000,
                     tol=1e-13, substeps=4, threads=0):
    """Central-difference Jacobian (B, 71, 99) of the surrogate step of the adjoint's gradient mode (clamp_kv,
    normal, soft) in the tangent basis, float64, converged solves: the derivative that mode's analytic VJP must give
    (oracle/g1_oracle.cpp: Mode). clamp_kv=1, normal=0 is the plain step's Jacobian (fd_jacobian)."""
    B = np.asarray(qpos).shape[0]
    args = [_c(qpos, (B, NQ)), _c(qvel, (B, NV)), _c(warm, (B, NV)), _c(ctrl, (B, NU)), _c(friction, (B,)),
            _c(com, (B, 3))]
    J = np.zeros((B, NQ + NV, 2 * NV + NU))
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    rc = lib().g1_oracle_fd_jacobian_mode(B, *map(p, args), int(iterations), int(substeps), float(tol), int(clamp_kv),
                                          int(normal), float(soft), float(h), int(threads), p(J))
    if rc:
        raise ValueError(f"g1_oracle_fd_jacobian_mode failed ({rc})")
    return J


def core_stats(qpos, qvel, warm, ctrl, friction, com, iterations=10, substeps=4):
    """Per world of one step: the smallest centre distance nu (m) of a sphere-core (self) contact over the substeps
    (1e300: none), the number of capsule contacts the near-parallel rule holds (normal option on), and the pair of
    the smallest-nu contact (-1: none)."""
    B = np.asarray(qpos).shape[0]
    args = [_c(qpos, (B, NQ)), _c(qvel, (B, NV)), _c(warm, (B, NV)), _c(ctrl, (B, NU)), _c(friction, (B,)),
            _c(com, (B, 3))]
    nu, nh, pr = np.zeros(B), np.zeros(B, np.int32), np.zeros(B, np.int32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    if lib().g1_oracle_core_stats(B, *map(p, args), int(iterations), int(substeps), p(nu), p(nh), p(pr)):
        raise ValueError("g1_oracle_core_stats failed")
    return nu, nh, pr


def threads_available():
    return len(os.sched_getaffinity(0))
