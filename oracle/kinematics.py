"""CPU restatement (float64, numpy) of the kinematics outputs of a G1 state — test infrastructure only (the parity
checker of the CUDA kernels nb_g1_kinematics / nb_g1_kinematics_vjp; nothing in the product calls it).

Semantics as the reference states them (src/nablaengine/g1_engine/kinematics.py:1-47, MuJoCo MJX 3.17
kinematics + com_pos + com_vel):
  qpos_n       qpos with the root quaternion normalised;
  xpos, xquat  (B, 31, 3 / 4) body frames, the world body (0, (1, 0, 0, 0)) included; the root (qpos[0:3], normalised
               quaternion); a hinge body: pos = xpos[p] + R_p body_pos[b], quat = xquat[p] body_quat[b]
               axis_angle(axis, q) (not renormalised);
  subtree_com  (B, 31, 3) sum(m xipos) / sum(m) over each subtree, xipos = xpos + R body_ipos (the torso's ipos plus
               the per-world com offset); subtree_com[0] = subtree_com[1];
  cvel         (B, 31, 6) [W_b; V_b + W_b x (subtree_com[1] - xpos[b])], W_b the world angular velocity (root:
               R_1 qvel[3:6]; child: W_p + axis_b qd_b), V_b the velocity of the body origin (root: qvel[0:3]; child:
               V_p + W_p x (xpos[b] - xpos[p])); body 0 zeros.
vjp_fd: central differences (float64) of the cotangent-weighted outputs with respect to the raw qpos (36) and qvel.
"""
from pathlib import Path

import numpy as np

MODEL = Path(__file__).resolve().parents[1] / "nablaengine_b200" / "model" / "g1_model.npz"
_M = []


def model():
    if not _M:
        with np.load(MODEL) as z:
            _M.append({k: z[k] for k in z.files})
    return _M[0]


def quat_mul(a, b):
    w1, x1, y1, z1 = np.moveaxis(a, -1, 0)
    w2, x2, y2, z2 = np.moveaxis(b, -1, 0)
    return np.stack([w1 * w2 - x1 * x2 - y1 * y2 - z1 * z2, w1 * x2 + x1 * w2 + y1 * z2 - z1 * y2,
                     w1 * y2 - x1 * z2 + y1 * w2 + z1 * x2, w1 * z2 + x1 * y2 - y1 * x2 + z1 * w2], -1)


def quat_rot(q, v):
    """v rotated by the unit quaternion q (..., 4): v + w t + u x t with t = 2 u x v."""
    w, u = q[..., :1], q[..., 1:]
    t = 2.0 * np.cross(u, v)
    return v + w * t + np.cross(u, t)


def kinematics(qpos, qvel, com):
    m = model()
    qpos, qvel, com = (np.asarray(x, np.float64) for x in (qpos, qvel, com))
    B, NB = qpos.shape[0], m["body_parentid"].shape[0]
    par = m["body_parentid"]
    xpos, xquat = np.zeros((B, NB, 3)), np.zeros((B, NB, 4))
    W, V = np.zeros((B, NB, 3)), np.zeros((B, NB, 3))
    xquat[:, 0, 0] = 1.0
    qn = qpos.copy()
    qn[:, 3:7] = qpos[:, 3:7] / np.linalg.norm(qpos[:, 3:7], axis=1, keepdims=True)
    xpos[:, 1], xquat[:, 1] = qpos[:, 0:3], qn[:, 3:7]
    W[:, 1] = quat_rot(xquat[:, 1], qvel[:, 3:6])
    V[:, 1] = qvel[:, 0:3]
    for b in range(2, NB):
        p, j = par[b], m["body_jntadr"][b]
        qa, da = m["jnt_qposadr"][j], m["jnt_dofadr"][j]
        axis = m["jnt_axis"][j]
        xpos[:, b] = xpos[:, p] + quat_rot(xquat[:, p], np.broadcast_to(m["body_pos"][b], (B, 3)))
        q0 = quat_mul(xquat[:, p], np.broadcast_to(m["body_quat"][b], (B, 4)))
        ang = qpos[:, qa]
        ha = np.concatenate([np.cos(ang / 2)[:, None], np.sin(ang / 2)[:, None] * axis[None]], 1)
        xquat[:, b] = quat_mul(q0, ha)
        aw = quat_rot(xquat[:, b], np.broadcast_to(axis, (B, 3)))
        W[:, b] = W[:, p] + aw * qvel[:, da][:, None]
        V[:, b] = V[:, p] + np.cross(W[:, p], xpos[:, b] - xpos[:, p])
    ipos = np.broadcast_to(m["body_ipos"], (B, NB, 3)).copy()
    ipos[:, int(m["torso_body"])] += com
    xipos = xpos + quat_rot(xquat, ipos)
    mass = m["body_mass"]
    S = xipos * mass[None, :, None]
    Mt = np.broadcast_to(mass, (B, NB)).copy()
    for b in range(NB - 1, 0, -1):
        if par[b] != 0:
            S[:, par[b]] += S[:, b]
            Mt[:, par[b]] += Mt[:, b]
    sc = np.zeros((B, NB, 3))
    sc[:, 1:] = S[:, 1:] / Mt[:, 1:, None]
    sc[:, 0] = sc[:, 1]
    cvel = np.zeros((B, NB, 6))
    cvel[:, 1:, :3] = W[:, 1:]
    cvel[:, 1:, 3:] = V[:, 1:] + np.cross(W[:, 1:], sc[:, 1:2] - xpos[:, 1:])
    return dict(qpos_n=qn, xpos=xpos, xquat=xquat, cvel=cvel, subtree_com=sc)


def _dot(out, cot):
    return sum(np.sum(out[k].reshape(len(out[k]), -1) * cot[k].reshape(len(cot[k]), -1), 1) for k in cot)


def vjp_fd(qpos, qvel, com, cot, h=1e-6):
    """(gq (B, 36), gv (B, 35)): central differences of sum_k <cot[k], out[k]> in each raw qpos and qvel entry."""
    qpos, qvel = np.asarray(qpos, np.float64), np.asarray(qvel, np.float64)
    gq, gv = np.zeros(qpos.shape), np.zeros(qvel.shape)
    for i in range(qpos.shape[1]):
        a, b = qpos.copy(), qpos.copy()
        a[:, i] += h
        b[:, i] -= h
        gq[:, i] = (_dot(kinematics(a, qvel, com), cot) - _dot(kinematics(b, qvel, com), cot)) / (2 * h)
    for i in range(qvel.shape[1]):
        a, b = qvel.copy(), qvel.copy()
        a[:, i] += h
        b[:, i] -= h
        gv[:, i] = (_dot(kinematics(qpos, a, com), cot) - _dot(kinematics(qpos, b, com), cot)) / (2 * h)
    return gq, gv
