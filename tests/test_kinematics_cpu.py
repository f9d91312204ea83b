"""The kinematics oracle (oracle/kinematics.py) pinned to MuJoCo Warp: the body poses it computes put every floor
contact's sphere centre / capsule end where MuJoCo Warp 3.17's collision found it at the input state (the
reference's fixture mjw317_mf_s0.npz `con`: pair, dist, pos, normal; contact pos = centre - n (r + dist / 2))."""
import numpy as np

import kinematics as K


def test_oracle_poses_match_mujoco_warp_contacts(golden):
    d = golden("mjw_contacts.npz")
    m = K.model()
    out = K.kinematics(d["qpos"], d["qvel"], d["com"])
    xpos, xquat = out["xpos"], out["xquat"]
    checked, worst = 0, 0.0
    for w in range(len(d["qpos"])):
        for c in range(int(d["con_count"][w])):
            cw = d["con"][w, c]
            pr, dist, pos, nrm = int(cw[0]), float(cw[1]), cw[2:5], cw[5:8]
            g1, g2 = int(m["pair_g1"][pr]), int(m["pair_g2"][pr])
            if m["geom_type"][g1] != 0:
                continue  # floor contacts only
            b = int(m["geom_bodyid"][g2])
            r = float(m["geom_size"][g2][0])
            centre = xpos[w, b] + K.quat_rot(xquat[w, b], m["geom_pos"][g2])
            want = pos.astype(np.float64) + nrm.astype(np.float64) * (r + 0.5 * dist)
            if m["geom_type"][g2] == 3:  # capsule: the nearer end along its axis
                gq = K.quat_mul(xquat[w, b], m["geom_quat"][g2])
                ax = K.quat_rot(gq, np.array([0.0, 0.0, 1.0]))
                hl = float(m["geom_size"][g2][1])
                ends = [centre + hl * ax, centre - hl * ax]
                centre = min(ends, key=lambda e: np.linalg.norm(e - want))
            err = float(np.linalg.norm(centre - want))
            worst = max(worst, err)
            checked += 1
    assert checked > 100, checked
    assert worst < 1e-6, worst  # measured 1.7e-7 m (the float32 fixture)
