"""Generate tests/golden/mode_states.npz: states whose self contacts exercise the adjoint's normal options 2 and 3
(a sphere-core contact with centre distance nu below their 1 mm threshold), made from the reference's self-contact
gradient states (truth_grad.npz, group G6) by turning one hinge.

For each G6 state, take its self contact closest to degenerate (smallest nu, the CPU oracle's collision at the
input state); turning the hinge of one of its two bodies (or of their parents) over the joint's range sweeps the
capsules' axes across each other, and a scan of the hinge angle, refined twice, finds where the smallest nu of any
self contact is smallest; near that crossing, the angle whose nu is closest to NU_AIM (0.5 mm) is kept.

    python tests/golden/make_mode_states.py

Test infrastructure: uses the CPU oracle (oracle/), not the product library; the tests read the .npz it writes.
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT / "oracle"))
import oracle  # noqa: E402

KEYS = ("qpos", "qvel", "qacc_warmstart", "ctrl", "friction", "com")
# nu in (NU_LO, NU_MAX): below the options' 1 mm threshold by a margin float32 cannot cross, and far above the
# central differences' step (1e-6), which must stay small against nu for the normal's derivative to be resolved
NU_LO, NU_AIM, NU_MAX, WANT = 2e-4, 5e-4, 8e-4, 8


def closest(states, hinge_q, angles):
    """Smallest nu (and its pair) of the states with qpos[hinge_q] set to each angle (collision at the input)."""
    B = len(angles)
    x = {k: np.repeat(states[k][None], B, 0) for k in KEYS}
    x["qpos"] = x["qpos"].copy()
    x["qpos"][:, hinge_q] = angles
    nu, _, pair = oracle.core_stats(*(x[k] for k in KEYS), iterations=0, substeps=1)
    return nu, pair


def main():
    m = np.load(ROOT / "nablaengine_b200" / "model" / "g1_model.npz")
    d = np.load(HERE / "truth_grad.npz")
    idx = np.flatnonzero(d["group_G6"])
    keep = {k: [] for k in KEYS}
    nus, src = [], []
    for i in idx:
        s = {k: d[k][i] for k in KEYS}
        nu0, _, pair = oracle.core_stats(*(s[k][None] for k in KEYS), iterations=0, substeps=1)
        p = int(pair[0])
        if p < 0:
            continue
        g1, g2 = int(m["pair_g1"][p]), int(m["pair_g2"][p])
        b1, b2 = int(m["geom_bodyid"][g1]), int(m["geom_bodyid"][g2])
        par = m["body_parentid"]
        found = None
        for body in (b1, b2, int(par[b1]), int(par[b2])):  # the pair's bodies' hinges, then their parents'
            if body < 2:
                continue
            q = body + 4 + 1  # the body's hinge dof is body + 4, its angle qpos[dof + 1]
            lo, hi = (float(x) for x in m["dof_range"][body + 4])
            ang = np.linspace(lo, hi, 401)
            coarse = ang[1] - ang[0]
            for _ in range(3):
                nu, _ = closest(s, q, ang)
                j = int(np.argmin(nu))
                step = ang[1] - ang[0]
                best_a, best = float(ang[j]), float(nu[j])
                ang = np.clip(np.linspace(best_a - 2 * step, best_a + 2 * step, 161), lo, hi)
            if best < NU_LO:  # near the crossing: the angle whose nu is closest to NU_AIM
                ang = np.clip(np.linspace(best_a - coarse, best_a + coarse, 801), lo, hi)
                nu, _ = closest(s, q, ang)
                j = int(np.argmin(np.abs(nu - NU_AIM)))
                if NU_LO < nu[j] < NU_MAX:
                    found = (q, float(ang[j]))
                    break
        if found is None:
            continue
        s["qpos"] = s["qpos"].copy()
        s["qpos"][found[0]] = np.float32(found[1])
        nu_f, _, _ = oracle.core_stats(*(s[k][None] for k in KEYS), iterations=0, substeps=1)
        if not NU_LO < nu_f[0] < NU_MAX:  # (the float32 rounding of the angle moved it)
            continue
        for k in KEYS:
            keep[k].append(s[k])
        nus.append(float(nu_f[0]))
        src.append(int(d["index"][i]))
        if len(nus) == WANT:
            break
    out = {k: np.stack(v).astype(np.float32) for k, v in keep.items()}
    out.update(min_nu=np.array(nus), source_index=np.array(src, np.int32))
    np.savez_compressed(HERE / "mode_states.npz", **out)
    print("mode_states.npz:", len(nus), "states, min nu (m):", np.round(nus, 6))


if __name__ == "__main__":
    main()
