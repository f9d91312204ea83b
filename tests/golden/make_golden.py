"""Generate the committed golden fixtures of tests/golden/ from the reference's own data files.

Run once where the reference repository is readable: python tests/golden/make_golden.py --ref <reference checkout>.
The outputs are small subsets of the reference's Apache-2.0 benchmark data (benchmarks/data, fixtures/mjlab):

  truth_check.npz  the 64 "check" states of each corpus mf_s0..mf_s3 (inputs and MuJoCo C float64 forward truth at
                   2000 iterations, tolerance 1e-13; model_flags 0 = MuJoCo C and MuJoCo Warp agree on the state)
  truth_grad.npz   mf_s0's gradient states: inputs, the 3 stored cotangents, the FD VJP truth (h = 1e-6) and its
                   floor (h = 1e-7) in the tangent basis (qpos tangent 35, qvel 35, ctrl 29), validity bits, groups
  mjw_sample.npz   the first 256 states of mf_s0 with MuJoCo Warp 3.17's one-step outputs (50 iterations, float32)
                   and its per-substep contact / row / iteration counts
  mjw_contacts.npz the first 64 states of mf_s0 with MuJoCo Warp 3.17's contacts at the input state (pair, dist,
                   pos[3], normal[3]): pins the body poses of the kinematics outputs
  truth_jac.npz    16 of mf_s0's Jacobian states (the G0 sample): inputs, the MuJoCo C float64 FD Jacobian (71 x 99,
                   stored float32 by the reference, h = 1e-6, tangent columns), its per-column floor, validity bits
  corpus_mf_s0.npz the whole mf_s0 corpus the reference's published timings run on (4096 states): the step inputs,
                   the stored cotangent 0 (its fwd+grad and backward legs use it) and the MuJoCo C labels of the
                   state's heaviest substep (contacts, rows, solver iterations)

Existing files are kept unless --force is given (each is written once; the tests pin their contents).

Nothing at test time reads the reference; the tests read these files.
"""
import argparse
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
INPUTS = ("qpos", "qvel", "qacc_warmstart", "ctrl", "friction", "com")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="the reference repository root")
    ap.add_argument("--force", action="store_true", help="rewrite files that exist")
    a = ap.parse_args()
    ref = Path(a.ref)
    data = ref / "benchmarks" / "data"
    write = lambda name: a.force or not (HERE / name).exists()  # noqa: E731
    if write("corpus_mf_s0.npz"):
        c = np.load(data / "mf_s0.npz")
        corp = {k: c[k] for k in INPUTS}
        corp.update(cot_qpos=c["cot_qpos"][:, 0], cot_qvel=c["cot_qvel"][:, 0], ncon_max=c["label_ncon_max"],
                    nefc_max=c["label_nefc_max"], niter_max=c["label_niter_max"])
        np.savez_compressed(HERE / "corpus_mf_s0.npz", **corp)
        print("corpus_mf_s0.npz", (HERE / "corpus_mf_s0.npz").stat().st_size, "bytes")
    if write("truth_jac.npz"):
        c, t = np.load(data / "mf_s0.npz"), np.load(data / "truth" / "mf_s0.npz")
        n = 16
        pos = t["jac_index"][:n]  # positions into the gradient states
        jidx = t["index"][pos]     # corpus states
        jac = {k: c[k][jidx] for k in INPUTS}
        jac.update(index=jidx, jacobian=t["jacobian"][:n], jacobian_dcol=t["jacobian_dcol"][:n], bad=t["bad"][pos],
                   model_flags=t["model_flags"][jidx])
        np.savez_compressed(HERE / "truth_jac.npz", **jac)
        print("truth_jac.npz", (HERE / "truth_jac.npz").stat().st_size, "bytes")
    if write("mjw_contacts.npz"):
        c = np.load(data / "mf_s0.npz")
        m = np.load(ref / "fixtures" / "mjlab" / "mjw317_mf_s0.npz")
        n = 64
        w = {k: c[k][:n] for k in INPUTS}
        w.update(con=m["con"][:n], con_count=m["con_count"][:n])
        np.savez_compressed(HERE / "mjw_contacts.npz", **w)
        print("mjw_contacts.npz", (HERE / "mjw_contacts.npz").stat().st_size, "bytes")
    if not write("truth_check.npz"):
        return
    out = {k: [] for k in INPUTS + ("check_out", "model_flags", "corpus", "index")}
    for s in range(4):
        c, t = np.load(data / f"mf_s{s}.npz"), np.load(data / "truth" / f"mf_s{s}.npz")
        idx = t["check_index"]
        for k in INPUTS:
            out[k].append(c[k][idx])
        out["check_out"].append(t["check_out"])
        out["model_flags"].append(t["model_flags"][idx])
        out["corpus"].append(np.full(len(idx), s, np.int8))
        out["index"].append(idx)
    np.savez_compressed(HERE / "truth_check.npz", **{k: np.concatenate(v) for k, v in out.items()})

    c, t = np.load(data / "mf_s0.npz"), np.load(data / "truth" / "mf_s0.npz")
    idx = t["index"]
    g = {k: c[k][idx] for k in INPUTS}
    g.update(cot_qpos=c["cot_qpos"][idx], cot_qvel=c["cot_qvel"][idx], index=idx, out=t["out"],
             fd_vjp=t["fd_vjp"], fd_vjp_floor=t["fd_vjp_floor"], bad=t["bad"], model_flags=t["model_flags"][idx])
    for k in t.files:
        if k.startswith("group_"):
            g[k] = t[k]
    np.savez_compressed(HERE / "truth_grad.npz", **g)

    m = np.load(ref / "fixtures" / "mjlab" / "mjw317_mf_s0.npz")
    n = 256
    w = {k: c[k][:n] for k in INPUTS}
    w.update(out_qpos=m["out_qpos"][:n], out_qvel=m["out_qvel"][:n], ncon=m["ncon"][:n], nefc=m["nefc"][:n],
             niter=m["niter"][:n], model_flags=t["model_flags"][:n])
    np.savez_compressed(HERE / "mjw_sample.npz", **w)
    for f in ("truth_check.npz", "truth_grad.npz", "mjw_sample.npz"):
        print(f, (HERE / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()
