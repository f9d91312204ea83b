"""Extract the mjlab Unitree G1 model arrays from MuJoCo 3.17's binary model file (g1_train.mjb) without MuJoCo.

Test infrastructure and build-time tooling, not part of the product path: it runs once, where the reference's fixture
file is readable, and writes `nablaengine_b200/model/g1_model.npz` (the arrays the step reads, float64 / int32) plus
`nablaengine_b200/csrc/g1_model_data.h` (the same arrays as C literals, for the oracle and the CUDA library). Both are
committed; nothing at run time reads the .mjb.

The reference loads this file with `mujoco.MjModel.from_binary_path` (reference `src/nablaengine/fixtures.py:99`) and
packs the arrays its kernels read (`src/nablaengine/g1_engine/source.py:28-77` constants, `step.py:123-152`
pair_constants). MuJoCo is not installable here, so the file is decoded directly. Format, as observed in this file:
a 5-word int32 header (magic 54321, sizeof(mjtNum) = 8, number of size fields = 98, version 3017000, number of
arrays = 485), 98 int64 sizes (nq, nv, nu, ...), the option / visual / statistic structs, then every model array
back to back with no padding, in MuJoCo's fixed field order. Each array used here was located by content (qpos0 =
the free joint at (0, 0, 0.793) and unit quaternion, body_parentid, the joint/dof/geom/pair/actuator/keyframe blocks,
the names buffer) and the offsets below are checked against anchors every run (sizes, names, unit quaternions, the
README's sha256 of the file), so a different file fails loudly instead of decoding garbage.

Usage: python oracle/mjb_extract.py --mjb <path to g1_train.mjb> [--check]
"""
import argparse
import hashlib
import json
import math
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[1]
MJB_SHA256 = "757b0997d992073b645732a1daaeab92587f00e29691b93aa76094a3f02ef379"  # fixtures/mjlab/README.md
NQ, NV, NU, NBODY, NJNT, NGEOM, NPAIR, NKEY = 36, 35, 29, 31, 30, 34, 502, 2

# (name, dtype, rows, cols, byte offset): located by content in the 3.17 file (module docstring)
LAYOUT = [
    ("opt_real", "f8", 1, 31, 804),          # timestep impratio tolerance ls_tol noslip_tol ccd_tol sleep_tol
                                             # gravity[3] wind[3] magnetic[3] density viscosity o_margin
                                             # o_solref[2] o_solimp[5] o_friction[5]
    ("opt_int", "i4", 1, 13, 1052),          # integrator cone jacobian solver iterations ls_iterations noslip_it
                                             # ccd_it disableflags enableflags disableactuator sdf_initpoints sdf_it
    ("stat", "f8", 1, 7, 1740),              # meaninertia meanmass meansize extent center[3]
    ("qpos0", "f8", 1, NQ, 1799),
    ("body_parentid", "i4", NBODY, 1, 2375),
    ("body_jntnum", "i4", NBODY, 1, 2871),
    ("body_jntadr", "i4", NBODY, 1, 2995),
    ("body_dofnum", "i4", NBODY, 1, 3119),
    ("body_dofadr", "i4", NBODY, 1, 3243),
    ("body_geomnum", "i4", NBODY, 1, 3491),
    ("body_geomadr", "i4", NBODY, 1, 3615),
    ("body_pos", "f8", NBODY, 3, 3801),
    ("body_quat", "f8", NBODY, 4, 4545),
    ("body_ipos", "f8", NBODY, 3, 5537),
    ("body_iquat", "f8", NBODY, 4, 6281),
    ("body_mass", "f8", NBODY, 1, 7273),
    ("body_subtreemass", "f8", NBODY, 1, 7521),
    ("body_inertia", "f8", NBODY, 3, 7769),
    ("body_invweight0", "f8", NBODY, 2, 8513),
    ("jnt_type", "i4", NJNT, 1, 10189),
    ("jnt_qposadr", "i4", NJNT, 1, 10309),
    ("jnt_dofadr", "i4", NJNT, 1, 10429),
    ("jnt_bodyid", "i4", NJNT, 1, 10549),
    ("jnt_limited", "u1", NJNT, 1, 10909),
    ("jnt_actfrclimited", "u1", NJNT, 1, 10939),
    ("jnt_solref", "f8", NJNT, 2, 10999),
    ("jnt_solimp", "f8", NJNT, 5, 11479),
    ("jnt_pos", "f8", NJNT, 3, 12679),
    ("jnt_axis", "f8", NJNT, 3, 13399),
    ("jnt_range", "f8", NJNT, 2, 14839),
    ("jnt_actfrcrange", "f8", NJNT, 2, 15319),
    ("jnt_margin", "f8", NJNT, 1, 15799),
    ("dof_bodyid", "i4", NV, 1, 16039),
    ("dof_jntid", "i4", NV, 1, 16179),
    ("dof_parentid", "i4", NV, 1, 16319),
    ("dof_Madr", "i4", NV, 1, 16599),
    ("dof_solref", "f8", NV, 2, 16879),
    ("dof_solimp", "f8", NV, 5, 17439),
    ("dof_frictionloss", "f8", NV, 1, 18839),
    ("dof_armature", "f8", NV, 1, 19119),
    ("dof_damping", "f8", NV, 1, 19399),
    ("dof_invweight0", "f8", NV, 1, 20239),
    ("geom_type", "i4", NGEOM, 1, 21099),
    ("geom_contype", "i4", NGEOM, 1, 21235),
    ("geom_conaffinity", "i4", NGEOM, 1, 21371),
    ("geom_condim", "i4", NGEOM, 1, 21507),
    ("geom_bodyid", "i4", NGEOM, 1, 21643),
    ("geom_size", "f8", NGEOM, 3, 24669),
    ("geom_rbound", "f8", NGEOM, 1, 27117),
    ("geom_pos", "f8", NGEOM, 3, 27389),
    ("geom_quat", "f8", NGEOM, 4, 28205),
    ("geom_friction", "f8", NGEOM, 3, 29293),
    ("geom_margin", "f8", NGEOM, 1, 30109),
    ("geom_gap", "f8", NGEOM, 1, 30381),
    ("pair_dim", "i4", NPAIR, 1, 37792),
    ("pair_geom1", "i4", NPAIR, 1, 39800),
    ("pair_geom2", "i4", NPAIR, 1, 41808),
    ("pair_solref", "f8", NPAIR, 2, 45824),
    ("pair_solreffriction", "f8", NPAIR, 2, 53856),
    ("pair_solimp", "f8", NPAIR, 5, 61888),
    ("pair_margin", "f8", NPAIR, 1, 81968),
    ("pair_gap", "f8", NPAIR, 1, 85984),
    ("pair_friction", "f8", NPAIR, 5, 94016),
    ("actuator_trnid", "i4", NU, 2, 115372),
    ("actuator_gainprm", "f8", NU, 10, 118156),
    ("actuator_biasprm", "f8", NU, 10, 120476),
    ("actuator_ctrlrange", "f8", NU, 2, 125580),
    ("key_qpos", "f8", NKEY, NQ, 129836),
    ("key_ctrl", "f8", NKEY, NU, 130972),
]
NAMES_AT = 134048  # the names buffer: model name, then bodies, joints, geoms, ... (null-separated)


def read_mjb(path):
    b = Path(path).read_bytes()
    sha = hashlib.sha256(b).hexdigest()
    if sha != MJB_SHA256:
        raise SystemExit(f"{path}: sha256 {sha} is not the mjlab G1 model's ({MJB_SHA256})")
    hdr = np.frombuffer(b[:20], np.int32)
    assert hdr.tolist() == [54321, 8, 98, 3017000, 485], hdr
    sizes = np.frombuffer(b[20:20 + 8 * 98], np.int64)
    assert sizes[:3].tolist() == [NQ, NV, NU] and sizes[6] == NBODY and sizes[11] == NJNT and sizes[17] == NGEOM
    assert sizes[57] == NPAIR
    m = {}
    for name, dt, r, c, off in LAYOUT:
        n = r * c
        a = np.frombuffer(b[off:off + n * np.dtype(dt).itemsize], dt).copy()
        m[name] = a.reshape(r, c) if c > 1 or r == 1 and c > 1 else a.reshape(r) if c == 1 else a.reshape(r, c)
    m["opt_real"], m["opt_int"], m["stat"], m["qpos0"] = (m["opt_real"].ravel(), m["opt_int"].ravel(),
                                                         m["stat"].ravel(), m["qpos0"].ravel())
    names = b[NAMES_AT:NAMES_AT + 3000].split(b"\x00")
    assert names[0] == b"g1 mjx flat terrain scene", names[:2]
    m["body_names"] = [x.decode() for x in names[1:1 + NBODY]]
    m["joint_names"] = [x.decode() for x in names[1 + NBODY:1 + NBODY + NJNT]]
    m["geom_names"] = [x.decode() for x in names[1 + NBODY + NJNT:1 + NBODY + NJNT + NGEOM]]
    return m, sha


def check(m):
    """Anchors that hold only when every array was read at its true offset."""
    assert m["body_names"][0] == "world" and m["body_names"][16] == "torso_link", m["body_names"]
    assert m["joint_names"][0] == "floating_base_joint" and m["geom_names"][0] == "floor"
    assert m["body_parentid"].tolist()[:8] == [0, 0, 1, 2, 3, 4, 5, 6]
    for key in ("body_quat", "body_iquat", "geom_quat"):
        assert np.allclose(np.linalg.norm(m[key], axis=1), 1.0, atol=1e-9), key
    assert np.allclose(np.linalg.norm(m["jnt_axis"][1:], axis=1), 1.0)
    assert m["jnt_type"].tolist() == [0] + [3] * 29  # free, then hinges
    assert (m["jnt_limited"][1:] == 1).all() and (m["jnt_actfrclimited"][1:] == 1).all()
    assert (m["jnt_range"][1:, 0] < m["jnt_range"][1:, 1]).all()
    assert (m["jnt_actfrcrange"][1:, 0] == -m["jnt_actfrcrange"][1:, 1]).all()
    assert set(m["geom_type"].tolist()) == {0, 2, 3}  # plane, sphere, capsule
    assert set(m["pair_dim"].tolist()) == {1, 3}
    assert (m["pair_geom1"] < NGEOM).all() and (m["pair_geom2"] < NGEOM).all()
    assert (m["pair_friction"][:, 0] == m["pair_friction"][:, 1]).all()
    assert (m["pair_margin"] == 0).all() and (m["pair_gap"] == 0).all()
    assert (m["actuator_trnid"][:, 0] == np.arange(1, NU + 1)).all()
    kp = m["actuator_gainprm"][:, 0]
    assert np.allclose(kp, -m["actuator_biasprm"][:, 1]) and (m["actuator_biasprm"][:, 2] < 0).all()
    arm = m["dof_armature"][6:]
    assert np.allclose(kp, arm * (2 * math.pi * 10) ** 2, rtol=1e-12)  # mjlab: kp = armature (2 pi 10 Hz)^2
    assert m["opt_real"][0] == 0.005 and m["opt_int"][0] == 3 and m["opt_int"][1] == 0 and m["opt_int"][3] == 2
    assert abs(m["stat"][0] - 3.2641499757457035) < 1e-15  # meaninertia
    assert m["key_qpos"][0, 2] == 0.783675 and m["key_qpos"][1, 2] == 0.755


def derive(m):
    """The per-model tables the step uses, in the engine's terms (dof-indexed actuator gains, limits, foot pairs)."""
    nb = NBODY
    depth = np.zeros(nb, np.int32)
    for b in range(1, nb):
        depth[b] = depth[m["body_parentid"][b]] + 1
    kp, kv, frclim = np.zeros(NV), np.zeros(NV), np.full(NV, np.inf)
    for a in range(NU):
        j = m["actuator_trnid"][a, 0]
        d = m["jnt_dofadr"][j]
        assert d == 6 + a
        kp[d], kv[d] = m["actuator_gainprm"][a, 0], -m["actuator_biasprm"][a, 2]
        frclim[d] = m["jnt_actfrcrange"][j, 1]
    jrange = np.zeros((NV, 2))
    for j in range(1, NJNT):
        jrange[m["jnt_dofadr"][j]] = m["jnt_range"][j]
    # contact pairs with geom1 of the lower type (MuJoCo's collision table order: plane < sphere < capsule)
    g1, g2 = m["pair_geom1"].copy(), m["pair_geom2"].copy()
    sw = m["geom_type"][g1] > m["geom_type"][g2]
    g1[sw], g2[sw] = m["pair_geom2"][sw], m["pair_geom1"][sw]
    names = m["geom_names"]
    foot = np.array([int(names[g1[p]] == "floor" and "foot" in names[g2[p]]) for p in range(NPAIR)], np.int32)
    child = np.zeros((nb, 3), np.int32)
    nchild = np.zeros(nb, np.int32)
    for b in range(2, nb):
        p = m["body_parentid"][b]
        child[p, nchild[p]] = b
        nchild[p] += 1
    dofmask = np.zeros(nb, np.uint64)  # bit i: dof i moves body b (its own dofs and its ancestors')
    for b in range(1, nb):
        k, bits = b, 0
        while k >= 1:
            for i in range(m["body_dofadr"][k], m["body_dofadr"][k] + m["body_dofnum"][k]):
                bits |= 1 << int(i)
            k = m["body_parentid"][k]
        dofmask[b] = bits
    return dict(body_nchild=nchild, body_child=child, body_dofmask=dofmask, body_depth=depth, dof_kp=kp, dof_kv=kv, dof_frclim=frclim, dof_range=jrange, pair_g1=g1, pair_g2=g2,
                pair_foot=foot, torso_body=np.int32(m["body_names"].index("torso_link")))


def carr(name, ctype, a, per_line=6):
    a = np.asarray(a).ravel()
    if ctype == "double":
        vals = [repr(float(x)) if np.isfinite(x) else "1e30" for x in a]  # (no limit: a float-safe 1e30)
    elif ctype == "unsigned long long":
        vals = [f"{int(x)}ull" for x in a]
    else:
        vals = [str(int(x)) for x in a]
    lines = [", ".join(vals[i:i + per_line]) for i in range(0, len(vals), per_line)]
    ctype = "NB_REAL" if ctype == "double" else ctype
    return f"NB_MODEL_CONST {ctype} {name}[{len(a)}] = {{\n  " + ",\n  ".join(lines) + "};\n"


def write_header(m, d, path, sha):
    """The model as C arrays (float64 values, exact decimal round trip). The oracle instantiates them as double
    (NB_REAL's default); the CUDA library defines NB_REAL as float, so the compiler rounds each literal once."""
    geoms = sorted(set(d["pair_g1"].tolist()) | set(d["pair_g2"].tolist()))
    assert geoms == list(range(NGEOM))
    pw = m["pair_friction"][:, 0]
    parts = [
        "// Generated by oracle/mjb_extract.py from the mjlab Unitree G1 model (g1_train.mjb, MuJoCo 3.17 binary,\n"
        f"// sha256 {sha}). Model data: Unitree Robotics, BSD-3-Clause (nablaengine_b200/model/LICENSE).\n"
        "// Do not edit: regenerate with the script.\n#pragma once\n",
        "#ifndef NB_MODEL_CONST\n#define NB_MODEL_CONST static const\n#endif\n"
        "#ifndef NB_REAL  // the element type of the real-valued tables (the CUDA library: float)\n#define NB_REAL double\n"
        "#endif\n",
        f"#define G1_NQ {NQ}\n#define G1_NV {NV}\n#define G1_NU {NU}\n#define G1_NBODY {NBODY}\n"
        f"#define G1_NGEOM {NGEOM}\n#define G1_NPAIR {NPAIR}\n#define G1_TORSO {int(d['torso_body'])}\n"
        f"#define G1_MAXDEPTH {int(d['body_depth'].max())}\n",
        f"#define G1_TIMESTEP {float(m['opt_real'][0])!r}\n#define G1_IMPRATIO {float(m['opt_real'][1])!r}\n"
        f"#define G1_TOLERANCE {float(m['opt_real'][2])!r}\n#define G1_MEANINERTIA {float(m['stat'][0])!r}\n"
        f"#define G1_GRAVITY_Z {float(m['opt_real'][9])!r}\n",
        carr("g1_body_parent", "int", m["body_parentid"]),
        carr("g1_body_depth", "int", d["body_depth"]),
        carr("g1_body_dofadr", "int", m["body_dofadr"]),
        carr("g1_body_nchild", "int", d["body_nchild"]),
        carr("g1_body_child", "int", d["body_child"]),
        carr("g1_body_dofmask", "unsigned long long", d["body_dofmask"], 4),
        carr("g1_body_qposadr", "int", [0, 0] + [m["jnt_qposadr"][m["body_jntadr"][b]] for b in range(2, NBODY)]),
        carr("g1_body_pos", "double", m["body_pos"]),
        carr("g1_body_quat", "double", m["body_quat"]),
        carr("g1_body_ipos", "double", m["body_ipos"]),
        carr("g1_body_iquat", "double", m["body_iquat"]),
        carr("g1_body_mass", "double", m["body_mass"]),
        carr("g1_body_inertia", "double", m["body_inertia"]),
        carr("g1_body_invweight0", "double", m["body_invweight0"][:, 0]),
        carr("g1_body_axis", "double", np.vstack([np.zeros((2, 3)),
                                                  m["jnt_axis"][[m["body_jntadr"][b] for b in range(2, NBODY)]]])),
        carr("g1_dof_body", "int", m["dof_bodyid"]),
        carr("g1_dof_armature", "double", m["dof_armature"]),
        carr("g1_dof_damping", "double", m["dof_damping"]),
        carr("g1_dof_invweight0", "double", m["dof_invweight0"]),
        carr("g1_dof_kp", "double", d["dof_kp"]),
        carr("g1_dof_kv", "double", d["dof_kv"]),
        carr("g1_dof_frclim", "double", d["dof_frclim"]),
        carr("g1_dof_range", "double", d["dof_range"]),
        carr("g1_jnt_solref", "double", m["jnt_solref"][1]),
        carr("g1_jnt_solimp", "double", m["jnt_solimp"][1]),
        carr("g1_geom_type", "int", m["geom_type"]),
        carr("g1_geom_body", "int", m["geom_bodyid"]),
        carr("g1_geom_size", "double", m["geom_size"]),
        carr("g1_geom_pos", "double", m["geom_pos"]),
        carr("g1_geom_quat", "double", m["geom_quat"]),
        carr("g1_geom_rbound", "double", m["geom_rbound"]),
        carr("g1_pair_g1", "int", d["pair_g1"], 16),
        carr("g1_pair_g2", "int", d["pair_g2"], 16),
        carr("g1_pair_dim", "int", m["pair_dim"], 16),
        carr("g1_pair_foot", "int", d["pair_foot"], 16),
        carr("g1_pair_mu", "double", pw, 8),
        carr("g1_pair_solref", "double", m["pair_solref"][0]),
        carr("g1_pair_solimp", "double", m["pair_solimp"][0]),
        carr("g1_key_qpos", "double", m["key_qpos"]),
        carr("g1_ctrlrange", "double", m["actuator_ctrlrange"]),
    ]
    path.write_text("".join(parts))


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--mjb", required=True)
    ap.add_argument("--check", action="store_true", help="verify the committed outputs instead of writing them")
    a = ap.parse_args()
    m, sha = read_mjb(a.mjb)
    check(m)
    d = derive(m)
    # every pair shares one solref / solimp (asserted so a single constant serves all pairs)
    assert (m["pair_solref"] == m["pair_solref"][0]).all() and (m["pair_solimp"] == m["pair_solimp"][0]).all()
    assert (m["jnt_solref"][1:] == m["jnt_solref"][1]).all() and (m["jnt_solimp"][1:] == m["jnt_solimp"][1]).all()
    assert not m["dof_frictionloss"].any() and not m["dof_damping"].any() and not m["jnt_margin"].any()
    assert m["pair_solimp"][0][4] == 2.0 and m["jnt_solimp"][1][4] == 2.0  # the kernels fold the power-2 impedance
    out = {k: v for k, v in m.items() if isinstance(v, np.ndarray)}
    out.update({k: np.asarray(v) for k, v in d.items()})
    for k in ("body_names", "joint_names", "geom_names"):
        out[k] = np.asarray(m[k])
    npz = REPO / "nablaengine_b200" / "model" / "g1_model.npz"
    hdr = REPO / "nablaengine_b200" / "csrc" / "g1_model_data.h"
    if a.check:
        old = np.load(npz)
        for k, v in out.items():
            assert np.array_equal(old[k], v), k
        tmp = hdr.with_suffix(".check")
        write_header(m, d, tmp, sha)
        same = tmp.read_text() == hdr.read_text()
        tmp.unlink()
        assert same, "header differs"
        print("committed model files match the .mjb")
        return
    np.savez(npz, **out)
    write_header(m, d, hdr, sha)
    (REPO / "nablaengine_b200" / "model" / "g1_model.json").write_text(json.dumps(
        {"source": "mjlab Unitree G1 (g1_train.mjb, MuJoCo 3.17.0 binary)", "mjb_sha256": sha,
         "npz_sha256": hashlib.sha256(npz.read_bytes()).hexdigest(),
         "header_sha256": hashlib.sha256(hdr.read_bytes()).hexdigest(),
         "nq": NQ, "nv": NV, "nu": NU, "nbody": NBODY, "ngeom": NGEOM, "npair": NPAIR,
         "foot_pairs": [int(p) for p in np.nonzero(d["pair_foot"])[0]], "torso_body": "torso_link"}, indent=1) + "\n")
    print(f"wrote {npz} and {hdr}")


if __name__ == "__main__":
    main()
