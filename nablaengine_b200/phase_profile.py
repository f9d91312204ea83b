"""Phase profile of the forward and adjoint kernels (the reference's -DDK_PROFILE build, g1_engine/step.py:44-53,
318-328; adjoint.py:101-107): a build of the library with -DNB_PROFILE (lib/libnabla_g1_prof.so, not the product
library) in which lane 0 of every world adds the clock64() cycles of each phase to device counters. The cycles are a
world's own elapsed time per phase (its warp shares the SM with nine others), so the table gives shares, not a
kernel time. Needs a CUDA device.

    python -m nablaengine_b200.phase_profile [--worlds 4096] [--npz states.npz]
"""
import argparse
import ctypes

import numpy as np

from . import build, synthetic

# forward counters (nb_g1_step.cuh PROF / PROF_COUNT slots)
FWD = [(0, "kinematics + dof motions"), (1, "body terms"), (2, "mass matrix, forces"), (3, "qacc_smooth (factor)"),
       (4, "collision"), (5, "contact setup, rows"), (6, "Newton start"), (26, "Hessian: M, limit rows"),
       (27, "Hessian: group stiffness K"), (28, "Hessian: K S"), (29, "Hessian: support pairs"),
       (7, "Hessian: rest"), (8, "factorisation"), (9, "solve"), (10, "line search"), (11, "update, gradient"),
       (12, "implicitfast, integration"), (24, "wait before an iteration"), (25, "wait after convergence")]
ADJ = [(0, "integrator"), (1, "solves"), (2, "replay, motions"), (3, "(rows' geometry setup)"), (4, "contacts"),
       (5, "limit rows, actuators"), (6, "sweep")]
KEYS = ("qpos", "qvel", "warm", "ctrl", "friction", "com")


def _load():
    lib = ctypes.CDLL(str(build.build(extra=["-DNB_PROFILE"], out=build.PROFILE_LIB)))
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.nb_g1_forward.argtypes = [vp, i32] + [vp] * 6 + [i32, i32] + [vp] * 7
    lib.nb_g1_adjoint.argtypes = [vp, i32, i32] + [vp] * 10 + [ctypes.c_float, i32, i32]
    lib.nb_g1_upload.argtypes = [vp, vp]
    lib.nb_g1_sizes.argtypes = [vp]
    lib.nb_g1_work_bytes.argtypes, lib.nb_g1_work_bytes.restype = [i32], ctypes.c_longlong
    lib.nb_g1_profile_read.argtypes = [vp, i32]
    return lib


def _read(lib, n=32):
    buf = (ctypes.c_ulonglong * n)()
    rc = lib.nb_g1_profile_read(buf, n)
    if rc:
        raise RuntimeError(f"nb_g1_profile_read failed ({rc})")
    return np.array(list(buf), np.float64)


def _npz_states(path, worlds):
    """Forward inputs from an .npz of states (keys qpos, qvel, warm or qacc_warmstart, ctrl, friction, com)."""
    with np.load(path) as z:
        warm = "warm" if "warm" in z.files else "qacc_warmstart"
        s = {k: np.ascontiguousarray(z[w][:worlds]) for k, w in zip(KEYS, ("qpos", "qvel", warm, "ctrl",
                                                                           "friction", "com"))}
    return s


def run(worlds=4096, npz=None):
    import torch
    lib = _load()
    if lib.nb_g1_upload(None, None):
        raise RuntimeError("nb_g1_upload failed")
    sizes = (ctypes.c_longlong * 8)()
    lib.nb_g1_sizes(sizes)
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for cfg in (("npz",) if npz else ()) + ("forward", "vjp"):
        s = _npz_states(npz, worlds) if cfg == "npz" else synthetic.config_states(cfg, B=worlds)
        t = [torch.from_numpy(np.ascontiguousarray(s[k])).cuda() for k in KEYS]
        B = t[0].shape[0]
        out = [torch.empty((B, 36), device="cuda"), torch.empty((B, 35), device="cuda"),
               torch.empty((B, 35), device="cuda"), torch.empty((B, 4), dtype=torch.int32, device="cuda")]
        tape = torch.empty((B, 4 * sizes[6]), device="cuda")
        torch.cuda.synchronize()
        _read(lib)
        taped = cfg == "vjp"  # (the forward configuration runs without a tape, as the benchmark's forward)
        work = torch.empty((lib.nb_g1_work_bytes(B),), dtype=torch.uint8, device="cuda")  # the world order
        if lib.nb_g1_forward(st, B, *map(p, t), 10, 4, *map(p, out), None, p(tape) if taped else None, p(work)):
            raise RuntimeError("nb_g1_forward failed")
        torch.cuda.synchronize()
        v = _read(lib)
        ws = v[20]
        tot = sum(v[k] for k, _ in FWD)
        what = {"npz": npz, "forward": "configuration 2", "vjp": "configuration 3"}[cfg]
        print(f"== forward, {what}, B = {B}: {tot / ws:.0f} cycles per "
              f"world-substep; {v[16] / ws:.2f} Newton iterations, {v[17] / max(v[16], 1):.2f} line-search "
              f"evaluations per iteration, {v[18] / ws:.1f} contacts, {v[19] / ws:.1f} rows per world-substep")
        for k, name in FWD:
            print(f"   {name:28s} {v[k] / ws:9.0f}  {100 * v[k] / tot:5.1f} %")
        if cfg != "vjp":
            continue
        gq, gv = torch.zeros((B, 36), device="cuda"), 2 * out[1]
        r = [torch.empty((B, 36), device="cuda"), torch.empty((B, 35), device="cuda"),
             torch.empty((B, 29), device="cuda"), torch.empty((B,), dtype=torch.int32, device="cuda")]
        if lib.nb_g1_adjoint(st, B, 4, p(tape), p(t[4]), p(t[5]), p(gq), p(gv), *map(p, r), None,
                             ctypes.c_float(0.0), 1, 0):
            raise RuntimeError("nb_g1_adjoint failed")
        torch.cuda.synchronize()
        v = _read(lib)
        tot = sum(v[k] for k, _ in ADJ)
        print(f"== adjoint (exact mode), configuration 3, B = {B}: {tot / (4 * B):.0f} cycles per world-substep")
        for k, name in ADJ:
            print(f"   {name:28s} {v[k] / (4 * B):9.0f}  {100 * v[k] / tot:5.1f} %")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--worlds", type=int, default=4096)
    ap.add_argument("--npz", default=None, help="also profile the forward on these states (e.g. a corpus)")
    a = ap.parse_args(argv)
    run(a.worlds, a.npz)


if __name__ == "__main__":
    main()
