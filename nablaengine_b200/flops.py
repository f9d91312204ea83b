"""Algorithmic FP32 FLOP count of a control step from the kernel's own per-substep work counters.

The counters come from nb_g1_forward_stats (contacts kept c, constraint rows r, Newton iterations, line-search
evaluations, Hessian factorisations, broad-phase candidates). The per-unit costs are counted from the algorithm, not
measured (n = 35 dofs, 31 bodies, 502 pairs): a dense Cholesky factorisation is n^3 / 3 flops, a pair of triangular
solves or a dense mat-vec 2 n^2; the smooth dynamics (forward kinematics, Newton-Euler bias forces, the
composite-rigid-body mass matrix) about 21.5 kflop; a contact's Hessian term J' C J on a 16-dof support about 1.4 kflop,
its J v or J' f 96 flops (3 rows of 16); a row's impedance and reference acceleration about 50 flops.
"""
import numpy as np

N = 35
CHOL = N ** 3 // 3          # 14,291 flops per factorisation
SOLVE = 2 * N * N           # 2,450: forward + backward substitution
MATVEC = 2 * N * N          # 2,450
SMOOTH = 21_500
BROAD = 502 * 12            # bounding test of every pair
NARROW = 60                 # per candidate pair
CONTACT_SETUP = 480         # frame, moments, support of a contact
ROW_SETUP = 50
HESS_CONTACT = 1_400
JV_CONTACT = 96
LS_ROW = 6                  # per row and line-search evaluation
ROW_ITER = 10               # per row and Newton iteration (forces, cost)
IMPLICIT_EXTRA = 300


def per_substep(c, r, it, nls, nfact, ncand):
    """FLOPs of one world-substep from its counters (arrays broadcast)."""
    c, r, it, nls, nfact, ncand = (np.asarray(x, np.float64) for x in (c, r, it, nls, nfact, ncand))
    base = SMOOTH + CHOL + SOLVE + BROAD + NARROW * ncand + CONTACT_SETUP * c + ROW_SETUP * r
    init = 2 * (MATVEC + JV_CONTACT * c + ROW_ITER * r)  # warm start and qacc_smooth costs
    newton = it * (HESS_CONTACT * c + MATVEC + 2 * JV_CONTACT * c + ROW_ITER * r + SOLVE) + nfact * CHOL
    ls = nls * LS_ROW * r
    implicit = CHOL + SOLVE + MATVEC + IMPLICIT_EXTRA
    return base + init + newton + ls + implicit


def per_step(stats):
    """Total FLOPs of one control step of all worlds; stats (B, nsub, 8) int32 from nb_g1_forward_stats."""
    s = np.asarray(stats)
    return float(per_substep(s[..., 0], s[..., 1], s[..., 2], s[..., 3], s[..., 4], s[..., 5]).sum())
