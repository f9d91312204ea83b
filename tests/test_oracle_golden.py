"""The CPU oracle against the reference's golden data (CPU only): MuJoCo C float64 truth and MuJoCo Warp outputs."""
import numpy as np
import pytest

import oracle

INPUTS = ("qpos", "qvel", "qacc_warmstart", "ctrl", "friction", "com")


def rel_world(a, b):
    return np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-9)


def test_oracle_matches_mujoco_truth(golden):
    """Converged float64 oracle vs MuJoCo C float64 (2000 iterations, tolerance 1e-13) on the 256 check states."""
    g = golden("truth_check.npz")
    oq, ov, _, info = oracle.step(*(g[k] for k in INPUTS), iterations=2000, tol=1e-13)
    ok = g["model_flags"] == 0
    ev = rel_world(ov, g["check_out"][:, 36:])
    eq = np.abs(oq - g["check_out"][:, :36]).max(1)
    assert ok.sum() >= 250
    assert np.median(ev[ok]) < 1e-12, np.median(ev[ok])
    assert np.percentile(ev[ok], 95) < 1e-10
    assert ev[ok].max() < 1e-4
    assert np.median(eq[ok]) < 1e-14
    assert (info[:, 3] == 0).all()


def test_oracle_matches_mujoco_warp(golden):
    """float64 oracle at 50 iterations vs MuJoCo Warp 3.17 (float32, 50 iterations): the reference's own gate
    (scripts/engine_step_check.py: qvel median / p99 <= 5e-6 / 5e-5 on model-ok states), and its contact counts."""
    g = golden("mjw_sample.npz")
    oq, ov, _, info = oracle.step(*(g[k] for k in INPUTS), iterations=50, tol=1e-8)
    ok = g["model_flags"] == 0
    ev = rel_world(ov, g["out_qvel"])
    assert np.median(ev[ok]) <= 5e-6 and np.percentile(ev[ok], 99) <= 5e-5
    assert (info[:, 1] == g["ncon"][:, 3]).mean() >= 0.99
    assert (info[:, 2] == g["nefc"][:, 3]).mean() >= 0.99


def test_oracle_float32_close_to_float64(golden):
    g = golden("truth_check.npz")
    args = [g[k][:64] for k in INPUTS]
    _, v64, _, i64 = oracle.step(*args, iterations=10)
    _, v32, _, i32 = oracle.step(*args, iterations=10, precision=32)
    ev = rel_world(v32, v64)
    assert np.median(ev) < 1e-5
    assert (i64[:, 1] == i32[:, 1]).mean() > 0.95


def test_oracle_deterministic_and_thread_independent(golden):
    g = golden("mjw_sample.npz")
    args = [g[k][:64] for k in INPUTS]
    a = oracle.step(*args, threads=1)
    b = oracle.step(*args, threads=4)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_oracle_overflow_bits():
    """A world sunk into the floor overflows the 64-contact / 192-row capacity: bits 4 and 16, raw count kept."""
    from nablaengine_b200 import synthetic
    s = synthetic.states(4, 123)
    s["qpos"][:, 2] = 0.05  # pelvis at 5 cm: every sole, shin and hand capsule below the floor
    s["qpos"][:, 7:] = 0.0
    _, _, _, info = oracle.step(s["qpos"], s["qvel"], s["warm"], s["ctrl"], s["friction"], s["com"], substeps=1)
    assert (info[:, 1] > 0).all()
    over = info[:, 1] > 64
    assert ((info[:, 3] & 4) != 0).tolist() == over.tolist()


@pytest.mark.parametrize("h", [1e-6])
def test_oracle_fd_matches_truth_vjp(golden, h):
    """Central differences of the float64 oracle in the tangent basis reproduce the reference's FD VJP truth."""
    g = golden("truth_grad.npz")
    sel = np.nonzero(g["model_flags"] == 0)[0][:4]
    args = [g[k][sel] for k in INPUTS]
    J = oracle.fd_jacobian(*args, h=h)
    for j, w in enumerate(sel):
        for c in range(3):
            cot = np.concatenate([g["cot_qpos"][w, c], g["cot_qvel"][w, c]]).astype(np.float64)
            vjp = cot @ J[j]
            truth = g["fd_vjp"][w, c]
            valid = g["bad"][w] == 0
            err = np.abs(vjp - truth)[valid] / (np.abs(truth[valid]) + 1e-3 * np.abs(truth).max())
            assert np.median(err) < 1e-5, (w, c, np.median(err))


def test_oracle_fd_jacobian_matches_mujoco_jacobian_truth(golden):
    """The oracle's central-difference Jacobian (h = 1e-6, converged) against the reference's MuJoCo C float64 FD
    Jacobian of 16 G0 states (truth_jac.npz): Frobenius relative error per input block, floored at the truth's own
    per-column floor |J(1e-6) - J(1e-7)| (benchmarks/bench/accuracy/gradient.py jacobian_errors)."""
    import numpy as np
    import oracle
    d = golden("truth_jac.npz")
    J = oracle.fd_jacobian(d["qpos"], d["qvel"], d["qacc_warmstart"], d["ctrl"], d["friction"], d["com"])
    Jt = d["jacobian"].astype(np.float64)
    for sl in (slice(0, 35), slice(35, 70), slice(70, 99)):
        e = np.linalg.norm((J[:, :, sl] - Jt[:, :, sl]).reshape(len(J), -1), axis=1)
        nt = np.linalg.norm(Jt[:, :, sl].reshape(len(J), -1), axis=1)
        floor = np.linalg.norm(d["jacobian_dcol"][:, sl], axis=1)
        err = np.maximum(e, floor) / nt
        assert np.median(err) < 1e-5, (sl, err)
        assert err.max() < 1e-4, (sl, err)


def test_mode_surrogate_exact_mode_is_the_plain_step(golden):
    """The gradient-mode surrogate in the exact mode (clamp_kv=1, normal=0) is the plain step: its central
    differences equal fd_jacobian's bitwise; the frozen normal (normal=1) changes only states with self contacts."""
    g = golden("truth_grad.npz")
    keys = INPUTS
    idx = np.concatenate([np.flatnonzero(g["group_G0"])[:2], np.flatnonzero(g["group_G6"])[:2]])
    x = [g[k][idx] for k in keys]
    J0 = oracle.fd_jacobian(*x, iterations=200)
    J1 = oracle.fd_jacobian_mode(*x, clamp_kv=1, normal=0, iterations=200)
    assert np.array_equal(J0, J1)
    nu, _, _ = oracle.core_stats(*x)
    Jf = oracle.fd_jacobian_mode(*x, clamp_kv=1, normal=1, iterations=200)
    changed = np.abs(Jf - J1).reshape(len(idx), -1).max(1) > 0
    assert changed.tolist() == (nu < 1e299).tolist()
