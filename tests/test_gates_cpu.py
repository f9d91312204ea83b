"""Self-test of the gradient gate (reference scripts/gradient_check.py: the gate must reject gradients perturbed by
3e-3): the float64 FD truth itself passes the per-block p99 / cosine gates of test_gpu_adjoint, and the same truth with
a 3e-3 relative perturbation fails them. CPU only: the gate is the checker, this shows it can fail."""
import numpy as np

from test_gpu_adjoint import COS_P1, THRESHOLDS, _report


def _fails(truth, g):
    rows = _report(truth, g, ("G0", "G4", "G5", "G6"))
    return [(grp, b) for (grp, b), (n, med, p99, c) in rows.items() if p99 > THRESHOLDS[b] or c < COS_P1]


def test_gate_accepts_the_truth_and_rejects_a_3e3_perturbation(golden):
    truth = golden("truth_grad.npz")
    fd = truth["fd_vjp"]
    assert _fails(truth, fd) == []
    rng = np.random.default_rng(0)
    noisy = fd * (1.0 + 3e-3 * rng.standard_normal(fd.shape))
    failed = _fails(truth, noisy)
    assert failed, "a 3e-3 perturbation passed every gate"
    assert any(b == "ctrl" for _, b in failed)
