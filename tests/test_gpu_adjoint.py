"""The analytic adjoint (VJP of one control step) on the GPU, through nb_g1_adjoint / torch_ffi.backward.

Gradient parity follows the reference's gradient check (scripts/gradient_check.py, THRESHOLDS / COS_P1 :53-54, scorer
benchmarks/bench/accuracy/gradient.py block_errors :175): the VJPs of the three stored output cotangents of each
truth state against the MuJoCo C float64 central-difference truth (h = 1e-6) in the tangent basis (qpos tangent 35 |
qvel 35 | ctrl 29), per block on its valid columns, e = |g - fd| / max(|fd|, 1e-9) floored at the truth's own floor
|fd(1e-7) - fd(1e-6)| / max(|fd|, 1e-9); per group (G0, G4, G5, G6) on the model_ok states: p99(e) <= 2e-3 / 5e-4 /
1e-4 (qpos / qvel / ctrl) and the 1st percentile of the cosine >= 0.99999. The forward runs 50 Newton iterations (the
truth's reference count), the adjoint in the exact mode (clamp_kv=1, normal=0, the truth's semantics).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

THRESHOLDS = dict(qpos=2e-3, qvel=5e-4, ctrl=1e-4)
COS_P1 = 0.99999
BLOCKS = dict(qpos=slice(0, 35), qvel=slice(35, 70), ctrl=slice(70, 99))
KEYS = ("qpos", "qvel", "qacc_warmstart", "ctrl", "friction", "com")


def qpos_tangent(g, q):
    """qpos-form cotangents (S, 36) -> dof-tangent form (S, 35) at the states q: the quaternion part 1/2 Im(xi* (x) g)
    / |xi|^2 (reference src/nablaengine/reference/adjoint_groups.py:218)."""
    xi, gq = np.asarray(q, np.float64)[:, 3:7], np.asarray(g, np.float64)[:, 3:7]
    w, x, y, z = xi.T
    a, b, c, d = gq.T
    v = np.stack([w * b - x * a - y * d + z * c, w * c + x * d - y * a - z * b, w * d - x * c + y * b - z * a], 1)
    g = np.asarray(g, np.float64)
    return np.concatenate([g[:, :3], 0.5 * v / np.sum(xi * xi, 1, keepdims=True), g[:, 7:]], 1)


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _vjps(d, iterations=50, clamp_kv=1, normal=0):
    """(N, 3, 99) tangent-form VJPs of the fixture's three cotangents, and the backward infos."""
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    t = [torch.from_numpy(np.ascontiguousarray(d[k], np.float32)).cuda() for k in KEYS]
    q1, v1, w1, info, tape = torch_ffi.forward(*t, iterations=iterations, tape=True)
    out, infos = [], []
    ctrl = t[3] if clamp_kv == 2 else None
    for c in range(d["cot_qpos"].shape[1]):
        cq = torch.from_numpy(np.ascontiguousarray(d["cot_qpos"][:, c], np.float32)).cuda()
        cv = torch.from_numpy(np.ascontiguousarray(d["cot_qvel"][:, c], np.float32)).cuda()
        gq, gv, gu, binfo = torch_ffi.backward(tape, t[4], t[5], cq, cv, clamp_kv=clamp_kv, normal=normal, ctrl=ctrl)
        gq = qpos_tangent(gq.cpu().numpy(), d["qpos"])
        out.append(np.concatenate([gq, gv.cpu().numpy().astype(np.float64), gu.cpu().numpy().astype(np.float64)], 1))
        infos.append(binfo.cpu().numpy())
    return np.stack(out, 1), np.stack(infos, 1)


def _block_errors(g, fd, floor, valid):
    """{block: (floored e (N, C), cos (N, C))} on each block's valid columns (nan where a state has none)."""
    res = {}
    for name, sl in BLOCKS.items():
        e = np.full(g.shape[:2], np.nan)
        cos = np.full(g.shape[:2], np.nan)
        for w in range(len(g)):
            v = valid[w, sl]
            if not v.any():
                continue
            a, b, f = g[w, :, sl][:, v], fd[w, :, sl][:, v], floor[w, :, sl][:, v]
            nb = np.linalg.norm(b, axis=1)
            raw = np.linalg.norm(a - b, axis=1) / np.maximum(nb, 1e-9)
            flo = np.linalg.norm(f - b, axis=1) / np.maximum(nb, 1e-9)
            e[w] = np.maximum(raw, flo)
            cos[w] = np.sum(a * b, 1) / np.maximum(np.linalg.norm(a, axis=1) * nb, 1e-30)
        res[name] = (e, cos)
    return res


@pytest.fixture(scope="module")
def truth(golden):
    return golden("truth_grad.npz")


@pytest.fixture(scope="module")
def exact(truth):
    return _vjps(truth)


def _report(truth, g, groups):
    valid = truth["bad"] == 0
    err = _block_errors(g, truth["fd_vjp"], truth["fd_vjp_floor"], valid)
    ok = truth["model_flags"] == 0
    rows = {}
    for grp in groups:
        m = truth[f"group_{grp}"] & ok
        for b, (e, cos) in err.items():
            ee, cc = e[m].ravel(), cos[m].ravel()
            keep = np.isfinite(ee)
            rows[(grp, b)] = (int(keep.sum()), float(np.median(ee[keep])), float(np.quantile(ee[keep], 0.99)),
                              float(np.quantile(cc[keep], 0.01)))
    return rows


def test_vjp_matches_fd_truth_exact_mode(truth, exact):
    g, infos = exact
    assert np.isfinite(g).all()
    rows = _report(truth, g, ("G0", "G4", "G5", "G6"))
    lines = [f"{grp} {b}: n={n} median={med:.2e} p99={p99:.2e} cos_p1={c:.7f}" for (grp, b), (n, med, p99, c) in
             rows.items()]
    print("\n".join(lines))
    for (grp, b), (n, med, p99, c) in rows.items():
        assert n > 0, (grp, b)
        assert p99 <= THRESHOLDS[b], f"{grp} {b}: p99 {p99:.3e} > {THRESHOLDS[b]:.0e}\n" + "\n".join(lines)
        assert c >= COS_P1, f"{grp} {b}: cos p1 {c:.7f}\n" + "\n".join(lines)


def test_vjp_default_mode_on_unclamped_states(truth):
    """The interface default (clamp_kv=0, normal=3) equals the truth wherever no PD force is clamped and no self
    contact is within 1 mm: the G0 (normal) states."""
    g, _ = _vjps(truth, clamp_kv=0, normal=3)
    rows = _report(truth, g, ("G0",))
    for (grp, b), (n, med, p99, c) in rows.items():
        assert p99 <= THRESHOLDS[b], (grp, b, p99)
        assert c >= COS_P1, (grp, b, c)


def test_replay_has_no_mismatch(exact):
    _, infos = exact
    assert (infos & (1 << 13)).sum() == 0


def test_backward_is_deterministic_and_tape_leaves_forward_bitwise(truth):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    t = [torch.from_numpy(np.ascontiguousarray(truth[k], np.float32)).cuda() for k in KEYS]
    a = torch_ffi.forward(*t)
    b = torch_ffi.forward(*t, tape=True)
    for x, y in zip(a, b[:4]):
        assert torch.equal(x, y)
    tape = b[4]
    cq = torch.from_numpy(np.ascontiguousarray(truth["cot_qpos"][:, 0], np.float32)).cuda()
    cv = torch.from_numpy(np.ascontiguousarray(truth["cot_qvel"][:, 0], np.float32)).cuda()
    r1 = torch_ffi.backward(tape, t[4], t[5], cq, cv)
    r2 = torch_ffi.backward(tape, t[4], t[5], cq, cv)
    for x, y in zip(r1, r2):
        assert torch.equal(x, y)


def test_vjp_is_linear_in_the_cotangent(truth):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    t = [torch.from_numpy(np.ascontiguousarray(truth[k], np.float32)).cuda() for k in KEYS]
    tape = torch_ffi.forward(*t, tape=True)[4]
    cq = [torch.from_numpy(np.ascontiguousarray(truth["cot_qpos"][:, c], np.float32)).cuda() for c in range(2)]
    cv = [torch.from_numpy(np.ascontiguousarray(truth["cot_qvel"][:, c], np.float32)).cuda() for c in range(2)]
    g0 = torch_ffi.backward(tape, t[4], t[5], cq[0], cv[0])
    g1 = torch_ffi.backward(tape, t[4], t[5], cq[1], cv[1])
    gs = torch_ffi.backward(tape, t[4], t[5], cq[0] + 2 * cq[1], cv[0] + 2 * cv[1])
    for a, b, s in zip(g0[:3], g1[:3], gs[:3]):
        ref = a + 2 * b
        err = (s - ref).norm(dim=1) / ref.norm(dim=1).clamp_min(1e-9)
        assert float(err.median()) < 1e-5, float(err.median())


def test_vjp_matches_oracle_fd_on_synthetic_states():
    """The exact-mode VJP against central differences of the float64 oracle (converged, 2000 iterations) on seeded
    synthetic states of the gradient configuration (12 worlds, one random cotangent each)."""
    torch = _cuda()
    import oracle
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("vjp", B=12)
    keys = ("qpos", "qvel", "warm", "ctrl", "friction", "com")
    J = oracle.fd_jacobian(*(s[k] for k in keys))  # (B, 71, 99)
    rng = np.random.default_rng(7)
    cq, cv = rng.standard_normal((12, 36)), rng.standard_normal((12, 35))
    cq[:, 3:7] = 0.0  # the quaternion block's cotangent in qpos form
    fd = np.einsum("bi,bij->bj", np.concatenate([cq, cv], 1), J)
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in keys]
    tape = torch_ffi.forward(*t, iterations=50, tape=True)[4]
    gq, gv, gu, info = torch_ffi.backward(tape, t[4], t[5], torch.from_numpy(cq.astype(np.float32)).cuda(),
                                          torch.from_numpy(cv.astype(np.float32)).cuda(), clamp_kv=1, normal=0)
    g = np.concatenate([qpos_tangent(gq.cpu().numpy(), s["qpos"]), gv.cpu().numpy(), gu.cpu().numpy()], 1)
    for name, sl in BLOCKS.items():
        e = np.linalg.norm(g[:, sl] - fd[:, sl], axis=1) / np.maximum(np.linalg.norm(fd[:, sl], axis=1), 1e-9)
        assert np.median(e) < 1e-3, (name, np.median(e), e)


def test_autograd_step_equals_backward(truth):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    t = [torch.from_numpy(np.ascontiguousarray(truth[k][:32], np.float32)).cuda() for k in KEYS]
    q = t[0].clone().requires_grad_(True)
    v = t[1].clone().requires_grad_(True)
    u = t[3].clone().requires_grad_(True)
    q1, v1, w1 = torch_ffi.step(q, v, t[2], u, t[4], t[5], grad_decay=0.5)
    assert not w1.requires_grad
    cq = torch.from_numpy(np.ascontiguousarray(truth["cot_qpos"][:32, 0], np.float32)).cuda()
    cv = torch.from_numpy(np.ascontiguousarray(truth["cot_qvel"][:32, 0], np.float32)).cuda()
    ((q1 * cq).sum() + (v1 * cv).sum()).backward()
    tape = torch_ffi.forward(*t, tape=True)[4]
    gq, gv, gu, _ = torch_ffi.backward(tape, t[4], t[5], cq, cv)
    assert torch.equal(q.grad, gq * 0.5) and torch.equal(v.grad, gv * 0.5) and torch.equal(u.grad, gu)
    # scale_grad: identity forward, cotangent times gamma
    x = torch.ones(3, device="cuda", requires_grad=True)
    (torch_ffi.scale_grad({"a": x}, 0.25)["a"].sum()).backward()
    assert torch.equal(x.grad, torch.full_like(x, 0.25))


def test_backward_argument_errors(truth):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    t = [torch.from_numpy(np.ascontiguousarray(truth[k][:4], np.float32)).cuda() for k in KEYS]
    tape = torch_ffi.forward(*t, tape=True)[4]
    z36, z35 = torch.zeros(4, 36, device="cuda"), torch.zeros(4, 35, device="cuda")
    with pytest.raises(TypeError):
        torch_ffi.backward(tape, t[4], t[5], z36.double(), z35)
    with pytest.raises(TypeError):
        torch_ffi.backward(tape[:, :-1].contiguous(), t[4], t[5], z36, z35)
    with pytest.raises(ValueError):
        torch_ffi.backward(tape, t[4], t[5], z36, z35, clamp_kv=3)
    with pytest.raises(ValueError):
        torch_ffi.backward(tape, t[4], t[5], z36, z35, clamp_kv=2)  # the soft clamp needs ctrl
    with pytest.raises(ValueError):
        torch_ffi.backward(tape, t[4], t[5], z36, z35, clamp_soft=0.1)
    gq, gv, gu, info = torch_ffi.backward(tape, t[4], t[5], z36, z35, clamp_kv=2, ctrl=t[3])
    assert float(gq.abs().max()) == 0.0 and float(gu.abs().max()) == 0.0


@pytest.mark.parametrize("substeps", [1, 2])
def test_vjp_other_substep_counts_match_oracle_fd(substeps):
    """The adjoint of a control step of 1 or 2 substeps (the tape's records chained in reverse) against the float64
    oracle's central differences of the same step (exact mode, converged forward)."""
    torch = _cuda()
    import oracle
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("vjp", B=6)
    s["qpos"][:3, 2] -= 0.08
    keys = ("qpos", "qvel", "warm", "ctrl", "friction", "com")
    J = oracle.fd_jacobian(*(s[k] for k in keys), substeps=substeps)
    rng = np.random.default_rng(11)
    cq, cv = rng.standard_normal((6, 36)), rng.standard_normal((6, 35))
    cq[:, 3:7] = 0.0
    fd = np.einsum("bi,bij->bj", np.concatenate([cq, cv], 1), J)
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in keys]
    tape = torch_ffi.forward(*t, iterations=50, substeps=substeps, tape=True)[4]
    gq, gv, gu, info = torch_ffi.backward(tape, t[4], t[5], torch.from_numpy(cq.astype(np.float32)).cuda(),
                                          torch.from_numpy(cv.astype(np.float32)).cuda(), substeps=substeps,
                                          clamp_kv=1, normal=0)
    g = np.concatenate([qpos_tangent(gq.cpu().numpy(), s["qpos"]), gv.cpu().numpy(), gu.cpu().numpy()], 1)
    for name, sl in BLOCKS.items():
        e = np.linalg.norm(g[:, sl] - fd[:, sl], axis=1) / np.maximum(np.linalg.norm(fd[:, sl], axis=1), 1e-9)
        assert np.median(e) < 1e-3, (name, substeps, e)


def test_nonfinite_inputs_are_flagged_not_fatal():
    """A NaN state propagates to that world's outputs and gradients only, and the diagnostics count it."""
    torch = _cuda()
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("forward", B=8)
    t = [torch.from_numpy(s[k]).cuda() for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    t[1][2, 5] = float("nan")
    torch_ffi.read_diagnostics(reset=True)
    q1, v1, w1, info, tape = torch_ffi.forward(*t, tape=True)
    gq, gv, gu, binfo = torch_ffi.backward(tape, t[4], t[5], torch.zeros_like(q1), torch.ones_like(v1))
    ok = [i for i in range(8) if i != 2]
    assert torch.isfinite(v1[ok]).all() and torch.isfinite(gq[ok]).all()
    d = torch_ffi.read_diagnostics(reset=True)
    assert d["nonfinite_rows"] >= 1 and (int(binfo[2].item()) >> 16) & 7


# every (clamp_kv, normal) gradient mode of nb_g1_adjoint against central differences of the float64 oracle's
# surrogate step for that mode (oracle/g1_oracle.cpp: Mode, the derivative the mode defines): the reference's
# clamped (G4), limit-row (G5) and self-contact (G6) gradient states, and states whose self contacts come within
# 1 mm of degenerate (nu ~ 0.5 mm, tests/golden/mode_states.npz), where the normal options 2 and 3 differ from the
# exact derivative. Gates: on the reference's states, the gradient check's p99 bounds per block on the relative
# error per state; on the near-degenerate ones (max over states), NEAR_THRESHOLDS: there the contact normal n =
# (c2 - c1) / nu is computed in float32 from centres ~1 m from the origin with nu ~ 5e-4 m, so it carries a relative
# error ~ 1e-7 m / nu ~ 2e-4, which the contact's force and Hessian terms carry into the gradient. The exact normal
# derivative (normal 0) there is 1 / nu-sensitive: reported, not gated.
MODES = [(kv, n) for kv in (0, 1, 2) for n in (0, 1, 2, 3)]
NEAR_THRESHOLDS = dict(qpos=5e-3, qvel=2e-3, ctrl=1e-3)


@pytest.fixture(scope="module")
def mode_cases(golden):
    t = golden("truth_grad.npz")
    pick = np.concatenate([np.flatnonzero(t[f"group_{g}"] & (t["model_flags"] == 0))[:n]
                           for g, n in (("G4", 8), ("G5", 4), ("G6", 8))])
    s = {k: t[k][pick] for k in KEYS}
    s["cot_qpos"], s["cot_qvel"] = t["cot_qpos"][pick, 0], t["cot_qvel"][pick, 0]
    m = golden("mode_states.npz")
    rng = np.random.default_rng(5)
    n = m["qpos"].shape[0]
    cq, cv = rng.standard_normal((n, 36)).astype(np.float32), rng.standard_normal((n, 35)).astype(np.float32)
    cq[:, 3:7] = 0.0
    for k in KEYS:
        s[k] = np.concatenate([s[k], m[k]])
    s["cot_qpos"], s["cot_qvel"] = np.concatenate([s["cot_qpos"], cq]), np.concatenate([s["cot_qvel"], cv])
    near = np.zeros(len(s["qpos"]), bool)
    near[len(pick):] = True
    return s, near


def _mode_vjp(s, clamp_kv, normal):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in KEYS]
    tape = torch_ffi.forward(*t, iterations=50, tape=True)[4]
    cq = torch.from_numpy(np.ascontiguousarray(s["cot_qpos"], np.float32)).cuda()
    cv = torch.from_numpy(np.ascontiguousarray(s["cot_qvel"], np.float32)).cuda()
    gq, gv, gu, info = torch_ffi.backward(tape, t[4], t[5], cq, cv, clamp_kv=clamp_kv, normal=normal,
                                          ctrl=t[3] if clamp_kv == 2 else None)
    return np.concatenate([qpos_tangent(gq.cpu().numpy(), s["qpos"]), gv.cpu().numpy(), gu.cpu().numpy()], 1)


@pytest.mark.parametrize("clamp_kv,normal", MODES)
def test_every_gradient_mode_against_the_oracle_surrogate(mode_cases, clamp_kv, normal):
    import oracle
    s, near = mode_cases
    J = oracle.fd_jacobian_mode(*(s[k] for k in KEYS), clamp_kv=clamp_kv, normal=normal, soft=0.2)
    cot = np.concatenate([s["cot_qpos"], s["cot_qvel"]], 1).astype(np.float64)
    fd = np.einsum("bi,bij->bj", cot, J)
    g = _mode_vjp(s, clamp_kv, normal)
    lines = []
    for name, sl in BLOCKS.items():
        e = np.linalg.norm(g[:, sl] - fd[:, sl], axis=1) / np.maximum(np.linalg.norm(fd[:, sl], axis=1), 1e-9)
        lines.append(f"({clamp_kv}, {normal}) {name}: reference states p99 {np.quantile(e[~near], 0.99):.2e}, "
                     f"near-degenerate states max {e[near].max():.2e}")
        assert np.quantile(e[~near], 0.99) <= THRESHOLDS[name], "\n".join(lines)
        if normal != 0:
            assert e[near].max() <= NEAR_THRESHOLDS[name], "\n".join(lines)
    print("\n".join(lines))


def test_gradient_modes_differ_where_they_should(mode_cases):
    """The options change the gradient only where they act: the clamp options on states with a clamped actuator
    (G4), the options 2 and 3 only near a degenerate self contact (and there only where that contact carries a force:
    a contact whose rows are all inactive adds nothing to the gradient)."""
    s, near = mode_cases
    base = _mode_vjp(s, 1, 0)
    g4 = np.zeros(len(near), bool)
    g4[:8] = True
    for kv in (0, 2):
        d = np.abs(_mode_vjp(s, kv, 0) - base).max(1)
        assert (d[g4] > 0).any()
    for n in (2, 3):
        d = np.abs(_mode_vjp(s, 1, n) - base).max(1)
        print(f"normal {n}: gradient changed on {int((d[near] > 0).sum())} of {int(near.sum())} near-degenerate states")
        assert (d[near] > 0).any() and (d[~near] == 0).all()
