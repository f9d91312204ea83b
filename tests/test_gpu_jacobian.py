"""The full step Jacobian (B, 71, 99) on the GPU (nb_g1_jacobian / torch_ffi.jacobian).

Parity: against the reference's MuJoCo C float64 FD Jacobian (truth_jac.npz, 16 G0 states; the reference's scorer
benchmarks/bench/accuracy/gradient.py jacobian_errors: Frobenius relative error per input block, floored at the
truth's per-column floor), against the float64 oracle's central differences on synthetic multi-contact states, and
row by row against the VJP entry (the reference's Jacobian is 71 backward calls, scripts/paper_bench/ours.py:99-110).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

KEYS = ("qpos", "qvel", "qacc_warmstart", "ctrl", "friction", "com")
BLOCKS = dict(qpos=slice(0, 35), qvel=slice(35, 70), ctrl=slice(70, 99))
# Frobenius relative error bounds per block (the gradient check's p99 bounds, scripts/gradient_check.py:53)
BOUND = dict(qpos=2e-3, qvel=5e-4, ctrl=1e-4)


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _frob(J, Jt, floor_cols=None):
    out = {}
    for name, sl in BLOCKS.items():
        e = np.linalg.norm((J[:, :, sl] - Jt[:, :, sl]).reshape(len(J), -1), axis=1)
        if floor_cols is not None:
            e = np.maximum(e, np.linalg.norm(floor_cols[:, sl], axis=1))
        out[name] = e / np.maximum(np.linalg.norm(Jt[:, :, sl].reshape(len(J), -1), axis=1), 1e-9)
    return out


def test_jacobian_matches_mujoco_fd_truth(golden):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    d = golden("truth_jac.npz")
    t = [torch.from_numpy(np.ascontiguousarray(d[k], np.float32)).cuda() for k in KEYS]
    tape = torch_ffi.forward(*t, iterations=50, tape=True)[4]
    J, info = torch_ffi.jacobian(tape, t[4], t[5])
    J = J.cpu().numpy().astype(np.float64)
    assert np.isfinite(J).all() and (info.cpu().numpy() & (1 << 13)).sum() == 0
    err = _frob(J, d["jacobian"].astype(np.float64), d["jacobian_dcol"].astype(np.float64))
    print({k: (float(np.median(v)), float(v.max())) for k, v in err.items()})
    for name, e in err.items():
        assert e.max() <= BOUND[name], (name, e)


def test_jacobian_matches_oracle_fd_on_synthetic_states():
    torch = _cuda()
    import oracle
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("vjp", B=8)
    s["qpos"][:4, 2] -= 0.1  # multi-contact feet
    keys = ("qpos", "qvel", "warm", "ctrl", "friction", "com")
    Jf = oracle.fd_jacobian(*(s[k] for k in keys))
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in keys]
    tape = torch_ffi.forward(*t, iterations=50, tape=True)[4]
    J = torch_ffi.jacobian(tape, t[4], t[5])[0].cpu().numpy().astype(np.float64)
    err = _frob(J, Jf)
    print({k: (float(np.median(v)), float(v.max())) for k, v in err.items()})
    for name, e in err.items():
        assert np.median(e) <= BOUND[name], (name, e)


# The Jacobian kernel carries the 70 tangent-basis cotangents of a world on the lanes of one block and backward one
# cotangent on a warp: the same mathematics in another order of float32 operations (and the quaternion rows as
# combinations of the rotation cotangents). Per (world, row): the relative difference over the 99 tangent columns.
ROW_TOL = {"median": 1e-5, "p99": 1e-3, "max": 1e-2}


def _backward_rows(torch_ffi, torch, tape, t, rows, **kw):
    """(B, len(rows), 99) float64: backward's VJP of each row's unit cotangent in the Jacobian's tangent columns."""
    B = t[0].shape[0]
    xi = t[0][:, 3:7].double()
    out = []
    for r in rows:
        cq, cv = torch.zeros(B, 36, device="cuda"), torch.zeros(B, 35, device="cuda")
        if r < 36:
            cq[:, r] = 1.0
        else:
            cv[:, r - 36] = 1.0
        gq, gv, gu, _ = torch_ffi.backward(tape, t[4], t[5], cq, cv, **kw)
        # the qpos block: qpos form -> tangent, 1/2 Im(xi* (x) g) / |xi|^2
        g = gq.double()
        w, x, y, z = xi.unbind(1)
        a, b, c, e = g[:, 3:7].unbind(1)
        rot = 0.5 * torch.stack([w * b - x * a - y * e + z * c, w * c + x * e - y * a - z * b,
                                 w * e - x * c + y * b - z * a], 1) / (xi * xi).sum(1, keepdim=True)
        out.append(torch.cat([g[:, :3], rot, g[:, 7:], gv.double(), gu.double()], 1))
    return torch.stack(out, 1)


def _assert_rows_close(J, ref):
    num = (J.double() - ref).norm(dim=2)
    rel = (num / ref.norm(dim=2).clamp_min(1e-9)).flatten().cpu().numpy()
    stats = {"median": float(np.median(rel)), "p99": float(np.percentile(rel, 99)), "max": float(rel.max())}
    print(stats)
    for k, bound in ROW_TOL.items():
        assert stats[k] <= bound, (k, stats)


def test_jacobian_rows_equal_the_vjp_of_unit_cotangents(golden):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    d = golden("truth_jac.npz")
    t = [torch.from_numpy(np.ascontiguousarray(d[k], np.float32)).cuda() for k in KEYS]
    tape = torch_ffi.forward(*t, tape=True)[4]
    J = torch_ffi.jacobian(tape, t[4], t[5], clamp_kv=0, normal=3)[0]
    rows = (0, 4, 12, 40, 70)
    ref = _backward_rows(torch_ffi, torch, tape, t, rows, clamp_kv=0, normal=3)
    _assert_rows_close(J[:, list(rows)], ref)


def test_jacobian_argument_errors(golden):
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    d = golden("truth_jac.npz")
    t = [torch.from_numpy(np.ascontiguousarray(d[k][:2], np.float32)).cuda() for k in KEYS]
    tape = torch_ffi.forward(*t, tape=True)[4]
    with pytest.raises(TypeError):
        torch_ffi.jacobian(tape.double(), t[4], t[5])
    with pytest.raises(ValueError):
        torch_ffi.jacobian(tape, t[4], t[5], clamp_kv=2)
    J, info = torch_ffi.jacobian(tape[:0], t[4][:0], t[5][:0])
    assert J.shape == (0, 71, 99)


@pytest.mark.parametrize("substeps,clamp_kv,normal", [(1, 1, 0), (3, 1, 0), (4, 2, 2), (4, 0, 1)])
def test_jacobian_rows_equal_backward_ragged_batch(substeps, clamp_kv, normal):
    """A batch of 37 worlds (no multiple of anything in the launch), odd numbers of records and the gradient modes:
    every row of the Jacobian equals backward's VJP of its unit cotangent within ROW_TOL."""
    torch = _cuda()
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("vjp", B=37)
    s["qpos"][:9, 2] -= 0.08
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda()
         for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    tape = torch_ffi.forward(*t, substeps=substeps, tape=True)[4]
    mode = dict(substeps=substeps, clamp_kv=clamp_kv, normal=normal)
    if clamp_kv == 2:
        mode.update(ctrl=t[3], clamp_soft=0.2)
    J = torch_ffi.jacobian(tape, t[4], t[5], **mode)[0]
    ref = _backward_rows(torch_ffi, torch, tape, t, range(71), **mode)
    _assert_rows_close(J, ref)


def test_jacobian_many_contacts_and_long_steps():
    """Worlds lowered into the floor (records of more than 32 contacts: the preparation's contact items take two
    rounds of the block's threads) and a step of 9 substeps: every row equals backward's VJP within ROW_TOL."""
    torch = _cuda()
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("vjp", B=24, seed_offset=7)
    s["qpos"][:, 2] -= np.linspace(0.0, 0.45, 24, dtype=np.float32)
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda()
         for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    out = torch_ffi.forward(*t, substeps=9, tape=True)
    info, tape = out[3], out[4]
    ncon = info[:, 1].cpu().numpy()
    print("contacts of the last substep: max", int(ncon.max()), "worlds above 32:", int((ncon > 32).sum()))
    assert (ncon > 32).sum() >= 3
    J, jinfo = torch_ffi.jacobian(tape, t[4], t[5], substeps=9)
    assert torch.isfinite(J).all()
    ref = _backward_rows(torch_ffi, torch, tape, t, range(71), substeps=9, clamp_kv=1, normal=0)
    _assert_rows_close(J, ref)
