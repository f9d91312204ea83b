"""The kinematics outputs and their VJP on the GPU (nb_g1_kinematics / _vjp, torch_ffi.kinematics and
step(kinematics=True)) against the float64 kinematics oracle (oracle/kinematics.py, its poses pinned to MuJoCo Warp)
and its central differences. Bounds as the reference's kinematics check (scripts/kinematics_check.py: xpos /
subtree_com 1e-5 m, xquat 1e-6, cvel 1e-5 p99 relative; VJP 1e-4 p99)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
OUT = ("qpos_n", "xpos", "xquat", "cvel", "subtree_com")


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _states(B=64):
    from nablaengine_b200 import synthetic
    s = synthetic.config_states("rollout", B=B)  # includes falling, tilted worlds
    return s["qpos"], s["qvel"], s["com"]


def test_kinematics_outputs_match_the_oracle():
    torch = _cuda()
    import kinematics as K
    from nablaengine_b200 import torch_ffi
    q, v, c = _states()
    q = q.copy()
    q[:, 3:7] *= 1.3  # an unnormalised quaternion: qpos_n normalises it
    ref = K.kinematics(q, v, c)
    out = torch_ffi.kinematics(*(torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (q, v, c)))
    got = {k: x.cpu().numpy().astype(np.float64) for k, x in zip(OUT, out)}
    assert np.abs(got["qpos_n"] - ref["qpos_n"]).max() < 1e-6
    assert np.abs(got["xpos"] - ref["xpos"]).max() < 1e-5
    assert np.abs(got["subtree_com"] - ref["subtree_com"]).max() < 1e-5
    assert np.abs(got["xquat"] - ref["xquat"]).max() < 1e-6
    cv = np.linalg.norm(got["cvel"] - ref["cvel"], axis=2) / np.maximum(np.linalg.norm(ref["cvel"], axis=2), 1e-3)
    assert np.quantile(cv, 0.99) < 1e-5, np.quantile(cv, 0.99)


def test_kinematics_vjp_matches_central_differences():
    torch = _cuda()
    import kinematics as K
    from nablaengine_b200 import torch_ffi
    q, v, c = _states(16)
    rng = np.random.default_rng(5)
    ref = K.kinematics(q, v, c)
    cot = {k: rng.standard_normal(x.shape) for k, x in ref.items()}
    cot["xquat"][:, 0] = 0.0  # the world body's frame is constant
    fq, fv = K.vjp_fd(q, v, c, cot)
    tq, tv, tc = (torch.from_numpy(np.ascontiguousarray(x)).cuda() for x in (q, v, c))
    tq.requires_grad_(True)
    tv.requires_grad_(True)
    out = torch_ffi.kinematics(tq, tv, tc)
    loss = sum((o * torch.from_numpy(cot[k].astype(np.float32)).cuda()).sum() for k, o in zip(OUT, out))
    loss.backward()
    gq, gv = tq.grad.cpu().numpy(), tv.grad.cpu().numpy()
    eq = np.linalg.norm(gq - fq, axis=1) / np.linalg.norm(fq, axis=1)
    ev = np.linalg.norm(gv - fv, axis=1) / np.linalg.norm(fv, axis=1)
    print(np.median(eq), eq.max(), np.median(ev), ev.max())
    assert np.quantile(eq, 0.99) < 1e-4 and np.quantile(ev, 0.99) < 1e-4, (eq, ev)


def test_step_kinematics_is_kinematics_of_the_output_and_differentiates():
    torch = _cuda()
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("forward", B=32)
    x = [torch.from_numpy(s[k]).cuda() for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    r = torch_ffi.step(*x, kinematics=True)
    k = torch_ffi.kinematics(r[0], r[1], x[5])
    for a, b in zip(r[3:], k):
        assert torch.equal(a, b)
    f = torch_ffi.forward(*x, kinematics=True)
    for a, b in zip(f[4:], k):
        assert torch.equal(a, b)
    # autograd through step(kinematics=True): the kinematics cotangents pulled back onto (qpos', qvel') and added
    q = x[0].clone().requires_grad_(True)
    out = torch_ffi.step(q, x[1], x[2], x[3], x[4], x[5], kinematics=True)
    (out[1].sum() + out[4].sum() + out[6].square().sum()).backward()
    q1, v1 = out[0].detach(), out[1].detach()
    tape = torch_ffi.forward(*x, tape=True)[4]
    z = lambda *sh: torch.zeros(sh, device="cuda")  # noqa: E731
    cot = (z(32, 36), torch.ones(32, 31, 3, device="cuda"), z(32, 31, 4), 2 * out[6].detach(), z(32, 31, 3))
    gq1, gv1 = torch_ffi.kinematics_backward(q1, v1, x[5], cot, z(32, 36), torch.ones(32, 35, device="cuda"))
    gq, _, _, _ = torch_ffi.backward(tape, x[4], x[5], gq1, gv1)
    err = (q.grad - gq).norm() / gq.norm()
    assert float(err) < 1e-5, float(err)
