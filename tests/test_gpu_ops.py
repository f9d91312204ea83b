"""The torch.library custom ops (nabla_b200::forward / backward / kinematics / kinematics_backward, the reference's
torch_ffi.py:595-657): fake implementations for tracing, torch.compile(fullgraph=True) equal to eager, and the
backward's kinematics cotangents (reference torch_ffi.py:854)."""
import pytest

pytestmark = pytest.mark.gpu
KEYS = ("qpos", "qvel", "warm", "ctrl", "friction", "com")


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _x(B=16):
    torch = _cuda()
    from nablaengine_b200 import synthetic
    s = synthetic.config_states("forward", B=B)
    return [torch.from_numpy(s[k]).cuda() for k in KEYS]


def test_compiled_fullgraph_equals_eager():
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    x = _x()
    torch_ffi.init()

    def f(*a):
        q1, v1, w1 = torch_ffi.step(*a)
        return q1, v1 * 2.0, w1

    eager = f(*x)
    comp = torch.compile(f, fullgraph=True)(*x)
    for a, b in zip(eager, comp):
        assert torch.equal(a, b)


def test_fake_shapes():
    torch = _cuda()
    from torch._subclasses.fake_tensor import FakeTensorMode
    from nablaengine_b200 import torch_ffi
    ops = torch_ffi.custom_ops()
    x = _x(4)
    with FakeTensorMode(allow_non_fake_inputs=True) as mode:
        fx = [mode.from_tensor(t) for t in x]
        r = ops["forward"](*fx, 10, 4, True)
        assert [tuple(t.shape) for t in r[:4]] == [(4, 36), (4, 35), (4, 35), (4, 4)]
        assert r[4].shape[0] == 4
        k = ops["kinematics"](fx[0], fx[1], fx[5])
        assert [tuple(t.shape) for t in k] == [(4, 36), (4, 31, 3), (4, 31, 4), (4, 31, 6), (4, 31, 3)]


def test_backward_with_kinematics_cotangents():
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    x = _x()
    q1, v1, w1, info, tape = torch_ffi.forward(*x, tape=True)
    B = q1.shape[0]
    gq, gv = torch.zeros(B, 36, device="cuda"), torch.ones(B, 35, device="cuda")
    kc = (torch.zeros(B, 36, device="cuda"), torch.ones(B, 31, 3, device="cuda"), torch.zeros(B, 31, 4, device="cuda"),
          torch.zeros(B, 31, 6, device="cuda"), torch.zeros(B, 31, 3, device="cuda"))
    a = torch_ffi.backward(tape, x[4], x[5], gq, gv, kinematics=(q1, v1) + kc)
    cq, cv = torch_ffi.kinematics_backward(q1, v1, x[5], kc, gq, gv)
    b = torch_ffi.backward(tape, x[4], x[5], cq, cv)
    for u, w in zip(a[:3], b[:3]):
        assert torch.equal(u, w)


def test_cuda_graph_of_forward_backward_jacobian_kinematics():
    """A whole differentiated step (forward with tape, adjoint, Jacobian, kinematics and its VJP, the diagnostics
    kernels) captured in one CUDA graph and replayed equals the eager calls bitwise."""
    torch = _cuda()
    from nablaengine_b200 import torch_ffi
    x = _x(64)
    torch_ffi.init()
    z = lambda *sh: torch.zeros(sh, device="cuda")  # noqa: E731

    def run():
        q1, v1, w1, info, tape = torch_ffi.forward(*x, tape=True)
        g = torch_ffi.backward(tape, x[4], x[5], z(64, 36), 2 * v1)
        J, _ = torch_ffi.jacobian(tape, x[4], x[5])
        k = torch_ffi.kinematics(q1, v1, x[5])
        kg = torch_ffi.kinematics_backward(q1, v1, x[5], (z(64, 36), k[1], z(64, 31, 4), z(64, 31, 6),
                                                          z(64, 31, 3)))
        return (q1, v1, w1, info) + tuple(g) + (J,) + tuple(k) + tuple(kg)

    ref = run()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        run()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = run()
    graph.replay()
    torch.cuda.synchronize()
    for a, b in zip(ref, out):
        assert torch.equal(a, b)
