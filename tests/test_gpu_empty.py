"""A batch of zero worlds through every differentiable entry: the forward with either tape, the backward, the Jacobian,
autograd through step, and the C entries themselves (nw = 0 with null buffers launches nothing and returns 0). A
training loop whose shard of worlds comes out empty on some rank reaches these calls with B = 0.
"""
import pytest

pytestmark = pytest.mark.gpu


def _zeros(*shape):
    import torch
    return torch.zeros(shape, dtype=torch.float32, device="cuda")


def test_zero_worlds_through_tapes_backward_and_jacobian():
    import torch
    from nablaengine_b200 import torch_ffi
    x = (_zeros(0, 36), _zeros(0, 35), _zeros(0, 35), _zeros(0, 29), _zeros(0), _zeros(0, 3))
    for mode, words in ((True, 1224), ("compact", 848)):
        out = torch_ffi.forward(*x, tape=mode)
        tape = out[4]
        assert tape.shape == (0, 4 * words)
        gq, gv, gu, info = torch_ffi.backward(tape, x[4], x[5], _zeros(0, 36), _zeros(0, 35))
        assert gq.shape == (0, 36) and gv.shape == (0, 35) and gu.shape == (0, 29) and info.shape == (0,)
        J, jinfo = torch_ffi.jacobian(tape, x[4], x[5])
        assert J.shape == (0, 71, 99) and jinfo.shape == (0,)
    torch.cuda.synchronize()


def test_zero_worlds_through_autograd_step():
    import torch
    from nablaengine_b200 import torch_ffi
    qpos, qvel, ctrl = (_zeros(0, 36).requires_grad_(), _zeros(0, 35).requires_grad_(),
                        _zeros(0, 29).requires_grad_())
    q1, v1, w1 = torch_ffi.step(qpos, qvel, _zeros(0, 35), ctrl, _zeros(0), _zeros(0, 3))
    assert q1.shape == (0, 36) and v1.shape == (0, 35) and w1.shape == (0, 35)
    (q1.sum() + (v1 * v1).sum()).backward()
    assert qpos.grad.shape == (0, 36) and qvel.grad.shape == (0, 35) and ctrl.grad.shape == (0, 29)


def test_zero_worlds_through_the_c_entries():
    import torch
    from nablaengine_b200 import capi
    lib = capi.load()
    torch.cuda.init()
    assert lib.nb_g1_upload(None, None) == 0
    assert lib.nb_g1_forward(None, 0, *([None] * 6), 10, 4, *([None] * 7)) == 0
    assert lib.nb_g1_adjoint(None, 0, 4, *([None] * 10), 0.0, 1, 0) == 0
    assert lib.nb_g1_jacobian(None, 0, 4, *([None] * 6), 0.0, 1, 0) == 0
    # a negative count is refused, not launched
    assert lib.nb_g1_jacobian(None, -1, 4, *([None] * 6), 0.0, 1, 0) != 0
    torch.cuda.synchronize()
