"""Diagnostics counters (nb_g1_diag_forward / _backward, torch_ffi.read_diagnostics): exact counts of the calls'
info bits, tape flags and non-finite rows, as the reference's counter kernels (src/nablaengine/torch_ffi.py:101-157)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
KEYS = ("qpos", "qvel", "warm", "ctrl", "friction", "com")


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def test_forward_and_backward_counters():
    torch = _cuda()
    from nablaengine_b200 import synthetic, torch_ffi
    s = synthetic.config_states("forward", B=64)
    s["qpos"][:8, 2] = 0.05  # sunk into the floor: more rows than the capacity
    x = [torch.from_numpy(s[k]).cuda() for k in KEYS]
    torch_ffi.read_diagnostics(reset=True)
    q1, v1, w1, info, tape = torch_ffi.forward(*x, tape=True)
    d = torch_ffi.read_diagnostics(reset=True)
    bits = info[:, 3].cpu().numpy()
    assert d["fwd_calls"] == 1 and d["fwd_worlds"] == 64 and d["tape_records"] == 64 * 4
    assert d["fwd_contact_overflow_worlds"] == int(((bits & 4) != 0).sum())
    assert d["fwd_row_overflow_worlds"] == int(((bits & 16) != 0).sum())
    assert d["fwd_contact_overflow_worlds"] + d["fwd_row_overflow_worlds"] > 0  # the sunk worlds overflow
    assert d["fwd_unsupported_worlds"] == int((bits != 0).sum())
    assert d["fwd_iteration_limit_worlds"] == int((info[:, 0].cpu().numpy() >= 10).sum())
    assert 0 <= d["refact_records"] <= 256 and 0 <= d["nonconv_records"] <= 256 and d["singular_records"] == 0
    # backward with one non-finite cotangent row
    gq, gv = torch.zeros_like(q1), 2 * v1
    gv[3, 0] = float("nan")
    r = torch_ffi.backward(tape, x[4], x[5], gq, gv)
    d = torch_ffi.read_diagnostics(reset=True)
    assert d["bwd_calls"] == 1 and d["bwd_rows"] == 64
    assert d["nonfinite_cotangent_rows"] == 1
    assert (r[3][3].item() >> 16) & 8
    # switched off: no counting
    prev = torch_ffi.set_diagnostics(False)
    torch_ffi.forward(*x)
    assert torch_ffi.read_diagnostics(reset=True)["fwd_calls"] == 0
    torch_ffi.set_diagnostics(prev)


def test_overflow_warning():
    _cuda()
    from nablaengine_b200 import torch_ffi
    with pytest.warns(RuntimeWarning, match="contact capacity"):
        assert torch_ffi.warn_overflow({"fwd_contact_overflow_worlds": 2, "fwd_row_overflow_worlds": 0}) == 2
