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


def test_last_forward_record():
    """The last-forward record (nb_g1_last_forward): worlds, contacts summed, the most contacts and rows of a world,
    from the call's info; one record per batch size besides the latest (the reference's last_forward)."""
    torch = _cuda()
    from nablaengine_b200 import synthetic, torch_ffi
    xs = {}
    for B in (64, 32):
        s = synthetic.config_states("vjp", B=B)
        xs[B] = [torch.from_numpy(s[k]).cuda() for k in KEYS]
    info = {B: torch_ffi.forward(*xs[B])[3].cpu().numpy() for B in (64, 32)}
    want = {B: {"worlds": B, "contacts": int(i[:, 1].sum()), "max_contacts": int(i[:, 1].max()),
                "max_rows": int(i[:, 2].max())} for B, i in info.items()}
    assert torch_ffi.last_forward() == want[32]
    assert torch_ffi.last_forward(32) == want[32]
    assert torch_ffi.last_forward(64) == want[64]
    assert torch_ffi.last_forward(5) == dict.fromkeys(torch_ffi.LAST, 0)


def test_launch_info():
    """nb_g1_launch: the kernels' shared memory and resident worlds (rows) per SM on this device."""
    torch = _cuda()
    import ctypes
    from nablaengine_b200 import capi, torch_ffi
    d = torch_ffi.launch_info(0)
    props = torch.cuda.get_device_properties(0)
    assert d["sms"] == props.multi_processor_count
    assert d["forward_worlds_per_sm"] >= 10 and d["adjoint_worlds_per_sm"] >= 10 and d["jacobian_rows_per_sm"] >= 2 * 70
    for k in ("forward_smem_bytes", "adjoint_smem_bytes", "jacobian_smem_bytes"):
        assert 0 < d[k] <= 227 * 1024
    out = (ctypes.c_longlong * 8)()
    assert capi.load().nb_g1_launch(0, out) == 0
    assert list(out[:7]) == [d[k] for k in ("forward_smem_bytes", "forward_worlds_per_sm", "adjoint_smem_bytes",
                                            "adjoint_worlds_per_sm", "jacobian_smem_bytes", "jacobian_rows_per_sm",
                                            "sms")]
