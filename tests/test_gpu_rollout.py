"""The BPTT rollout (nablaengine_b200/rollout.py) through the CUDA step: its autograd ctrl gradient equals a manual
chain of per-step adjoints (forward with tape, then torch_ffi.backward in reverse), as the reference's rollout
window check (scripts/jax_ffi_check.py: a 64-step scan window against a manual VJP chain)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bptt_equals_manual_adjoint_chain():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nablaengine_b200 import rollout, torch_ffi
    B, T = 64, 4
    inp = rollout.rollout_inputs(B, T, 0, "cuda")
    loss, g = rollout.bptt(inp)
    assert torch.isfinite(loss) and torch.isfinite(g).all()
    # manual: forward with tapes, then the adjoint chain
    q, v, w = inp["qpos"], inp["qvel"], inp["warm"]
    tapes, vs = [], []
    for t in range(T):
        q, v, w, _, tp = torch_ffi.forward(q, v, w, inp["ctrl_seq"][t].contiguous(), inp["friction"], inp["com"],
                                           tape=True)
        tapes.append(tp)
        vs.append(v)
    norm = 1.0 / (T * B)
    gq, gv = torch.zeros_like(q), torch.zeros_like(v)
    gu = [None] * T
    man_loss = sum(float((x * x).sum()) for x in vs) * norm
    for t in reversed(range(T)):
        gv = gv + 2.0 * norm * vs[t]
        gq, gv, gu[t], _ = torch_ffi.backward(tapes[t], inp["friction"], inp["com"], gq.contiguous(), gv.contiguous())
    gm = torch.stack(gu)
    assert float(loss) == pytest.approx(man_loss, rel=1e-5)
    err = (g - gm).norm() / gm.norm()
    assert float(err) < 1e-5, float(err)


def test_reduce_stats_single_process():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nablaengine_b200 import rollout
    g = torch.tensor([[[1.0, 2.0], [float("nan"), 0.0]]], device="cuda")
    vec = rollout.reduce_stats(torch.tensor(3.0, device="cuda"), g).cpu().numpy()
    assert np.allclose(vec, [3.0, 5.0, 2.0, 1.0])
