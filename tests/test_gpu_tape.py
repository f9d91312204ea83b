"""The forward tape (what the adjoint reads), checked the way the reference checks its own (reference
scripts/engine_step_check.py:285-590, forward-tape checks T1-T8): every word of every record written (T8, the buffer
pre-filled with a sentinel), the state chain from record to record and to the outputs (T2), the factor of M + h kv
against the float64 oracle's mass matrix (T4) and the Newton Hessian's factor against the oracle's M + J'DJ at the
recorded solution's active rows (T5). T1 (tape on/off bitwise) is in test_gpu_adjoint.py.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# record layout in float32 words (nablaengine_b200/csrc/nb_g1_step.cuh, T_*): substep input qpos, qvel, the Newton
# solution a*, a_adv, L_H's inverse diagonal and packed lower triangle, the contact table, zones, clamp masks, header
# and flags (the compact record ends there), then L_Q's inverse diagonal and its pattern entries
T_QPOS, T_QVEL, T_ASTAR, T_AADV, T_DINVH, T_LH = 0, 36, 71, 106, 141, 176
NQ, NV, NU, NTRI = 36, 35, 29, 630
REC_COMPACT = 848
T_DINVQ = REC_COMPACT
T_LQ = T_DINVQ + NV
# L_Q is stored in tree-block order (legs, arms, waist, root: nb_g1_step.cuh tb_dof): position p holds dof TB_DOF[p],
# and only the entries of its pattern (p in q's chain or an ancestor chain of it), in packed-triangle order
TB_DOF = list(range(6, 18)) + list(range(21, 35)) + [18, 19, 20] + list(range(6))
_CHAIN = [0] * 6 + [1] * 6 + [2] * 7 + [3] * 7 + [4] * 3 + [5] * 6
TB_PATTERN = [(p, q) for p in range(35) for q in range(p + 1)
              if _CHAIN[p] == _CHAIN[q] or _CHAIN[p] == 5 or (_CHAIN[p] == 4 and _CHAIN[q] in (2, 3))]
NTB = len(TB_PATTERN)
H_STEP = np.float32(0.005)
KEYS = ("qpos", "qvel", "warm", "ctrl", "friction", "com")
SENTINEL = np.uint32(0xA5A5A5A5)


def _cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _forward_with_tape(s, nsub=4, iterations=10, compact=False):
    """Outputs and the (B, nsub, record words) tape of nb_g1_forward_ex called through the C ABI on a tape buffer
    pre-filled with the sentinel word (full or compact records)."""
    torch = _cuda()
    from nablaengine_b200 import capi, torch_ffi
    torch_ffi.init(0)
    lib = capi.load()
    rec = capi.tape_words(compact)
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in KEYS]
    B = t[0].shape[0]
    q1, v1, w1 = torch.empty((B, NQ), device="cuda"), torch.empty((B, NV), device="cuda"), torch.empty(
        (B, NV), device="cuda")
    info = torch.empty((B, 4), dtype=torch.int32, device="cuda")
    tape = torch.full((B, nsub * rec), int(SENTINEL.view(np.int32)), dtype=torch.int32, device="cuda")
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    rc = lib.nb_g1_forward_ex(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), B, *map(p, t), iterations,
                              nsub, p(q1), p(v1), p(w1), p(info), None, p(tape), None, rec)
    torch.cuda.synchronize()
    assert rc == 0, rc
    raw = tape.cpu().numpy().reshape(B, nsub, rec)
    return [x.cpu().numpy() for x in (q1, v1, w1, info)], raw, raw.view(np.float32)


@pytest.fixture(scope="module")
def taped():
    from nablaengine_b200 import synthetic
    s = synthetic.config_states("vjp", B=64)
    return (s,) + tuple(_forward_with_tape(s))


def _unpack(flat):
    """(B, NTRI) packed lower triangles -> (B, NV, NV) lower-triangular matrices."""
    i, j = np.tril_indices(NV)
    L = np.zeros(flat.shape[:-1] + (NV, NV))
    L[..., i, j] = flat
    return L


def test_every_word_of_every_record_is_written(taped):
    _, _, raw, _ = taped
    assert not np.any(raw.view(np.uint32) == SENTINEL), np.argwhere(raw.view(np.uint32) == SENTINEL)[:5]


def _fma32(a, b, c):
    """float32 a + b c rounded once (the device's fused multiply-add), through float64."""
    return (a.astype(np.float64) + np.float64(b) * c.astype(np.float64)).astype(np.float32)


def _within_ulp(x, y, n):
    return np.all(np.abs(x.astype(np.float64) - y) <= n * np.spacing(np.abs(y)).astype(np.float64))


def test_state_chain(taped):
    """qvel of record k + 1 = qvel_k + h a_adv_k (one fused multiply-add, within an ulp) and the hinge qpos advances
    by h qvel_{k+1}; the last record chains to the outputs."""
    _, (q1, v1, w1, info), _, tp = taped
    nsub = tp.shape[1]
    for k in range(nsub):
        v_next = tp[:, k + 1, T_QVEL:T_QVEL + NV] if k + 1 < nsub else v1
        q_next = tp[:, k + 1, T_QPOS:T_QPOS + NQ] if k + 1 < nsub else q1
        assert _within_ulp(v_next, _fma32(tp[:, k, T_QVEL:T_QVEL + NV], H_STEP, tp[:, k, T_AADV:T_AADV + NV]), 1), k
        assert _within_ulp(q_next[:, 7:], _fma32(tp[:, k, T_QPOS + 7:T_QPOS + NQ], H_STEP, v_next[:, 6:]), 1), k
    assert np.array_equal(w1, tp[:, -1, T_ASTAR:T_ASTAR + NV])  # warm' is the last substep's Newton solution


def _oracle_matrices(s, tp, k):
    import oracle
    return oracle.matrices(tp[:, k, T_QPOS:T_QPOS + NQ], tp[:, k, T_QVEL:T_QVEL + NV],
                           tp[:, k, T_ASTAR:T_ASTAR + NV], s["ctrl"], s["friction"], s["com"])


def test_factor_of_m_plus_h_kv_matches_the_oracle_mass_matrix(taped):
    """L_Q L_Q' = P (M + h kv) P' at each record's input state (P the tree-block order): relative Frobenius error
    of the float32 reconstruction against the float64 oracle's matrix, and dinv = 1 / diag(L_Q)."""
    s, _, _, tp = taped
    for k in range(tp.shape[1]):
        _, Q, _, _ = _oracle_matrices(s, tp, k)
        Q = Q[:, TB_DOF][:, :, TB_DOF]
        L = np.zeros((tp.shape[0], NV, NV))
        pi, qi = np.array(TB_PATTERN).T
        L[:, pi, qi] = tp[:, k, T_LQ:T_LQ + NTB].astype(np.float64)
        e = np.linalg.norm(L @ L.transpose(0, 2, 1) - Q, axis=(1, 2)) / np.linalg.norm(Q, axis=(1, 2))
        assert np.median(e) < 2e-6 and e.max() < 2e-5, (k, np.median(e), e.max())
        d = np.diagonal(L, axis1=1, axis2=2)
        np.testing.assert_allclose(tp[:, k, T_DINVQ:T_DINVQ + NV] * d, 1.0, rtol=1e-6)


def test_hessian_factor_matches_the_oracle_hessian(taped):
    """L_H L_H' = M + sum D J'J over the rows active at the recorded Newton solution (the final zones). A row within
    rounding of its zone boundary may sit on either side in float32 and float64, so the bound is on the median and
    on 90 % of the worlds."""
    s, _, _, tp = taped
    for k in range(tp.shape[1]):
        _, _, H, nrow = _oracle_matrices(s, tp, k)
        L = _unpack(tp[:, k, T_LH:T_LH + NTRI].astype(np.float64))
        e = np.linalg.norm(L @ L.transpose(0, 2, 1) - H, axis=(1, 2)) / np.linalg.norm(H, axis=(1, 2))
        assert np.median(e) < 1e-5 and np.quantile(e, 0.9) < 1e-4, (k, np.median(e), np.quantile(e, 0.9))
        assert nrow.max() > 0


# ---- the compact tape: records without L_Q, which the adjoint and the Jacobian rebuild from the replayed poses ------
def test_compact_records_are_the_full_records_first_words(taped):
    """Every word of a compact record is written, the outputs are bitwise those of the full tape, and the compact
    record is the full record's first REC_COMPACT words bit for bit."""
    from nablaengine_b200 import capi
    s, outs, raw, _ = taped
    assert capi.tape_words(True) == REC_COMPACT and capi.tape_words(False) == raw.shape[2]
    outs_c, raw_c, _ = _forward_with_tape(s, compact=True)
    assert raw_c.shape[2] == REC_COMPACT
    assert not np.any(raw_c.view(np.uint32) == SENTINEL)
    for a, b in zip(outs, outs_c):
        assert np.array_equal(a, b)
    assert np.array_equal(raw[:, :, :REC_COMPACT], raw_c)


def test_compact_tape_adjoint_and_jacobian_match_the_full_tape():
    """backward and jacobian on compact records (L_Q rebuilt from the replayed poses) equal those on full records
    within float32 rounding, in the exact and the default gradient modes; a record size other than the two is refused."""
    torch = _cuda()
    from nablaengine_b200 import capi, synthetic, torch_ffi
    s = synthetic.config_states("vjp", B=96, seed_offset=3)
    s["qpos"][:24, 2] -= 0.1
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in KEYS]
    full = torch_ffi.forward(*t, tape=True)
    comp = torch_ffi.forward(*t, tape="compact")
    assert comp[4].shape[1] == 4 * REC_COMPACT and full[4].shape[1] == 4 * capi.tape_words(False)
    for a, b in zip(full[:4], comp[:4]):
        assert torch.equal(a, b)
    g = torch.Generator(device="cuda").manual_seed(5)
    cq = torch.randn(96, NQ, device="cuda", generator=g)
    cv = torch.randn(96, NV, device="cuda", generator=g)

    def rel(a, b):
        return float(((a.double() - b.double()).norm(dim=-1) / b.double().norm(dim=-1).clamp_min(1e-9)).max())

    for kv, nm in ((1, 0), (0, 3)):
        rf = torch_ffi.backward(full[4], t[4], t[5], cq, cv, clamp_kv=kv, normal=nm)
        rc = torch_ffi.backward(comp[4], t[4], t[5], cq, cv, clamp_kv=kv, normal=nm)
        errs = [rel(a, b) for a, b in zip(rc[:3], rf[:3])]
        print("backward", kv, nm, errs)
        assert max(errs) < 1e-3 and torch.equal(rc[3], rf[3]), errs
    Jf = torch_ffi.jacobian(full[4], t[4], t[5])[0]
    Jc = torch_ffi.jacobian(comp[4], t[4], t[5])[0]
    err = (Jc.double() - Jf.double()).norm(dim=2) / Jf.double().norm(dim=2).clamp_min(1e-9)
    print("jacobian rows: median", float(err.median()), "max", float(err.max()))
    assert float(err.median()) < 1e-5 and float(err.max()) < 1e-2
    lib = capi.load()
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    bad = lib.nb_g1_jacobian_ex(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), 96, 4, p(full[4]), p(t[4]),
                                p(t[5]), p(Jf), p(rc[3]), None, ctypes.c_float(0.0), 1, 0, 1000)
    assert bad != 0
