"""Parity of the CUDA forward step (libnabla_g1.so, through the torch API and the C ABI) with the CPU oracle and the
reference's golden data. Needs a GPU."""
import numpy as np
import pytest

import oracle
from nablaengine_b200 import synthetic

pytestmark = pytest.mark.gpu
INPUTS = ("qpos", "qvel", "qacc_warmstart", "ctrl", "friction", "com")
# float32 step against the float64 oracle (same algorithm, 10 iterations): per-world relative error of qvel', the
# median bound of the forward parity target; every world above MAX_TOL must be one whose Newton solve hit its
# iteration cap in some substep (unconverged: the float32 and float64 iterates stop at different points)
MEDIAN_TOL, P99_TOL, MAX_TOL = 1e-6, 1e-4, 1e-4
# a contact found by one run and not the other must be this close to touching (|dist| in m): the two runs' bodies
# differ by float32 rounding of the trajectory, so a contact at the edge of touching may fall on either side
CONTACT_EPS = 1e-4


def rel_world(a, b):
    return np.linalg.norm(a - b, axis=1) / np.maximum(np.linalg.norm(b, axis=1), 1e-9)


def gpu_forward(args, iterations=10, substeps=4):
    import torch
    from nablaengine_b200 import torch_ffi
    t = [torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda() for a in args]
    out = torch_ffi.forward(*t, iterations=iterations, substeps=substeps)
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in out]


def check_parity(args, iterations=10, substeps=4, med=MEDIAN_TOL, p99=P99_TOL, mx=MAX_TOL):
    q1, v1, w1, info = gpu_forward(args, iterations, substeps)
    oq, ov, ow, oinfo, ost = oracle.step(*args, iterations=iterations, substeps=substeps, stats=True)
    ev = rel_world(v1, ov)
    assert np.isfinite(v1).all() and np.isfinite(q1).all()
    assert np.median(ev) <= med, np.median(ev)
    assert np.percentile(ev, 99) <= p99, np.percentile(ev, 99)
    if mx is not None:  # the worlds above the max bound: each at the iteration cap in some substep
        capped = (ost[:, :, 2] >= iterations).any(1)
        above = ev > mx
        print(f"qvel' relative error: median {np.median(ev):.2e}, max {ev.max():.2e}; {int(above.sum())} of "
              f"{len(ev)} worlds above {mx:g}, all iteration-capped: {bool((capped | ~above).all())}")
        assert (capped | ~above).all(), (np.flatnonzero(above & ~capped), ev[above & ~capped])
    return q1, v1, w1, info, oinfo, ev


def gpu_forward_contacts(args, iterations=10, substeps=4):
    """(info, contacts): the C ABI's forward with its contact output, the last substep's contacts (B, 64, 8) =
    (pair, dist, pos[3], normal[3]), pair -1 past the count."""
    import ctypes
    import torch
    from nablaengine_b200 import capi, torch_ffi
    torch_ffi.init(0)
    lib = capi.load()
    t = [torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda() for a in args]
    B = t[0].shape[0]
    out = [torch.empty((B, 36), device="cuda"), torch.empty((B, 35), device="cuda"),
           torch.empty((B, 35), device="cuda"), torch.empty((B, 4), dtype=torch.int32, device="cuda"),
           torch.empty((B, 64, 8), device="cuda")]
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    work = torch.empty((lib.nb_g1_work_bytes(B),), dtype=torch.uint8, device="cuda")
    rc = lib.nb_g1_forward(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), B, *map(p, t), iterations,
                           substeps, *map(p, out), None, p(work))
    torch.cuda.synchronize()
    assert rc == 0, rc
    return out[3].cpu().numpy(), out[4].cpu().numpy()


def unexplained_contact_differences(con_gpu, con_oracle, eps=CONTACT_EPS):
    """Per world, compare the two runs' last-substep contacts pair by pair: where a pair has more contacts in one
    run, that run's surplus must be at |dist| < eps (contacts of a pair come in slot order in both; the surplus is
    taken as the ones closest to touching). Returns (worlds whose contact sets differ, worlds where the difference
    is not explained that way)."""
    differ, unexplained = [], []
    for w in range(con_gpu.shape[0]):
        g = {}
        for pair, dist in con_gpu[w][:, :2]:
            if pair >= 0:
                g.setdefault(int(pair), []).append(float(dist))
        o = {}
        for pair, _slot, dist in con_oracle[w]:
            if pair >= 0:
                o.setdefault(int(pair), []).append(float(dist))
        explained = same = True
        for pair in set(g) | set(o):
            a, b = g.get(pair, []), o.get(pair, [])
            if len(a) == len(b):
                continue
            same = False
            more = a if len(a) > len(b) else b
            surplus = sorted(abs(x) for x in more)[:abs(len(a) - len(b))]
            explained = explained and max(surplus) < eps
        if not same:
            differ.append(w)
            if not explained:
                unexplained.append(w)
    return differ, unexplained


def check_contact_counts(args, iterations=10, substeps=4, label=""):
    """The raw contact counts, row counts and overflow bits of the last substep against the float64 oracle: every
    world whose contact count differs is reported, and each must differ only by contacts at |dist| < CONTACT_EPS; a
    world whose row count differs must be one of them (its rows are the contacts' 4 or 1 plus the limit rows, and
    the limits match) and the overflow bits are equal everywhere."""
    info, con = gpu_forward_contacts(args, iterations, substeps)
    _, _, _, oinfo, ocon = oracle.step(*args, iterations=iterations, substeps=substeps, contacts=True)
    ncon_diff = np.flatnonzero(info[:, 1] != oinfo[:, 1])
    nrow_diff = np.flatnonzero(info[:, 2] != oinfo[:, 2])
    differ, unexplained = unexplained_contact_differences(con, ocon)
    print(f"{label}: {len(info)} worlds; contact count differs on {len(ncon_diff)}, row count on {len(nrow_diff)}, "
          f"contact sets on {len(differ)} (all by contacts within {CONTACT_EPS:g} m of touching: "
          f"{not unexplained})")
    assert not unexplained, unexplained
    assert set(ncon_diff.tolist()) <= set(differ) and set(nrow_diff.tolist()) <= set(differ)
    assert (info[:, 3] == oinfo[:, 3]).all()
    return len(ncon_diff), len(nrow_diff)


def test_contact_counts_at_the_input_state(golden):
    """One substep from the golden states: both runs collide the same input state, so their contacts may differ
    only where a distance rounds to the other side of zero."""
    g = golden("truth_check.npz")
    check_contact_counts([g[k] for k in INPUTS], substeps=1, label="golden check states, 1 substep")


def test_contact_counts_after_a_step(golden):
    g = golden("truth_check.npz")
    check_contact_counts([g[k] for k in INPUTS], label="golden check states")
    s = synthetic.config_states("vjp", B=1024)
    check_contact_counts([s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")],
                         label="configuration 3, 1024 worlds")


def test_parity_golden_check_states(golden):
    g = golden("truth_check.npz")
    args = [g[k] for k in INPUTS]
    q1, v1, _, info, oinfo, _ = check_parity(args)
    assert (info[:, 3] == oinfo[:, 3]).all()
    # against MuJoCo's converged float64 truth on the model-ok states (the reference: median 8.5e-7)
    ok = g["model_flags"] == 0
    et = rel_world(v1, g["check_out"][:, 36:])
    assert np.median(et[ok]) <= 5e-6


def test_parity_synthetic_forward_config():
    s = synthetic.config_states("forward", B=1024)
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    check_parity(args)


def test_parity_lowered_multicontact():
    s = synthetic.config_states("vjp", B=512)
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    check_parity(args)


def test_mujoco_warp_gate(golden):
    """The reference's own gate against MuJoCo Warp (50 iterations): qvel median / p99 <= 5e-6 / 5e-5."""
    g = golden("mjw_sample.npz")
    _, v1, _, info = gpu_forward([g[k] for k in INPUTS], iterations=50)
    ok = g["model_flags"] == 0
    ev = rel_world(v1, g["out_qvel"])
    assert np.median(ev[ok]) <= 5e-6 and np.percentile(ev[ok], 99) <= 5e-5
    assert (info[:, 1] == g["ncon"][:, 3]).mean() >= 0.98


def test_deterministic_bitwise():
    s = synthetic.config_states("vjp", B=2048)
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    a = gpu_forward(args)
    b = gpu_forward(args)
    for x, y in zip(a, b):
        assert np.array_equal(x.view(np.uint32) if x.dtype == np.float32 else x,
                              y.view(np.uint32) if y.dtype == np.float32 else y)


def test_substeps_and_iterations_options():
    """Other iteration caps and substep counts. One to three Newton steps leave the solve unconverged, where float32
    rounding alone moves the result by ~1e-4 (the oracle's own float32 build differs from its float64 build by as
    much), so those caps get a tolerance of that size; 0 iterations (the warm-start choice) and converged caps keep
    the tight one."""
    s = synthetic.config_states("forward", B=64)
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    for it, ns, med, p99 in ((0, 1, 1e-6, 1e-4), (1, 2, 1e-3, 1e-2), (3, 1, 2e-4, 2e-3), (10, 8, 1e-6, 1e-4)):
        check_parity(args, iterations=it, substeps=ns, med=med, p99=p99, mx=MAX_TOL if it in (0, 10) else None)


def test_overflow_bits_and_raw_count():
    s = synthetic.states(8, 7)
    s["qpos"][:, 2] = 0.05
    s["qpos"][:, 7:] = 0.0
    args = [s[k] for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    _, _, _, info = gpu_forward(args, substeps=1)
    _, _, _, oinfo = oracle.step(*args, substeps=1)
    assert (info[:, 1] == oinfo[:, 1]).all()
    assert ((info[:, 3] & 4) != 0).tolist() == (info[:, 1] > 64).tolist()
    assert (info[:, 2] <= 192).all()


def test_zero_worlds_and_type_errors():
    import torch
    from nablaengine_b200 import torch_ffi
    e = lambda *s: torch.zeros(s, dtype=torch.float32, device="cuda")  # noqa: E731
    out = torch_ffi.forward(e(0, 36), e(0, 35), e(0, 35), e(0, 29), e(0), e(0, 3))
    assert out[0].shape == (0, 36) and out[3].shape == (0, 4)
    with pytest.raises(TypeError):
        torch_ffi.forward(e(2, 36).double(), e(2, 35), e(2, 35), e(2, 29), e(2), e(2, 3))
    with pytest.raises(TypeError):
        torch_ffi.forward(e(2, 36), e(2, 34), e(2, 35), e(2, 29), e(2), e(2, 3))
    with pytest.raises(TypeError):
        torch_ffi.forward(e(2, 36)[:, :36].t().contiguous().t(), e(2, 35), e(2, 35), e(2, 29), e(2), e(2, 3))


def test_cuda_graph_capture_replay():
    import torch
    from nablaengine_b200 import torch_ffi
    s = synthetic.config_states("forward", B=256)
    t = {k: torch.from_numpy(v).cuda() for k, v in s.items()}
    torch_ffi.init(0)
    ref = torch_ffi.forward(t["qpos"], t["qvel"], t["warm"], t["ctrl"], t["friction"], t["com"])
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        torch_ffi.forward(t["qpos"], t["qvel"], t["warm"], t["ctrl"], t["friction"], t["com"])
    torch.cuda.current_stream().wait_stream(side)
    with torch.cuda.graph(g):
        out = torch_ffi.forward(t["qpos"], t["qvel"], t["warm"], t["ctrl"], t["friction"], t["com"])
    g.replay()
    torch.cuda.synchronize()
    for a, b in zip(ref, out):
        assert torch.equal(a, b)


def test_world_order_changes_no_output_bit():
    """The work memory's world order (worlds sorted by root height, lowest first, each chunk of 4096 worlds on its
    own) only schedules: outputs, info and tape equal those of the index-order launch (work NULL) bit for bit, on a
    ragged batch of two chunks; the order itself is a permutation, the root heights non-decreasing within a chunk,
    ties in index order."""
    import ctypes
    import torch
    from nablaengine_b200 import capi, torch_ffi
    torch_ffi.init(0)
    lib = capi.load()
    s = synthetic.config_states("vjp", B=5000)
    B, nsub, rec = 5000, 4, int(capi.sizes()[6])
    s["qpos"][7:19, 2] = s["qpos"][3, 2]  # equal keys: the index decides
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda()
         for k in ("qpos", "qvel", "warm", "ctrl", "friction", "com")]
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nwork = lib.nb_g1_work_bytes(B)
    assert nwork == 16 * ((4 * B + 15) // 16)
    runs = []
    for work in (torch.full((nwork,), 0xAB, dtype=torch.uint8, device="cuda"), None):
        out = [torch.empty((B, 36), device="cuda"), torch.empty((B, 35), device="cuda"),
               torch.empty((B, 35), device="cuda"), torch.empty((B, 4), dtype=torch.int32, device="cuda")]
        tape = torch.empty((B, nsub * rec), device="cuda")
        rc = lib.nb_g1_forward(st, B, *map(p, t), 10, nsub, *map(p, out), None, p(tape),
                               None if work is None else p(work))
        torch.cuda.synchronize()
        assert rc == 0, rc
        runs.append([x.cpu().numpy().view(np.uint32) for x in out + [tape]] + [work])
    for a, b in zip(runs[0][:5], runs[1][:5]):
        assert np.array_equal(a, b)
    order = runs[0][5].cpu().numpy()[:4 * B].view(np.int32)
    assert np.array_equal(np.sort(order), np.arange(B))
    z = s["qpos"][:, 2].astype(np.float32)
    for c0 in range(0, B, 4096):
        o = order[c0:c0 + 4096]
        idx = np.arange(c0, min(B, c0 + 4096))
        assert np.array_equal(o, idx[np.lexsort((idx, z[idx]))])
