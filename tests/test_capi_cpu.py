"""The C-ABI library and the host-side API without a GPU: it loads, exports every declared symbol, reports its
compiled sizes, and the torch API rejects bad arguments before any launch."""
import ctypes

import numpy as np
import pytest

from nablaengine_b200 import capi, synthetic, torch_ffi


def test_library_exports_every_declared_symbol():
    lib = capi.load()
    declared = capi.declared_symbols()
    assert {"nb_g1_forward", "nb_g1_work_bytes", "nb_g1_upload", "nb_g1_sizes"} <= set(declared)
    for name in declared:
        assert hasattr(lib, name), name


def test_sizes_and_work_bytes():
    assert capi.sizes()[:6] == [36, 35, 29, 31, 64, 192]
    lib = capi.load()
    # the world order: one int32 per world, rounded up to 16 bytes
    assert lib.nb_g1_work_bytes(4096) == 16384
    assert lib.nb_g1_work_bytes(37) == 160
    assert lib.nb_g1_work_bytes(0) == 0
    assert lib.nb_g1_work_bytes(-1) < 0


def test_forward_rejects_bad_arguments_without_launching():
    lib = capi.load()
    nul = ctypes.c_void_p(0)
    # substeps out of range, negative iterations, negative worlds: cudaErrorInvalidValue (1) before any launch
    assert lib.nb_g1_forward(nul, 1, *[nul] * 6, 10, 0, *[nul] * 7) == 1
    assert lib.nb_g1_forward(nul, 1, *[nul] * 6, 10, 33, *[nul] * 7) == 1
    assert lib.nb_g1_forward(nul, 1, *[nul] * 6, -1, 4, *[nul] * 7) == 1
    assert lib.nb_g1_forward(nul, -1, *[nul] * 6, 10, 4, *[nul] * 7) == 1
    assert lib.nb_g1_forward(nul, 0, *[nul] * 6, 10, 4, *[nul] * 7) == 0  # no worlds: a no-op


def test_tape_record_sizes_and_the_ex_entries_reject_other_sizes():
    """The full and the compact record sizes; the _ex entries refuse any other record size (cudaErrorInvalidValue)
    before any launch, and the plain entries are the _ex ones with full records."""
    lib = capi.load()
    full, compact = capi.tape_words(False), capi.tape_words(True)
    assert (full, compact) == (capi.sizes()[6], 848) and capi.sizes()[7] == 4
    assert torch_ffi.tape_bytes(4096, compact=True) * full == torch_ffi.tape_bytes(4096) * compact
    nul, f0 = ctypes.c_void_p(0), ctypes.c_float(0.0)
    for words in (0, -1, full - 4, compact + 4, 2 * full):
        assert lib.nb_g1_forward_ex(nul, 1, *[nul] * 6, 10, 4, *[nul] * 7, words) == 1
        assert lib.nb_g1_adjoint_ex(nul, 1, 4, *[nul] * 10, f0, 1, 0, words) == 1
        assert lib.nb_g1_jacobian_ex(nul, 1, 4, *[nul] * 6, f0, 1, 0, words) == 1
        assert lib.nb_g1_diag_forward_ex(nul, nul, 1, 4, 10, nul, nul, words) == 1
    for words in (full, compact):  # no worlds: a no-op
        assert lib.nb_g1_forward_ex(nul, 0, *[nul] * 6, 10, 4, *[nul] * 7, words) == 0
        assert lib.nb_g1_adjoint_ex(nul, 0, 4, *[nul] * 10, f0, 1, 0, words) == 0
        assert lib.nb_g1_jacobian_ex(nul, 0, 4, *[nul] * 6, f0, 1, 0, words) == 0


def test_small_entries_reject_bad_arguments_without_launching():
    lib = capi.load()
    nul = ctypes.c_void_p(0)
    assert lib.nb_g1_last_forward(nul, -1, nul, nul, nul) == 1  # cudaErrorInvalidValue
    assert lib.nb_g1_last_forward(nul, 4, nul, nul, nul) == 1   # no info / record
    out = (ctypes.c_longlong * 8)(*range(1, 9))
    rc = lib.nb_g1_launch(0, out)
    if rc:  # no usable device here: an error code and a zeroed record
        assert list(out) == [0] * 8


def test_torch_api_type_errors_on_cpu_tensors():
    import torch
    s = {k: torch.from_numpy(v) for k, v in synthetic.states(2, 0).items()}
    with pytest.raises(TypeError):
        torch_ffi.forward(s["qpos"], s["qvel"], s["warm"], s["ctrl"], s["friction"], s["com"])
    with pytest.raises(ValueError):
        torch_ffi.step(s["qpos"], s["qvel"], s["warm"], s["ctrl"], s["friction"], s["com"], clamp_kv=5)


def test_synthetic_distribution():
    s = synthetic.states(2048, 1)
    m = synthetic.model()
    assert s["qpos"].dtype == np.float32 and s["qpos"].shape == (2048, 36)
    assert np.allclose(np.linalg.norm(s["qpos"][:, 3:7], axis=1), 1, atol=1e-6)
    assert (s["qpos"][:, 7:] >= m["dof_range"][6:, 0] - 1e-6).all()
    assert (s["qpos"][:, 7:] <= m["dof_range"][6:, 1] + 1e-6).all()
    assert 0.70 <= s["qpos"][:, 2].min() and s["qpos"][:, 2].max() <= 0.80
    assert abs(s["qvel"].std() - 0.5) < 0.01
    assert 0.4 <= s["friction"].min() and s["friction"].max() <= 1.2
    low = synthetic.states(4096, 2, lowered=0.1)
    assert 0.05 < (low["qpos"][:, 2] < 0.70).mean() < 0.15
