"""nb_g1_forward_noalloc, the forward for callers that cannot allocate device memory (code running where cudaMalloc
is not allowed or not wanted: host callbacks, fixed memory budgets, runtimes whose allocator the caller does not own):
it keeps the world order in the library's own buffer instead of caller work memory. Checked through the C ABI against
nb_g1_forward with work memory, on two calls in a row of different batches (the buffer keeps the first call's order
when the second begins), and its size limit. Needs a GPU. Collected last, so that a run stopping at its first failure
has run every other test before this one; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
KEYS = ("qpos", "qvel", "warm", "ctrl", "friction", "com")
NOALLOC_MAX_WORLDS = 262144  # include/nabla_g1.h NB_G1_NOALLOC_MAX_WORLDS


def _setup():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nablaengine_b200 import capi, torch_ffi
    torch_ffi.init(0)  # nb_g1_upload on device 0 (the kernels' shared-memory opt-in)
    return torch, capi.load(), int(capi.sizes()[6])


def _run(torch, lib, rec, s, noalloc, nsub=4):
    """Outputs (qpos', qvel', warm', info, tape) of one call, as raw 32-bit words."""
    B = s["qpos"].shape[0]
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in KEYS]
    out = [torch.empty((B, 36), device="cuda"), torch.empty((B, 35), device="cuda"),
           torch.empty((B, 35), device="cuda"), torch.empty((B, 4), dtype=torch.int32, device="cuda"),
           torch.empty((B, nsub * rec), device="cuda")]
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = lib.nb_g1_forward_noalloc(st, B, *map(p, t), 10, nsub, *map(p, out[:4]), None, p(out[4]))
    else:
        work = torch.empty((lib.nb_g1_work_bytes(B),), dtype=torch.uint8, device="cuda")
        rc = lib.nb_g1_forward(st, B, *map(p, t), 10, nsub, *map(p, out[:4]), None, p(out[4]), p(work))
    torch.cuda.synchronize()
    assert rc == 0, rc
    return [x.cpu().numpy().view(np.uint32) for x in out]


def test_forward_noalloc_equals_forward_on_two_calls_in_a_row():
    torch, lib, rec = _setup()
    from nablaengine_b200 import synthetic
    batches = [synthetic.config_states("vjp", B=5000), synthetic.config_states("forward", B=777, seed_offset=3)]
    first = [_run(torch, lib, rec, s, noalloc=True) for s in batches]  # back to back, the buffer shared
    for s, got in zip(batches, first):
        want = _run(torch, lib, rec, s, noalloc=False)
        for name, a, b in zip(("qpos'", "qvel'", "warm'", "info", "tape"), got, want):
            assert np.array_equal(a, b), name  # bitwise: the same kernels on the same order


def test_forward_noalloc_allocates_no_device_memory():
    """A call with every buffer already in place leaves the device's free memory and torch's reserved memory as they
    were (after a first call, which may load the kernels' code)."""
    torch, lib, rec = _setup()
    from nablaengine_b200 import synthetic
    s = synthetic.config_states("forward", B=2048)
    B = 2048
    t = [torch.from_numpy(np.ascontiguousarray(s[k], np.float32)).cuda() for k in KEYS]
    out = [torch.empty((B, 36), device="cuda"), torch.empty((B, 35), device="cuda"),
           torch.empty((B, 35), device="cuda"), torch.empty((B, 4), dtype=torch.int32, device="cuda")]
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    call = lambda: lib.nb_g1_forward_noalloc(st, B, *map(p, t), 10, 4, *map(p, out), None, None)  # noqa: E731
    assert call() == 0
    torch.cuda.synchronize()
    free0, reserved0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_reserved()
    for _ in range(3):
        assert call() == 0
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_reserved() == reserved0


def test_forward_noalloc_in_a_cuda_graph():
    """After a first call on the device (the buffer's address lookup), the call captures into a CUDA graph; replays
    on new inputs written into the captured buffers equal nb_g1_forward on those inputs bit for bit (the graph holds
    the library's buffer, not caller memory, as the world order's home)."""
    torch, lib, rec = _setup()
    from nablaengine_b200 import synthetic
    B = 1000
    s0 = synthetic.config_states("forward", B=B)
    t = [torch.from_numpy(np.ascontiguousarray(s0[k], np.float32)).cuda() for k in KEYS]
    out = [torch.empty((B, 36), device="cuda"), torch.empty((B, 35), device="cuda"),
           torch.empty((B, 35), device="cuda"), torch.empty((B, 4), dtype=torch.int32, device="cuda")]
    p = lambda x: ctypes.c_void_p(x.data_ptr())  # noqa: E731
    call = lambda: lib.nb_g1_forward_noalloc(  # noqa: E731
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), B, *map(p, t), 10, 4, *map(p, out), None, None)
    assert call() == 0
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        assert call() == 0
    for seed in (4, 5):
        s = synthetic.config_states("vjp", B=B, seed_offset=seed)
        for dst, k in zip(t, KEYS):
            dst.copy_(torch.from_numpy(np.ascontiguousarray(s[k], np.float32)))
        graph.replay()
        torch.cuda.synchronize()
        got = [x.cpu().numpy().view(np.uint32) for x in out]
        want = _run(torch, lib, rec, s, noalloc=False)
        for name, a, b in zip(("qpos'", "qvel'", "warm'", "info"), got, want[:4]):
            assert np.array_equal(a, b), (seed, name)
    del graph


def test_forward_noalloc_rejects_more_worlds_than_its_buffer():
    torch, lib, _ = _setup()
    nul = ctypes.c_void_p(0)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # cudaErrorInvalidValue (1) before any launch or pointer use
    assert lib.nb_g1_forward_noalloc(st, NOALLOC_MAX_WORLDS + 1, *[nul] * 6, 10, 4, *[nul] * 6) == 1
    assert lib.nb_g1_forward_noalloc(st, -1, *[nul] * 6, 10, 4, *[nul] * 6) == 1
    assert lib.nb_g1_forward_noalloc(st, 0, *[nul] * 6, 10, 4, *[nul] * 6) == 0
