"""PyTorch interface of the B200 G1 step: the reference's `nablaengine.torch_ffi` API (reference
`src/nablaengine/torch_ffi.py:817` step, :838 kinematics, :845 forward, :854 backward, :884 scale_grad), running the
CUDA kernels of libnabla_g1.so on torch's current stream of the inputs' device.

  step(qpos, qvel, warm, ctrl, friction, com, *, iterations=10, substeps=4, clamp_kv=0, normal=3, clamp_soft=None,
       grad_decay=1.0) -> (qpos', qvel', warm')
  forward(qpos, qvel, warm, ctrl, friction, com, *, iterations=10, substeps=4) -> (qpos', qvel', warm', info)

Arguments as the reference: float32 CUDA tensors on one device, contiguous, leading dimension B (the worlds): qpos
(B, 36), qvel (B, 35), warm (B, 35), ctrl (B, 29), friction (B,), com (B, 3). Other dtypes, devices or shapes raise
TypeError (nothing is cast or copied implicitly); bad options raise ValueError. The call only launches kernels and
allocates through torch's caching allocator, so after init(device) it can be captured in a CUDA graph. There is no
CPU fallback: without the CUDA library the call raises.
"""
import ctypes
import math
import threading

from . import capi

ITERATIONS, SUBSTEPS, CLAMP_KV, NORMAL = 10, 4, 0, 3
CLAMP_SOFT, GRAD_DECAY = 0.2, 1.0
OVERFLOW_CONTACTS, OVERFLOW_ROWS, UNSUPPORTED = 4, 16, 1
NQ, NV, NU, NBODY, MAXCON = capi.NQ, capi.NV, capi.NU, capi.NBODY, capi.MAXCON
DIAG = ("fwd_calls", "fwd_worlds", "fwd_unsupported_worlds", "fwd_iteration_limit_worlds",
        "fwd_contact_overflow_worlds", "fwd_row_overflow_worlds")

_LOCK = threading.Lock()
_READY = set()


def _err(msg, exc=TypeError):
    return exc(f"nablaengine_b200.torch_ffi: {msg}")


def init(device=None):
    """Load the library and prepare `device` (default: torch's current CUDA device); idempotent per device. The
    first call on a device synchronises it once: call it before capturing a CUDA graph."""
    import torch
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    if dev is None:
        dev = torch.cuda.current_device()
    with _LOCK:
        lib = capi.load()
        if dev not in _READY:
            with torch.cuda.device(dev):
                if torch.cuda.is_current_stream_capturing():
                    raise _err(f"cuda:{dev} is not prepared: call init({dev}) before capturing a CUDA graph",
                               RuntimeError)
                st = torch.cuda.current_stream(dev)
                rc = lib.nb_g1_upload(None, ctypes.c_void_p(st.cuda_stream))
                if rc:
                    raise _err(f"nb_g1_upload on cuda:{dev} failed (CUDA error {rc})", RuntimeError)
                st.synchronize()
            _READY.add(dev)
    return {"library": str(capi._build.LIB), "nq": NQ, "nv": NV, "nu": NU, "nbody": NBODY, "maxcon": MAXCON}


def _check(name, x, shape, dev):
    import torch
    if not isinstance(x, torch.Tensor):
        raise _err(f"{name} must be a torch.Tensor, got {type(x).__name__}")
    if x.dtype != torch.float32 or tuple(x.shape) != tuple(shape) or x.device.type != "cuda" or not x.is_contiguous():
        raise _err(f"{name} must be a contiguous torch.float32 CUDA tensor {tuple(shape)}, got {x.dtype} "
                   f"{tuple(x.shape)} on {x.device}{'' if x.is_contiguous() else ' (not contiguous)'}")
    if dev is not None and x.device.index != dev:
        raise _err(f"{name} is on {x.device}, the other tensors on cuda:{dev}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _forward_impl(qpos, qvel, warm, ctrl, friction, com, iterations, substeps):
    import torch
    if not isinstance(qpos, torch.Tensor) or qpos.device.type != "cuda":
        _check("qpos", qpos, (getattr(qpos, "shape", (0,))[0], NQ), None)
    if qpos.dim() != 2:
        raise _err(f"qpos must be (B, {NQ}), got {tuple(qpos.shape)}")
    B, dev = qpos.shape[0], qpos.device.index
    for name, x, shape in (("qpos", qpos, (B, NQ)), ("qvel", qvel, (B, NV)), ("warm", warm, (B, NV)),
                           ("ctrl", ctrl, (B, NU)), ("friction", friction, (B,)), ("com", com, (B, 3))):
        _check(name, x, shape, dev)
    if not (1 <= substeps <= 32) or iterations < 0:
        raise _err("substeps in 1..32 and iterations >= 0", ValueError)
    if dev not in _READY:
        init(dev)
    kw = dict(dtype=torch.float32, device=qpos.device)
    q1, v1, w1 = torch.empty((B, NQ), **kw), torch.empty((B, NV), **kw), torch.empty((B, NV), **kw)
    info = torch.empty((B, 4), dtype=torch.int32, device=qpos.device)
    if B == 0:
        return q1, v1, w1, info
    lib = capi.load()
    nwork = int(lib.nb_g1_work_bytes(B))
    work = torch.empty((nwork,), dtype=torch.uint8, device=qpos.device) if nwork > 0 else None
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.nb_g1_forward(ctypes.c_void_p(st), B, *map(_ptr, (qpos, qvel, warm, ctrl, friction, com)),
                               int(iterations), int(substeps), _ptr(q1), _ptr(v1), _ptr(w1), _ptr(info), None, None,
                               _ptr(work))
    if rc:
        raise _err(f"the forward launch failed (CUDA error {rc})", RuntimeError)
    return q1, v1, w1, info


def forward(qpos, qvel, warm, ctrl, friction, com, *, iterations=ITERATIONS, substeps=SUBSTEPS):
    """One control step without autograd: (qpos', qvel', warm', info (B, 4) int32), as the reference's forward:
    info = [Newton iterations of the last substep, its contact count (may exceed 64), its constraint rows, bits
    1 unsupported pair / 4 contacts beyond 64 / 16 rows beyond 192 over the substeps]."""
    return _forward_impl(qpos, qvel, warm, ctrl, friction, com, int(iterations), int(substeps))


def step(qpos, qvel, warm, ctrl, friction, com, *, iterations=ITERATIONS, substeps=SUBSTEPS, clamp_kv=CLAMP_KV,
         normal=NORMAL, clamp_soft=None, grad_decay=GRAD_DECAY):
    """One control step: (qpos', qvel', warm'). The gradient options (clamp_kv, normal, clamp_soft, grad_decay) are
    validated as the reference does."""
    import torch
    if int(clamp_kv) not in (0, 1, 2) or int(normal) not in (0, 1, 2, 3):
        raise _err("clamp_kv in {0, 1, 2}, normal in 0..3", ValueError)
    if int(clamp_kv) != 2 and clamp_soft is not None:
        raise _err(f"clamp_soft is the soft clamp's (clamp_kv=2), not clamp_kv={clamp_kv}", ValueError)
    if not math.isfinite(float(grad_decay)):
        raise _err(f"grad_decay must be finite, got {grad_decay}", ValueError)
    args = (qpos, qvel, warm, ctrl, friction, com)
    if torch.is_grad_enabled() and any(isinstance(x, torch.Tensor) and x.requires_grad for x in args):
        raise _err("the differentiable step (tape + adjoint) is not in this build yet; call it under "
                   "torch.no_grad() or with inputs that do not require grad", NotImplementedError)
    q1, v1, w1, _ = _forward_impl(*args, int(iterations), int(substeps))
    return q1, v1, w1
