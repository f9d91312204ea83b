"""PyTorch interface of the B200 G1 step: the reference's `nablaengine.torch_ffi` API (reference
`src/nablaengine/torch_ffi.py:817` step, :838 kinematics, :845 forward, :854 backward, :884 scale_grad), running the
CUDA kernels of libnabla_g1.so on torch's current stream of the inputs' device.

  step(qpos, qvel, warm, ctrl, friction, com, *, iterations=10, substeps=4, clamp_kv=0, normal=3, clamp_soft=None,
       grad_decay=1.0, kinematics=False) -> (qpos', qvel', warm'[, qpos_n, xpos, xquat, cvel, subtree_com])
  kinematics(qpos, qvel, com) -> (qpos_n, xpos, xquat, cvel, subtree_com)   (differentiable in qpos, qvel)
  forward(qpos, qvel, warm, ctrl, friction, com, *, iterations=10, substeps=4, tape=False, kinematics=False)
      -> (qpos', qvel', warm', info[, tape][, the kinematics outputs])
  backward(tape, friction, com, g_qpos, g_qvel, *, substeps=4, clamp_kv=0, normal=3, ctrl=None, clamp_soft=None)
      -> (g_qpos, g_qvel, g_ctrl, info)
  jacobian(tape, friction, com, *, substeps=4, clamp_kv=1, normal=0, ctrl=None, clamp_soft=None) -> (J, info)
  scale_grad(tree, gamma)

Arguments as the reference: float32 CUDA tensors on one device, contiguous, leading dimension B (the worlds): qpos
(B, 36), qvel (B, 35), warm (B, 35), ctrl (B, 29), friction (B,), com (B, 3). Other dtypes, devices or shapes raise
TypeError (nothing is cast or copied implicitly); bad options raise ValueError. step is differentiable
(torch.autograd): when an input requires grad the forward also writes the tape (B, substeps * REC_WORDS float32) and
keeps it for the backward, the analytic adjoint (deterministic), which returns d/dqpos (qpos form, 36), d/dqvel and
d/dctrl and no gradient for warm, friction and com. The calls only launch kernels and allocate through torch's
caching allocator, so after init(device) they can be captured in a CUDA graph. There is no CPU fallback: without
the CUDA library the call raises.
"""
import atexit
import ctypes
import math
import os
import threading

from . import capi

ITERATIONS, SUBSTEPS, CLAMP_KV, NORMAL = 10, 4, 0, 3
CLAMP_SOFT, GRAD_DECAY = 0.2, 1.0
OVERFLOW_CONTACTS, OVERFLOW_ROWS, UNSUPPORTED = 4, 16, 1
NQ, NV, NU, NBODY, MAXCON = capi.NQ, capi.NV, capi.NU, capi.NBODY, capi.MAXCON
# the device counters (nb_g1_diag_forward / _backward), in the library's order (the reference's DIAG names)
DIAG = ("fwd_calls", "fwd_worlds", "fwd_unsupported_worlds", "fwd_iteration_limit_worlds", "tape_records",
        "refact_records", "nonconv_records", "singular_records", "bwd_calls", "bwd_rows", "nonfinite_rows",
        "nonfinite_qpos_rows", "nonfinite_qvel_rows", "nonfinite_ctrl_rows", "nonfinite_cotangent_rows",
        "replay_mismatch_worlds", "fwd_contact_overflow_worlds", "fwd_row_overflow_worlds")
NONFINITE_QPOS, NONFINITE_QVEL, NONFINITE_CTRL, NONFINITE_COT, NONFINITE_SHIFT = 1, 2, 4, 8, 16

_LOCK = threading.Lock()
_READY = set()
_DIAG = {}                     # device -> int64 (len(DIAG),) counters
_DIAG_ON = [True]
_OVERFLOW_WARN = [os.environ.get("NB_OVERFLOW_WARN", "0") not in ("", "0")]


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
                if int(lib.nb_g1_diag_count()) != len(DIAG):
                    raise _err("the library's diagnostic counters do not match DIAG", RuntimeError)
                import torch as _t
                _DIAG[dev] = _t.zeros((len(DIAG),), dtype=_t.int64, device=f"cuda:{dev}")
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


def _rec_words():
    return int(capi.sizes()[6])


def tape_bytes(nworld, substeps=SUBSTEPS, steps=1):
    """Bytes of the tapes of `steps` differentiated control steps (reference torch_ffi.py:454)."""
    return 4 * _rec_words() * substeps * nworld * steps


def _forward_impl(qpos, qvel, warm, ctrl, friction, com, iterations, substeps, tape=False):
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
    tp = torch.empty((B if tape else 0, substeps * _rec_words()), **kw)
    if B == 0:
        return q1, v1, w1, info, tp
    lib = capi.load()
    nwork = int(lib.nb_g1_work_bytes(B))
    work = torch.empty((nwork,), dtype=torch.uint8, device=qpos.device) if nwork > 0 else None
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.nb_g1_forward(ctypes.c_void_p(st), B, *map(_ptr, (qpos, qvel, warm, ctrl, friction, com)),
                               int(iterations), int(substeps), _ptr(q1), _ptr(v1), _ptr(w1), _ptr(info), None,
                               _ptr(tp) if tape else None, _ptr(work))
    if rc:
        raise _err(f"the forward launch failed (CUDA error {rc})", RuntimeError)
    if _DIAG_ON[0]:
        with torch.cuda.device(dev):
            rc = lib.nb_g1_diag_forward(ctypes.c_void_p(st), _ptr(_DIAG[dev]), B, int(substeps), int(iterations),
                                        _ptr(info), _ptr(tp) if tape else None)
        if rc:
            raise _err(f"the forward diagnostics launch failed (CUDA error {rc})", RuntimeError)
    return q1, v1, w1, info, tp


def _soft(clamp_kv, clamp_soft):
    """The soft clamp's width for clamp_kv 2 (None: CLAMP_SOFT), None for 0 / 1, where it must be None (reference
    torch_ffi.py:436 _soft)."""
    if int(clamp_kv) != 2:
        if clamp_soft is not None:
            raise _err(f"clamp_soft is the soft clamp's (clamp_kv=2), not clamp_kv={clamp_kv}", ValueError)
        return None
    d = float(CLAMP_SOFT if clamp_soft is None else clamp_soft)
    if not (math.isfinite(d) and d >= 0.0):
        raise _err(f"clamp_soft must be finite and >= 0, got {clamp_soft}", ValueError)
    return d


def _backward_impl(tape, friction, com, g_qpos, g_qvel, ctrl, substeps, clamp_kv, normal, clamp_soft):
    import torch
    if not isinstance(tape, torch.Tensor) or tape.device.type != "cuda" or tape.dim() != 2:
        _check("tape", tape, (getattr(tape, "shape", (0,))[0], substeps * _rec_words()), None)
    B, dev = tape.shape[0], tape.device.index
    for name, x, shape in (("tape", tape, (B, substeps * _rec_words())), ("friction", friction, (B,)),
                           ("com", com, (B, 3)), ("g_qpos", g_qpos, (B, NQ)), ("g_qvel", g_qvel, (B, NV))):
        _check(name, x, shape, dev)
    if int(clamp_kv) not in (0, 1, 2) or int(normal) not in (0, 1, 2, 3):
        raise _err(f"no adjoint variant clamp_kv={clamp_kv} normal={normal}", ValueError)
    if (int(clamp_kv) == 2) != (ctrl is not None):
        raise _err("clamp_kv=2 (the soft clamp) needs the step's ctrl; 0 and 1 take none", ValueError)
    if ctrl is not None:
        _check("ctrl", ctrl, (B, NU), dev)
    if not (1 <= substeps <= 32):
        raise _err("substeps in 1..32", ValueError)
    if dev not in _READY:
        init(dev)
    kw = dict(dtype=torch.float32, device=tape.device)
    gq, gv, gu = torch.empty((B, NQ), **kw), torch.empty((B, NV), **kw), torch.empty((B, NU), **kw)
    info = torch.empty((B,), dtype=torch.int32, device=tape.device)
    if B == 0:
        return gq, gv, gu, info
    lib = capi.load()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.nb_g1_adjoint(ctypes.c_void_p(st), B, int(substeps),
                               *map(_ptr, (tape, friction, com, g_qpos, g_qvel, gq, gv, gu, info, ctrl)),
                               ctypes.c_float(clamp_soft), int(clamp_kv), int(normal))
    if rc:
        raise _err(f"the adjoint launch failed (CUDA error {rc})", RuntimeError)
    if _DIAG_ON[0]:
        with torch.cuda.device(dev):
            rc = lib.nb_g1_diag_backward(ctypes.c_void_p(st), _ptr(_DIAG[dev]), B,
                                         *map(_ptr, (gq, gv, gu, g_qpos, g_qvel, info)))
        if rc:
            raise _err(f"the backward diagnostics launch failed (CUDA error {rc})", RuntimeError)
    return gq, gv, gu, info


def jacobian(tape, friction, com, *, substeps=SUBSTEPS, clamp_kv=1, normal=0, ctrl=None, clamp_soft=None):
    """The full step Jacobian from a forward's tape: (J (B, 71, 99) float32, info (B,) int32). Rows: qpos' (36, qpos
    form) then qvel' (35); columns: qpos tangent (35), qvel (35), ctrl (29), each row the VJP of that output's unit
    cotangent (the reference's 71-backward Jacobian, scripts/paper_bench/ours.py:99-110, with its tangent map), in one
    launch. Defaults to the exact gradient mode (clamp_kv=1, normal=0)."""
    import torch
    soft = _soft(clamp_kv, clamp_soft)
    if soft is not None and ctrl is None:
        raise _err("clamp_kv=2 (the soft clamp) needs the step's ctrl", ValueError)
    if not isinstance(tape, torch.Tensor) or tape.device.type != "cuda" or tape.dim() != 2:
        _check("tape", tape, (getattr(tape, "shape", (0,))[0], substeps * _rec_words()), None)
    B, dev = tape.shape[0], tape.device.index
    for name, x, shape in (("tape", tape, (B, substeps * _rec_words())), ("friction", friction, (B,)),
                           ("com", com, (B, 3))):
        _check(name, x, shape, dev)
    if int(normal) not in (0, 1, 2, 3) or not (1 <= substeps <= 32):
        raise _err("normal in 0..3, substeps in 1..32", ValueError)
    if soft is not None:
        _check("ctrl", ctrl, (B, NU), dev)
    if dev not in _READY:
        init(dev)
    J = torch.empty((B, NQ + NV, 2 * NV + NU), dtype=torch.float32, device=tape.device)
    info = torch.empty((B,), dtype=torch.int32, device=tape.device)
    if B == 0:
        return J, info
    lib = capi.load()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.nb_g1_jacobian(ctypes.c_void_p(st), B, int(substeps), _ptr(tape), _ptr(friction), _ptr(com),
                                _ptr(J), _ptr(info), _ptr(ctrl if soft is not None else None),
                                ctypes.c_float(0.0 if soft is None else soft), int(clamp_kv), int(normal))
    if rc:
        raise _err(f"the Jacobian launch failed (CUDA error {rc})", RuntimeError)
    return J, info


def _kinematics_impl(qpos, qvel, com):
    import torch
    if not isinstance(qpos, torch.Tensor) or qpos.device.type != "cuda" or qpos.dim() != 2:
        _check("qpos", qpos, (getattr(qpos, "shape", (0,))[0], NQ), None)
    B, dev = qpos.shape[0], qpos.device.index
    for name, x, shape in (("qpos", qpos, (B, NQ)), ("qvel", qvel, (B, NV)), ("com", com, (B, 3))):
        _check(name, x, shape, dev)
    if dev not in _READY:
        init(dev)
    kw = dict(dtype=torch.float32, device=qpos.device)
    out = (torch.empty((B, NQ), **kw), torch.empty((B, NBODY, 3), **kw), torch.empty((B, NBODY, 4), **kw),
           torch.empty((B, NBODY, 6), **kw), torch.empty((B, NBODY, 3), **kw))
    if B == 0:
        return out
    lib = capi.load()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.nb_g1_kinematics(ctypes.c_void_p(st), B, *map(_ptr, (qpos, qvel, com) + out))
    if rc:
        raise _err(f"the kinematics launch failed (CUDA error {rc})", RuntimeError)
    return out


def _kinematics_backward_impl(qpos, qvel, com, cot, gq_in=None, gv_in=None):
    import torch
    B, dev = qpos.shape[0], qpos.device.index
    shapes = ((B, NQ), (B, NBODY, 3), (B, NBODY, 4), (B, NBODY, 6), (B, NBODY, 3))
    for name, x, shape in zip(("g_qpos_n", "g_xpos", "g_xquat", "g_cvel", "g_subtree_com"), cot, shapes):
        _check(name, x, shape, dev)
    kw = dict(dtype=torch.float32, device=qpos.device)
    gq, gv = torch.empty((B, NQ), **kw), torch.empty((B, NV), **kw)
    if B == 0:
        return gq, gv
    lib = capi.load()
    with torch.cuda.device(dev):
        st = torch.cuda.current_stream(dev).cuda_stream
        rc = lib.nb_g1_kinematics_vjp(ctypes.c_void_p(st), B, *map(_ptr, (qpos, qvel, com) + tuple(cot)),
                                      _ptr(gq_in), _ptr(gv_in), _ptr(gq), _ptr(gv))
    if rc:
        raise _err(f"the kinematics VJP launch failed (CUDA error {rc})", RuntimeError)
    return gq, gv


def _make_kin_fn():
    import torch

    class _Kin(torch.autograd.Function):
        """The kinematics outputs; backward = their VJP (reference torch_ffi.py:787-808)."""

        @staticmethod
        def forward(ctx, qpos, qvel, com):
            out = tuple(_ops()["kinematics"](qpos, qvel, com))
            ctx.save_for_backward(qpos, qvel, com)
            return out

        @staticmethod
        def backward(ctx, *g):
            qpos, qvel, com = ctx.saved_tensors
            B = qpos.shape[0]
            shapes = ((B, NQ), (B, NBODY, 3), (B, NBODY, 4), (B, NBODY, 6), (B, NBODY, 3))
            cot = tuple(qpos.new_zeros(sh) if x is None else x.contiguous() for x, sh in zip(g, shapes))
            gq, gv = _ops()["kinematics_backward"](qpos, qvel, com, *cot)
            return gq, gv, None

    return _Kin


def kinematics(qpos, qvel, com):
    """The kinematics outputs of states (qpos, qvel, com): (qpos_n (B, 36), xpos (B, 31, 3), xquat (B, 31, 4),
    cvel (B, 31, 6), subtree_com (B, 31, 3)), differentiable in qpos and qvel (none for com), as the reference's
    kinematics (torch_ffi.py:838; semantics g1_engine/kinematics.py:1-47)."""
    return _kin_outputs(qpos, qvel, com)


def _kin_outputs(qpos, qvel, com):
    import torch
    if torch.is_grad_enabled() and any(isinstance(x, torch.Tensor) and x.requires_grad for x in (qpos, qvel, com)):
        return _fn("kin", _make_kin_fn).apply(qpos, qvel, com)
    return tuple(_ops()["kinematics"](qpos, qvel, com))


# ---- custom ops (torch.library): the library calls as opaque nodes for torch.compile ---------------------------------
# (reference torch_ffi.py:595-657: nablaengine::forward / backward / kinematics / kinematics_backward with fake impls)
_OPS = {}


def _ops():
    if _OPS:  # (registered: no lock, so torch.compile traces through this lookup)
        return _OPS
    with _LOCK:
        if _OPS:
            return _OPS
        import torch
        from typing import List, Optional
        T = torch.Tensor

        @torch.library.custom_op("nabla_b200::forward", mutates_args=())
        def forward_op(qpos: T, qvel: T, warm: T, ctrl: T, friction: T, com: T, iterations: int, substeps: int,
                       tape: bool) -> List[T]:
            return list(_forward_impl(qpos, qvel, warm, ctrl, friction, com, iterations, substeps, tape))

        @forward_op.register_fake
        def _(qpos, qvel, warm, ctrl, friction, com, iterations, substeps, tape):
            B = qpos.shape[0]
            return [qpos.new_empty((B, NQ)), qpos.new_empty((B, NV)), qpos.new_empty((B, NV)),
                    qpos.new_empty((B, 4), dtype=torch.int32),
                    qpos.new_empty((B if tape else 0, substeps * _rec_words()))]

        @torch.library.custom_op("nabla_b200::backward", mutates_args=())
        def backward_op(tape: T, friction: T, com: T, g_qpos: T, g_qvel: T, ctrl: Optional[T], substeps: int,
                        clamp_kv: int, normal: int, clamp_soft: float) -> List[T]:
            return list(_backward_impl(tape, friction, com, g_qpos, g_qvel, ctrl, substeps, clamp_kv, normal,
                                       clamp_soft))

        @backward_op.register_fake
        def _(tape, friction, com, g_qpos, g_qvel, ctrl, substeps, clamp_kv, normal, clamp_soft):
            B = tape.shape[0]
            return [tape.new_empty((B, NQ)), tape.new_empty((B, NV)), tape.new_empty((B, NU)),
                    tape.new_empty((B,), dtype=torch.int32)]

        @torch.library.custom_op("nabla_b200::kinematics", mutates_args=())
        def kinematics_op(qpos: T, qvel: T, com: T) -> List[T]:
            return list(_kinematics_impl(qpos, qvel, com))

        @kinematics_op.register_fake
        def _(qpos, qvel, com):
            B = qpos.shape[0]
            return [qpos.new_empty((B, NQ)), qpos.new_empty((B, NBODY, 3)), qpos.new_empty((B, NBODY, 4)),
                    qpos.new_empty((B, NBODY, 6)), qpos.new_empty((B, NBODY, 3))]

        @torch.library.custom_op("nabla_b200::kinematics_backward", mutates_args=())
        def kinematics_backward_op(qpos: T, qvel: T, com: T, g_qpos_n: T, g_xpos: T, g_xquat: T, g_cvel: T,
                                   g_subtree_com: T) -> List[T]:
            return list(_kinematics_backward_impl(qpos, qvel, com, (g_qpos_n, g_xpos, g_xquat, g_cvel,
                                                                    g_subtree_com)))

        @kinematics_backward_op.register_fake
        def _(qpos, qvel, com, g_qpos_n, g_xpos, g_xquat, g_cvel, g_subtree_com):
            B = qpos.shape[0]
            return [qpos.new_empty((B, NQ)), qpos.new_empty((B, NV))]

        _OPS.update(forward=forward_op, backward=backward_op, kinematics=kinematics_op,
                    kinematics_backward=kinematics_backward_op)
        return _OPS


def forward(qpos, qvel, warm, ctrl, friction, com, *, iterations=ITERATIONS, substeps=SUBSTEPS, tape=False,
            kinematics=False):
    """One control step without autograd: (qpos', qvel', warm', info (B, 4) int32[, tape][, the kinematics outputs of
    (qpos', qvel')]), as the reference's forward (torch_ffi.py:845): info = [Newton iterations of the last substep,
    its contact count (may exceed 64), its constraint rows, bits 1 unsupported pair / 4 contacts beyond 64 / 16 rows
    beyond 192 over the substeps]."""
    r = _ops()["forward"](qpos, qvel, warm, ctrl, friction, com, int(iterations), int(substeps), bool(tape))
    out = tuple(r) if tape else tuple(r[:4])
    if kinematics:
        out = out + tuple(_ops()["kinematics"](r[0], r[1], com))
    return out


def backward(tape, friction, com, g_qpos, g_qvel, *, substeps=SUBSTEPS, clamp_kv=CLAMP_KV, normal=NORMAL, ctrl=None,
             clamp_soft=None, kinematics=None):
    """The adjoint of one control step from its tape (reference torch_ffi.py:854): (g_qpos (qpos form), g_qvel,
    g_ctrl, info (B,) int32: the replay flags, non-finite bits << 16). kinematics: None, or (qpos', qvel', g_qpos_n,
    g_xpos, g_xquat, g_cvel, g_subtree_com): the output state's kinematics cotangents, pulled back onto (qpos',
    qvel') and added to g_qpos, g_qvel first."""
    soft = _soft(clamp_kv, clamp_soft)
    if soft is not None and ctrl is None:
        raise _err("clamp_kv=2 (the soft clamp) needs the step's ctrl", ValueError)
    if kinematics is not None:
        if len(kinematics) != 7:
            raise _err("kinematics = (qpos', qvel', g_qpos_n, g_xpos, g_xquat, g_cvel, g_subtree_com)", ValueError)
        q1, v1 = kinematics[:2]
        _check("qpos'", q1, (q1.shape[0] if hasattr(q1, "shape") else 0, NQ), None)
        g_qpos, g_qvel = _kinematics_backward_impl(q1, v1, com, tuple(kinematics[2:]), gq_in=g_qpos, gv_in=g_qvel)
    return tuple(_ops()["backward"](tape, friction, com, g_qpos, g_qvel, ctrl if soft is not None else None,
                                    int(substeps), int(clamp_kv), int(normal), 0.0 if soft is None else soft))


def _make_step_fn():
    import torch

    class _Step(torch.autograd.Function):
        """Forward with tape; backward = the analytic adjoint (reference torch_ffi.py:747-779)."""

        @staticmethod
        def forward(ctx, qpos, qvel, warm, ctrl, friction, com, iterations, substeps, clamp_kv, normal, clamp_soft,
                    grad_decay):
            q1, v1, w1, _, tp = _ops()["forward"](qpos, qvel, warm, ctrl, friction, com, iterations, substeps, True)
            ctx.save_for_backward(tp, friction, com, ctrl)
            ctx.opts = (substeps, clamp_kv, normal, clamp_soft, grad_decay)
            ctx.mark_non_differentiable(w1)
            return q1, v1, w1

        @staticmethod
        def backward(ctx, g_q1, g_v1, g_w1):
            tp, friction, com, ctrl = ctx.saved_tensors
            substeps, clamp_kv, normal, clamp_soft, grad_decay = ctx.opts
            B = tp.shape[0]
            g_q1 = tp.new_zeros((B, NQ)) if g_q1 is None else g_q1.contiguous()
            g_v1 = tp.new_zeros((B, NV)) if g_v1 is None else g_v1.contiguous()
            gq, gv, gu, _ = _ops()["backward"](tp, friction, com, g_q1, g_v1, ctrl if clamp_kv == 2 else None,
                                               substeps, clamp_kv, normal, 0.0 if clamp_soft is None else clamp_soft)
            if grad_decay != 1.0:  # the state's cotangent through the physics times grad_decay, ctrl's not
                gq, gv = gq * grad_decay, gv * grad_decay
            return gq, gv, None, gu, None, None, None, None, None, None, None, None

    return _Step


_FNS = {}


def _fn(name, make):
    if name not in _FNS:
        _FNS[name] = make()
    return _FNS[name]


def step(qpos, qvel, warm, ctrl, friction, com, *, iterations=ITERATIONS, substeps=SUBSTEPS, clamp_kv=CLAMP_KV,
         normal=NORMAL, clamp_soft=None, grad_decay=GRAD_DECAY, kinematics=False):
    """One control step: (qpos', qvel', warm') (reference torch_ffi.py:817). Differentiable in qpos, qvel and ctrl when
    an input requires grad (the forward then also writes the tape); warm' is not differentiable. clamp_kv, normal,
    clamp_soft and grad_decay act on the backward only."""
    import torch
    if int(clamp_kv) not in (0, 1, 2) or int(normal) not in (0, 1, 2, 3):
        raise _err("clamp_kv in {0, 1, 2}, normal in 0..3", ValueError)
    soft = _soft(clamp_kv, clamp_soft)
    gd = float(grad_decay)
    if not math.isfinite(gd):
        raise _err(f"grad_decay must be finite, got {grad_decay}", ValueError)
    args = (qpos, qvel, warm, ctrl, friction, com)
    if torch.is_grad_enabled() and any(isinstance(x, torch.Tensor) and x.requires_grad for x in args):
        q1, v1, w1 = _fn("step", _make_step_fn).apply(*args, int(iterations), int(substeps), int(clamp_kv),
                                                      int(normal), soft, gd)
    else:
        q1, v1, w1 = _ops()["forward"](*args, int(iterations), int(substeps), False)[:3]
    if kinematics:  # the output state's kinematics; through autograd their cotangents add to (qpos', qvel')'s
        return (q1, v1, w1) + tuple(_kin_outputs(q1, v1, com))
    return q1, v1, w1


# ---- diagnostics (device counters; reference torch_ffi.py:679-745) -------------------------------------------------

def set_diagnostics(enabled):
    """Switch the device counters and the backward's non-finite info bits on (the default) or off; returns the previous
    setting. They are one small kernel per forward and per backward; outputs and gradients are the same either way."""
    prev = _DIAG_ON[0]
    _DIAG_ON[0] = bool(enabled)
    return prev


def diagnostics(device=None):
    """The device's counters: an int64 (len(DIAG),) CUDA tensor in DIAG order, added to by every call since init or
    the last reset; not copied or synchronised."""
    import torch
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    if dev is None:
        dev = torch.cuda.current_device()
    if dev not in _READY:
        init(dev)
    return _DIAG[dev]


def read_diagnostics(device=None, reset=True):
    """The device's counters as {name: int} (synchronises); reset=True zeroes them afterwards. With
    set_overflow_warnings(True) it warns when worlds exceeded the contact or constraint-row capacity."""
    d = diagnostics(device)
    out = dict(zip(DIAG, (int(x) for x in d.cpu())))
    if reset:
        d.zero_()
    if _OVERFLOW_WARN[0]:
        warn_overflow(out)
    return out


def warn_overflow(d, where="nablaengine_b200"):
    """A RuntimeWarning when the counters d count worlds whose contacts or rows exceeded the per-world capacity (64
    contacts, 192 rows: the excess is dropped, so those worlds miss support and friction forces); returns the count.
    The worlds of one call: info[:, 3] & OVERFLOW_CONTACTS / OVERFLOW_ROWS of forward()."""
    import warnings
    nc, nr = d.get("fwd_contact_overflow_worlds", 0), d.get("fwd_row_overflow_worlds", 0)
    if nc or nr:
        warnings.warn(f"{where}: {nc} world-steps exceeded the contact capacity (64 per world) and {nr} the "
                      f"constraint-row capacity (192); their extra contacts / rows were dropped, so those worlds miss "
                      f"support and friction forces", RuntimeWarning, stacklevel=3)
    return nc + nr


def set_overflow_warnings(enabled):
    """Switch the capacity-overflow warnings on or off (default off, or $NB_OVERFLOW_WARN=1): when on,
    read_diagnostics warns, and counts nobody read are reported once more at exit. Returns the previous setting."""
    prev = _OVERFLOW_WARN[0]
    _OVERFLOW_WARN[0] = bool(enabled)
    return prev


def _exit_report():
    try:
        if not (_DIAG_ON[0] and _OVERFLOW_WARN[0]):
            return
        for dev in sorted(_DIAG):
            warn_overflow(dict(zip(DIAG, (int(x) for x in _DIAG[dev].cpu()))), where=f"nablaengine_b200 (cuda:{dev})")
    except Exception:  # noqa: BLE001  (the interpreter or CUDA shutting down)
        pass


atexit.register(_exit_report)


def _make_scale_fn():
    import torch

    class _Scale(torch.autograd.Function):
        @staticmethod
        def forward(ctx, gamma, *xs):
            ctx.gamma = gamma
            return tuple(x.view_as(x) for x in xs)

        @staticmethod
        def backward(ctx, *g):
            return (None,) + tuple(None if x is None else x * ctx.gamma for x in g)

    return _Scale


def scale_grad(tree, gamma):
    """The identity on a pytree of tensors whose cotangent the backward multiplies by gamma (floating tensors only;
    others pass through), as the reference's scale_grad (torch_ffi.py:884): applied to the carried state at the top
    of each rollout step it gives an exact decay^n per step boundary."""
    import torch
    from torch.utils import _pytree
    g = float(gamma)
    if not math.isfinite(g):
        raise _err(f"scale_grad's gamma must be finite, got {gamma}", ValueError)
    leaves, spec = _pytree.tree_flatten(tree)
    idx = [i for i, x in enumerate(leaves) if isinstance(x, torch.Tensor) and x.is_floating_point()]
    if idx:
        out = _fn("scale", _make_scale_fn).apply(g, *(leaves[i] for i in idx))
        for i, x in zip(idx, out):
            leaves[i] = x
    return _pytree.tree_unflatten(leaves, spec)
