"""PyTorch interface of the B200 G1 step, with the API of the reference's `nablaengine.torch_ffi` (reference
`src/nablaengine/torch_ffi.py:817` step, :838 kinematics, :845 forward, :854 backward, :884 scale_grad, :454
tape_bytes, :679-745 diagnostics), running the CUDA kernels of libnabla_g1.so on torch's current stream of the
inputs' device.

  step(qpos, qvel, warm, ctrl, friction, com, *, iterations=10, substeps=4, clamp_kv=0, normal=3, clamp_soft=None,
       grad_decay=1.0, kinematics=False) -> (qpos', qvel', warm'[, qpos_n, xpos, xquat, cvel, subtree_com])
  kinematics(qpos, qvel, com) -> (qpos_n, xpos, xquat, cvel, subtree_com)   (differentiable in qpos, qvel)
  kinematics_backward(qpos, qvel, com, cotangents, g_qpos=None, g_qvel=None) -> (g_qpos, g_qvel)
  forward(qpos, qvel, warm, ctrl, friction, com, *, iterations=10, substeps=4, tape=False, kinematics=False)
      -> (qpos', qvel', warm', info[, tape][, the kinematics outputs])
  backward(tape, friction, com, g_qpos, g_qvel, *, substeps=4, clamp_kv=0, normal=3, ctrl=None, clamp_soft=None)
      -> (g_qpos, g_qvel, g_ctrl, info)
  jacobian(tape, friction, com, *, substeps=4, clamp_kv=1, normal=0, ctrl=None, clamp_soft=None) -> (J, info)
  scale_grad(tree, gamma)
  diagnostics: set_diagnostics, diagnostics, read_diagnostics, warn_overflow, set_overflow_warnings, last_forward

Inputs are float32 CUDA tensors on one device, contiguous, with the worlds as the leading dimension B: qpos (B, 36),
qvel (B, 35), warm (B, 35), ctrl (B, 29), friction (B,), com (B, 3). A tensor of another dtype, device, shape or
layout raises TypeError (nothing is cast or copied behind the caller's back); an option out of range raises
ValueError. step is differentiable through torch.autograd: when an input requires grad, the forward also writes the
tape (B, substeps * tape words) and keeps it for the backward, the analytic adjoint (deterministic), which gives
d/dqpos (qpos form, 36), d/dqvel and d/dctrl, and no gradient for warm, friction and com. The calls launch kernels and
take their outputs from torch's caching allocator, nothing else, so after init(device) they can be captured in a CUDA
graph. There is no CPU fallback: without the CUDA library every call raises.
"""
import atexit
import ctypes
import math
import os
import threading
import warnings

from . import capi

ITERATIONS, SUBSTEPS, CLAMP_KV, NORMAL = 10, 4, 0, 3
CLAMP_SOFT, GRAD_DECAY = 0.2, 1.0
OVERFLOW_CONTACTS, OVERFLOW_ROWS, UNSUPPORTED = 4, 16, 1
NQ, NV, NU, NBODY, MAXCON = capi.NQ, capi.NV, capi.NU, capi.NBODY, capi.MAXCON
NOUT, NTAN = NQ + NV, 2 * NV + NU  # the Jacobian's rows (qpos' in qpos form, qvel') and tangent columns
# the device counters of nb_g1_diag_forward / _backward, in the library's order (named as the reference's)
DIAG = ("fwd_calls", "fwd_worlds", "fwd_unsupported_worlds", "fwd_iteration_limit_worlds", "tape_records",
        "refact_records", "nonconv_records", "singular_records", "bwd_calls", "bwd_rows", "nonfinite_rows",
        "nonfinite_qpos_rows", "nonfinite_qvel_rows", "nonfinite_ctrl_rows", "nonfinite_cotangent_rows",
        "replay_mismatch_worlds", "fwd_contact_overflow_worlds", "fwd_row_overflow_worlds")
NONFINITE_QPOS, NONFINITE_QVEL, NONFINITE_CTRL, NONFINITE_COT, NONFINITE_SHIFT = 1, 2, 4, 8, 16
LAST = ("worlds", "contacts", "max_contacts", "max_rows")  # the last-forward record (nb_g1_last_forward)

# ---- shapes of the arguments: the trailing dimensions after the worlds ------------------------------------------
STATE_ARGS = (("qpos", (NQ,)), ("qvel", (NV,)), ("warm", (NV,)), ("ctrl", (NU,)), ("friction", ()), ("com", (3,)))
KIN_OUTPUTS = (("qpos_n", (NQ,)), ("xpos", (NBODY, 3)), ("xquat", (NBODY, 4)), ("cvel", (NBODY, 6)),
               ("subtree_com", (NBODY, 3)))


class _Settings:
    """Process-wide switches: the device counters (on by default) and the overflow warnings (off by default, or
    $NB_OVERFLOW_WARN=1)."""
    counters = True
    overflow_warnings = os.environ.get("NB_OVERFLOW_WARN", "0") not in ("", "0")


def _fail(msg, kind=TypeError):
    return kind(f"nablaengine_b200.torch_ffi: {msg}")


def _describe(x):
    import torch
    if not isinstance(x, torch.Tensor):
        return type(x).__name__
    return f"{x.dtype} {tuple(x.shape)} on {x.device}" + ("" if x.is_contiguous() else ", not contiguous")


def _validate(args, B=None, dev=None):
    """Check (name, tensor, trailing dims) triples: float32 CUDA tensors, contiguous, shape (B, *trailing), all on
    one device; B and the device default to the first tensor's. Returns (B, device index)."""
    import torch
    for name, x, trailing in args:
        ok = (isinstance(x, torch.Tensor) and x.dtype == torch.float32 and x.device.type == "cuda"
              and x.is_contiguous() and x.dim() == 1 + len(trailing))
        if ok and B is None:
            B = x.shape[0]
        ok = ok and tuple(x.shape) == (B, *trailing)
        if ok and dev is None:
            dev = x.device.index
        if not ok:
            want = ("B",) if B is None else (B,)
            raise _fail(f"{name} must be a contiguous torch.float32 CUDA tensor of shape {want + tuple(trailing)}, "
                        f"got {_describe(x)}")
        if x.device.index != dev:
            raise _fail(f"{name} is on {x.device}, the other arguments on cuda:{dev}")
    return B, dev


def _int_option(name, value, allowed):
    v = int(value)
    if v not in allowed:
        raise _fail(f"{name} must be one of {sorted(allowed)}, got {value}", ValueError)
    return v


def _substeps(value):
    v = int(value)
    if not 1 <= v <= 32:
        raise _fail(f"substeps must be in 1..32, got {value}", ValueError)
    return v


def _soft_width(clamp_kv, clamp_soft):
    """The soft clamp's width: only clamp_kv 2 takes one (default CLAMP_SOFT); None for the other modes."""
    if clamp_kv != 2:
        if clamp_soft is not None:
            raise _fail(f"clamp_soft belongs to the soft clamp (clamp_kv=2), not to clamp_kv={clamp_kv}", ValueError)
        return None
    width = CLAMP_SOFT if clamp_soft is None else float(clamp_soft)
    if not (math.isfinite(width) and width >= 0.0):
        raise _fail(f"clamp_soft must be a finite width >= 0, got {clamp_soft}", ValueError)
    return width


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


_REC_WORDS = {}


def _rec_words(compact=False):
    """Words per world and substep of a tape record (full or compact), asked of the library once."""
    key = bool(compact)
    if key not in _REC_WORDS:
        _REC_WORDS[key] = capi.tape_words(key)
    return _REC_WORDS[key]


def _tape_words(tape, nsub):
    """The record size of a tape argument (full or compact records), from its width; else the full one (for the
    shape check's message)."""
    import torch
    if isinstance(tape, torch.Tensor) and tape.dim() == 2:
        for words in (_rec_words(False), _rec_words(True)):
            if tape.shape[1] == nsub * words:
                return words
    return _rec_words(False)


def tape_bytes(nworld, substeps=SUBSTEPS, steps=1, compact=False):
    """Bytes of the tapes that `steps` differentiated control steps of nworld worlds hold until their backward
    (reference torch_ffi.py:454); compact: the compact tape's records (no L_Q)."""
    return 4 * _rec_words(compact) * substeps * nworld * steps


# ---- per-device state: preparation, counters, last-forward records ------------------------------------------------
class _Device:
    """One CUDA device's state: prepared once (nb_g1_upload), its diagnostic counters (int64, DIAG order, added to on
    the device by every call while counting is on) and its last-forward records (uint32 [LAST]: slot None for the
    last call of any batch size, one per batch size seen)."""

    def __init__(self, index, lib):
        import torch
        self.index = index
        with torch.cuda.device(index):
            if torch.cuda.is_current_stream_capturing():
                raise _fail(f"cuda:{index} is not prepared: call init({index}) before capturing a CUDA graph",
                            RuntimeError)
            stream = torch.cuda.current_stream(index)
            rc = lib.nb_g1_upload(None, ctypes.c_void_p(stream.cuda_stream))
            if rc:
                raise _fail(f"preparing cuda:{index} failed (nb_g1_upload: CUDA error {rc})", RuntimeError)
            if int(lib.nb_g1_diag_count()) != len(DIAG):
                raise _fail("the library counts other diagnostics than DIAG names", RuntimeError)
            self.counters = torch.zeros((len(DIAG),), dtype=torch.int64, device=f"cuda:{index}")
            self.last = {None: torch.zeros((len(LAST),), dtype=torch.int32, device=f"cuda:{index}")}
            stream.synchronize()

    def last_slot(self, B):
        """The record of batch size B (made on first use: call once outside a CUDA graph capture per batch size)."""
        import torch
        if B not in self.last:
            self.last[B] = torch.zeros((len(LAST),), dtype=torch.int32, device=f"cuda:{self.index}")
        return self.last[B]

    def read(self, reset):
        vals = dict(zip(DIAG, (int(v) for v in self.counters.cpu())))
        if reset:
            self.counters.zero_()
        return vals


_LOCK = threading.Lock()
_DEVICES = {}


def _device_index(device):
    import torch
    if device is None:
        return torch.cuda.current_device()
    d = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
    return torch.cuda.current_device() if d.index is None else d.index


def _device(index):
    state = _DEVICES.get(index)
    if state is None:
        with _LOCK:
            state = _DEVICES.get(index)
            if state is None:
                state = _DEVICES[index] = _Device(index, capi.load())
    return state


def init(device=None):
    """Load the library and prepare `device` (default: torch's current CUDA device); idempotent per device. The
    first call on a device synchronises it once: make it before capturing a CUDA graph."""
    _device(_device_index(device))
    return {"library": str(capi._build.LIB), "nq": NQ, "nv": NV, "nu": NU, "nbody": NBODY, "maxcon": MAXCON}


def _launch(dev, entry, *args):
    """Call the library entry on torch's current stream of device dev; a nonzero CUDA error raises."""
    import torch
    lib = capi.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    if torch.cuda.current_device() == dev:  # (the common case: no device switch around the call)
        rc = getattr(lib, entry)(stream, *args)
    else:
        with torch.cuda.device(dev):
            rc = getattr(lib, entry)(stream, *args)
    if rc:
        raise _fail(f"{entry} failed (CUDA error {rc})", RuntimeError)


# ---- the library calls --------------------------------------------------------------------------------------------
def _forward_impl(qpos, qvel, warm, ctrl, friction, com, iterations, substeps, tape=False, compact=False):
    import torch
    B, dev = _validate([(n, x, t) for (n, t), x in zip(STATE_ARGS, (qpos, qvel, warm, ctrl, friction, com))])
    nsub, iters = _substeps(substeps), int(iterations)
    if iters < 0:
        raise _fail(f"iterations must be >= 0, got {iterations}", ValueError)
    state = _device(dev)
    f32 = dict(dtype=torch.float32, device=qpos.device)
    outs = (torch.empty((B, NQ), **f32), torch.empty((B, NV), **f32), torch.empty((B, NV), **f32),
            torch.empty((B, 4), dtype=torch.int32, device=qpos.device))
    words = _rec_words(compact)
    tp = torch.empty((B if tape else 0, nsub * words), **f32)
    if B == 0:
        return outs + (tp,)
    nwork = int(capi.load().nb_g1_work_bytes(B))
    work = torch.empty((nwork,), dtype=torch.uint8, device=qpos.device)
    _launch(dev, "nb_g1_forward_ex", B, *map(_p, (qpos, qvel, warm, ctrl, friction, com)), iters, nsub,
            *map(_p, outs[:4]), None, _p(tp) if tape else None, _p(work), words)
    if _Settings.counters:
        _launch(dev, "nb_g1_diag_forward_ex", _p(state.counters), B, nsub, iters, _p(outs[3]),
                _p(tp) if tape else None, words)
        _launch(dev, "nb_g1_last_forward", B, _p(outs[3]), _p(state.last[None]), _p(state.last_slot(B)))
    return outs + (tp,)


def _backward_impl(tape, friction, com, g_qpos, g_qvel, ctrl, substeps, clamp_kv, normal, clamp_soft):
    import torch
    nsub = _substeps(substeps)
    kv = _int_option("clamp_kv", clamp_kv, {0, 1, 2})
    nm = _int_option("normal", normal, {0, 1, 2, 3})
    if (kv == 2) != (ctrl is not None):
        raise _fail("the soft clamp (clamp_kv=2) needs the step's ctrl, and only it takes one", ValueError)
    words = _tape_words(tape, nsub)
    args = [("tape", tape, (nsub * words,)), ("friction", friction, ()), ("com", com, (3,)),
            ("g_qpos", g_qpos, (NQ,)), ("g_qvel", g_qvel, (NV,))]
    if ctrl is not None:
        args.append(("ctrl", ctrl, (NU,)))
    B, dev = _validate(args)
    state = _device(dev)
    f32 = dict(dtype=torch.float32, device=tape.device)
    outs = (torch.empty((B, NQ), **f32), torch.empty((B, NV), **f32), torch.empty((B, NU), **f32),
            torch.empty((B,), dtype=torch.int32, device=tape.device))
    if B == 0:
        return outs
    _launch(dev, "nb_g1_adjoint_ex", B, nsub, *map(_p, (tape, friction, com, g_qpos, g_qvel) + outs + (ctrl,)),
            ctypes.c_float(clamp_soft), kv, nm, words)
    if _Settings.counters:
        _launch(dev, "nb_g1_diag_backward", _p(state.counters), B, *map(_p, outs[:3] + (g_qpos, g_qvel, outs[3])))
    return outs


def _kinematics_impl(qpos, qvel, com):
    import torch
    B, dev = _validate([("qpos", qpos, (NQ,)), ("qvel", qvel, (NV,)), ("com", com, (3,))])
    _device(dev)
    outs = tuple(torch.empty((B, *t), dtype=torch.float32, device=qpos.device) for _, t in KIN_OUTPUTS)
    if B:
        _launch(dev, "nb_g1_kinematics", B, *map(_p, (qpos, qvel, com) + outs))
    return outs


def _kinematics_backward_impl(qpos, qvel, com, cot, gq_in=None, gv_in=None):
    import torch
    cot = tuple(cot)
    if len(cot) != len(KIN_OUTPUTS):
        raise _fail(f"the kinematics cotangents are {len(KIN_OUTPUTS)} tensors, got {len(cot)}", ValueError)
    args = [("qpos", qpos, (NQ,)), ("qvel", qvel, (NV,)), ("com", com, (3,))]
    args += [(f"g_{n}", x, t) for (n, t), x in zip(KIN_OUTPUTS, cot)]
    args += [(n, x, t) for n, x, t in (("g_qpos", gq_in, (NQ,)), ("g_qvel", gv_in, (NV,))) if x is not None]
    B, dev = _validate(args)
    _device(dev)
    gq, gv = (torch.empty((B, n), dtype=torch.float32, device=qpos.device) for n in (NQ, NV))
    if B:
        _launch(dev, "nb_g1_kinematics_vjp", B, *map(_p, (qpos, qvel, com) + cot + (gq_in, gv_in, gq, gv)))
    return gq, gv


def jacobian(tape, friction, com, *, substeps=SUBSTEPS, clamp_kv=1, normal=0, ctrl=None, clamp_soft=None):
    """The full step Jacobian from a forward's tape: (J (B, 71, 99) float32, info (B,) int32). Rows: qpos' (36, qpos
    form) then qvel' (35); columns: the qpos tangent (35), qvel (35), ctrl (29); each row is the VJP of that output's
    unit cotangent (the reference's Jacobian of 71 backward calls, scripts/paper_bench/ours.py:99-110, with its
    tangent map), all in one launch. The default is the exact gradient mode (clamp_kv=1, normal=0)."""
    import torch
    nsub = _substeps(substeps)
    kv = _int_option("clamp_kv", clamp_kv, {0, 1, 2})
    nm = _int_option("normal", normal, {0, 1, 2, 3})
    width = _soft_width(kv, clamp_soft)
    if (kv == 2) != (ctrl is not None):
        raise _fail("the soft clamp (clamp_kv=2) needs the step's ctrl, and only it takes one", ValueError)
    words = _tape_words(tape, nsub)
    args = [("tape", tape, (nsub * words,)), ("friction", friction, ()), ("com", com, (3,))]
    if ctrl is not None:
        args.append(("ctrl", ctrl, (NU,)))
    B, dev = _validate(args)
    _device(dev)
    J = torch.empty((B, NOUT, NTAN), dtype=torch.float32, device=tape.device)
    info = torch.empty((B,), dtype=torch.int32, device=tape.device)
    if B:
        _launch(dev, "nb_g1_jacobian_ex", B, nsub, *map(_p, (tape, friction, com, J, info, ctrl)),
                ctypes.c_float(0.0 if width is None else width), kv, nm, words)
    return J, info


# ---- custom ops (torch.library): the library calls as opaque graph nodes, traced by torch.compile ---------------
# (the reference registers nablaengine::forward / backward / kinematics / kinematics_backward, torch_ffi.py:595-657)
_OPS = {}


def _register_ops():
    import torch
    from typing import List, Optional
    T = torch.Tensor

    def empty_like_outputs(x, shapes):
        return [x.new_empty(s, dtype=d) for s, d in shapes]

    @torch.library.custom_op("nabla_b200::forward", mutates_args=())
    def forward_op(qpos: T, qvel: T, warm: T, ctrl: T, friction: T, com: T, iterations: int, substeps: int,
                   tape: bool, compact: bool = False) -> List[T]:
        return list(_forward_impl(qpos, qvel, warm, ctrl, friction, com, iterations, substeps, tape, compact))

    @forward_op.register_fake
    def _(qpos, qvel, warm, ctrl, friction, com, iterations, substeps, tape, compact=False):
        B = qpos.shape[0]
        return empty_like_outputs(qpos, [((B, NQ), None), ((B, NV), None), ((B, NV), None), ((B, 4), torch.int32),
                                         ((B if tape else 0, substeps * _rec_words(compact)), None)])

    @torch.library.custom_op("nabla_b200::backward", mutates_args=())
    def backward_op(tape: T, friction: T, com: T, g_qpos: T, g_qvel: T, ctrl: Optional[T], substeps: int,
                    clamp_kv: int, normal: int, clamp_soft: float) -> List[T]:
        return list(_backward_impl(tape, friction, com, g_qpos, g_qvel, ctrl, substeps, clamp_kv, normal, clamp_soft))

    @backward_op.register_fake
    def _(tape, friction, com, g_qpos, g_qvel, ctrl, substeps, clamp_kv, normal, clamp_soft):
        B = tape.shape[0]
        return empty_like_outputs(tape, [((B, NQ), None), ((B, NV), None), ((B, NU), None), ((B,), torch.int32)])

    @torch.library.custom_op("nabla_b200::kinematics", mutates_args=())
    def kinematics_op(qpos: T, qvel: T, com: T) -> List[T]:
        return list(_kinematics_impl(qpos, qvel, com))

    @kinematics_op.register_fake
    def _(qpos, qvel, com):
        B = qpos.shape[0]
        return empty_like_outputs(qpos, [((B, *t), None) for _, t in KIN_OUTPUTS])

    @torch.library.custom_op("nabla_b200::kinematics_backward", mutates_args=())
    def kinematics_backward_op(qpos: T, qvel: T, com: T, g_qpos_n: T, g_xpos: T, g_xquat: T, g_cvel: T,
                               g_subtree_com: T) -> List[T]:
        return list(_kinematics_backward_impl(qpos, qvel, com, (g_qpos_n, g_xpos, g_xquat, g_cvel, g_subtree_com)))

    @kinematics_backward_op.register_fake
    def _(qpos, qvel, com, g_qpos_n, g_xpos, g_xquat, g_cvel, g_subtree_com):
        B = qpos.shape[0]
        return empty_like_outputs(qpos, [((B, NQ), None), ((B, NV), None)])

    return {"forward": forward_op, "backward": backward_op, "kinematics": kinematics_op,
            "kinematics_backward": kinematics_backward_op}


def custom_ops():
    """{name: op} of the torch.library custom ops nabla_b200::forward / backward / kinematics / kinematics_backward
    (registered on first use)."""
    if not _OPS:  # (once registered, no lock: torch.compile traces through this lookup)
        with _LOCK:
            if not _OPS:
                _OPS.update(_register_ops())
    return _OPS


# ---- autograd ---------------------------------------------------------------------------------------------------
_FUNCTIONS = {}


def _autograd_function(name):
    """The torch.autograd.Function classes, made on first use (torch is imported lazily)."""
    if name in _FUNCTIONS:
        return _FUNCTIONS[name]
    import torch

    class StepFunction(torch.autograd.Function):
        """Forward with tape; backward = the analytic adjoint on that tape."""

        @staticmethod
        def forward(ctx, qpos, qvel, warm, ctrl, friction, com, opts):
            q1, v1, w1, _, tp = custom_ops()["forward"](qpos, qvel, warm, ctrl, friction, com, opts["iterations"],
                                                        opts["substeps"], True, opts["compact_tape"])
            ctx.save_for_backward(tp, friction, com, ctrl)
            ctx.opts = opts
            ctx.mark_non_differentiable(w1)
            return q1, v1, w1

        @staticmethod
        def backward(ctx, g_q1, g_v1, _g_w1):
            tp, friction, com, ctrl = ctx.saved_tensors
            o = ctx.opts
            B = tp.shape[0]
            g_q1 = tp.new_zeros((B, NQ)) if g_q1 is None else g_q1.contiguous()
            g_v1 = tp.new_zeros((B, NV)) if g_v1 is None else g_v1.contiguous()
            soft = o["clamp_soft"]
            gq, gv, gu, _ = custom_ops()["backward"](tp, friction, com, g_q1, g_v1, ctrl if soft is not None else None,
                                                     o["substeps"], o["clamp_kv"], o["normal"],
                                                     0.0 if soft is None else soft)
            decay = o["grad_decay"]
            if decay != 1.0:  # the state's cotangent through the physics is decayed, the control's is not
                gq, gv = gq * decay, gv * decay
            return gq, gv, None, gu, None, None, None

    class KinematicsFunction(torch.autograd.Function):
        """The kinematics outputs; backward = their VJP."""

        @staticmethod
        def forward(ctx, qpos, qvel, com):
            ctx.save_for_backward(qpos, qvel, com)
            return tuple(custom_ops()["kinematics"](qpos, qvel, com))

        @staticmethod
        def backward(ctx, *grads):
            qpos, qvel, com = ctx.saved_tensors
            B = qpos.shape[0]
            cot = [qpos.new_zeros((B, *t)) if g is None else g.contiguous() for g, (_, t) in zip(grads, KIN_OUTPUTS)]
            gq, gv = custom_ops()["kinematics_backward"](qpos, qvel, com, *cot)
            return gq, gv, None

    class GradScale(torch.autograd.Function):
        """The identity on one tensor whose cotangent is multiplied by a constant."""

        @staticmethod
        def forward(ctx, x, gamma):
            ctx.gamma = gamma
            return x.view_as(x)

        @staticmethod
        def backward(ctx, g):
            return (None if g is None else g * ctx.gamma), None

    _FUNCTIONS.update(step=StepFunction, kinematics=KinematicsFunction, scale=GradScale)
    return _FUNCTIONS[name]


def _tracing():
    """True while torch.compile traces: the library calls then go through their custom ops (opaque graph nodes);
    eager calls go straight to the implementation (the same launches, without the dispatcher's overhead)."""
    import torch
    return torch.compiler.is_compiling()


def _differentiating(*xs):
    import torch
    return torch.is_grad_enabled() and any(isinstance(x, torch.Tensor) and x.requires_grad for x in xs)


# ---- the public API ---------------------------------------------------------------------------------------------
def forward(qpos, qvel, warm, ctrl, friction, com, *, iterations=ITERATIONS, substeps=SUBSTEPS, tape=False,
            kinematics=False):
    """One control step without autograd (reference torch_ffi.py:845): (qpos', qvel', warm', info (B, 4) int32
    [, tape][, the kinematics outputs of (qpos', qvel')]). info = [Newton iterations of the last substep, the
    contacts its collision found (may exceed 64), its constraint rows, bits 1 unsupported pair / 4 contacts beyond 64 /
    16 rows beyond 192, ORed over the substeps]. tape: False, True (full records) or "compact" (records without the
    factor of M + h kv, which backward and jacobian rebuild: 31 % less tape); backward and jacobian take either."""
    if tape not in (False, True, "compact"):
        raise _fail(f"tape must be False, True or 'compact', got {tape!r}", ValueError)
    args = (qpos, qvel, warm, ctrl, friction, com, int(iterations), int(substeps), bool(tape), tape == "compact")
    r = custom_ops()["forward"](*args) if _tracing() else _forward_impl(*args)
    out = tuple(r) if tape else tuple(r[:4])
    if kinematics:
        out += tuple(custom_ops()["kinematics"](r[0], r[1], com))
    return out


def kinematics_backward(qpos, qvel, com, cotangents, g_qpos=None, g_qvel=None):
    """The VJP of kinematics(qpos, qvel, com) with the five outputs' cotangents: (g_qpos (qpos form), g_qvel);
    g_qpos / g_qvel, when given, are added to the result (a step's own output cotangents)."""
    return _kinematics_backward_impl(qpos, qvel, com, cotangents, gq_in=g_qpos, gv_in=g_qvel)


def backward(tape, friction, com, g_qpos, g_qvel, *, substeps=SUBSTEPS, clamp_kv=CLAMP_KV, normal=NORMAL, ctrl=None,
             clamp_soft=None, kinematics=None):
    """The adjoint of one control step from its tape (reference torch_ffi.py:854): (g_qpos (qpos form), g_qvel,
    g_ctrl, info (B,) int32: the replay flags, with the non-finite bits << 16 while counting is on). kinematics: None,
    or (qpos', qvel', g_qpos_n, g_xpos, g_xquat, g_cvel, g_subtree_com): cotangents of the output state's kinematics,
    pulled back onto (qpos', qvel') and added to g_qpos, g_qvel first."""
    kv = _int_option("clamp_kv", clamp_kv, {0, 1, 2})
    width = _soft_width(kv, clamp_soft)
    if kv == 2 and ctrl is None:
        raise _fail("the soft clamp (clamp_kv=2) needs the step's ctrl", ValueError)
    if kinematics is not None:
        if len(kinematics) != 2 + len(KIN_OUTPUTS):
            raise _fail("kinematics = (qpos', qvel', g_qpos_n, g_xpos, g_xquat, g_cvel, g_subtree_com)", ValueError)
        g_qpos, g_qvel = kinematics_backward(kinematics[0], kinematics[1], com, kinematics[2:], g_qpos, g_qvel)
    return tuple(custom_ops()["backward"](tape, friction, com, g_qpos, g_qvel, ctrl if width is not None else None,
                                          int(substeps), kv, int(normal), 0.0 if width is None else width))


def kinematics(qpos, qvel, com):
    """The kinematics outputs of states (qpos, qvel, com) (reference torch_ffi.py:838; semantics
    g1_engine/kinematics.py:1-47): (qpos_n (B, 36), xpos (B, 31, 3), xquat (B, 31, 4), cvel (B, 31, 6),
    subtree_com (B, 31, 3)), differentiable in qpos and qvel (com gets no gradient)."""
    if _differentiating(qpos, qvel, com):
        return _autograd_function("kinematics").apply(qpos, qvel, com)
    return tuple(custom_ops()["kinematics"](qpos, qvel, com))


def step(qpos, qvel, warm, ctrl, friction, com, *, iterations=ITERATIONS, substeps=SUBSTEPS, clamp_kv=CLAMP_KV,
         normal=NORMAL, clamp_soft=None, grad_decay=GRAD_DECAY, kinematics=False, compact_tape=False):
    """One control step (reference torch_ffi.py:817): (qpos', qvel', warm'). Differentiable in qpos, qvel and ctrl
    when an input requires grad (the forward then also writes the tape; compact_tape=True: the compact records, kept
    until the backward in 31 % less memory, the backward rebuilding the factor of M + h kv); warm' is not
    differentiable. clamp_kv, normal, clamp_soft and grad_decay select the backward; with kinematics=True the output
    state's kinematics follow, and their cotangents flow back into (qpos', qvel')'s."""
    kv = _int_option("clamp_kv", clamp_kv, {0, 1, 2})
    nm = _int_option("normal", normal, {0, 1, 2, 3})
    opts = {"iterations": int(iterations), "substeps": int(substeps), "clamp_kv": kv, "normal": nm,
            "clamp_soft": _soft_width(kv, clamp_soft), "grad_decay": float(grad_decay),
            "compact_tape": bool(compact_tape)}
    if not math.isfinite(opts["grad_decay"]):
        raise _fail(f"grad_decay must be finite, got {grad_decay}", ValueError)
    state = (qpos, qvel, warm, ctrl, friction, com)
    if _differentiating(*state):
        q1, v1, w1 = _autograd_function("step").apply(*state, opts)
    else:
        args = state + (opts["iterations"], opts["substeps"], False)
        q1, v1, w1 = (custom_ops()["forward"](*args) if _tracing() else _forward_impl(*args))[:3]
    if kinematics:
        return (q1, v1, w1) + tuple(globals()["kinematics"](q1, v1, com))
    return q1, v1, w1


def scale_grad(tree, gamma):
    """The identity on a pytree of tensors whose floating tensors' cotangents the backward multiplies by gamma (other
    leaves pass through), as the reference's scale_grad (torch_ffi.py:884): applied to the carried state at the top
    of each rollout step it decays the gradient by gamma per step boundary."""
    import torch
    from torch.utils import _pytree
    g = float(gamma)
    if not math.isfinite(g):
        raise _fail(f"scale_grad's gamma must be finite, got {gamma}", ValueError)
    fn = _autograd_function("scale")
    return _pytree.tree_map(lambda x: fn.apply(x, g) if isinstance(x, torch.Tensor) and x.is_floating_point() else x,
                            tree)


# ---- diagnostics -------------------------------------------------------------------------------------------------
def set_diagnostics(enabled):
    """Switch the device counters, the last-forward records and the backward's non-finite info bits on (the default)
    or off; returns the previous setting. They cost one or two small kernels per call; outputs and gradients are the
    same either way."""
    prev, _Settings.counters = _Settings.counters, bool(enabled)
    return prev


def diagnostics_enabled():
    return _Settings.counters


def diagnostics(device=None):
    """The device's counters: an int64 (len(DIAG),) CUDA tensor in DIAG order, added to by every call since init or
    the last reset (no copy, no synchronisation)."""
    return _device(_device_index(device)).counters


def read_diagnostics(device=None, reset=True):
    """The device's counters as {name: int} (synchronises); reset=True zeroes them after reading. With
    set_overflow_warnings(True) it also warns about worlds that exceeded the contact or constraint-row capacity."""
    vals = _device(_device_index(device)).read(reset)
    if _Settings.overflow_warnings:
        warn_overflow(vals)
    return vals


def last_forward(nworld=None, device=None):
    """{LAST name: int} of the last forward on the device (nworld None) or of the last one with nworld worlds: the
    worlds, the contacts summed over the worlds, and the most contacts and constraint rows of one world, each from the
    last substep (reference jax_ffi.py:1487 last_forward); zeros when there was none, or while counting was off.
    Synchronises."""
    state = _device(_device_index(device))
    rec = state.last.get(None if nworld is None else int(nworld))
    if rec is None:
        return dict.fromkeys(LAST, 0)
    return {k: int(v) & 0xFFFFFFFF for k, v in zip(LAST, rec.cpu())}


def launch_info(device=None):
    """The kernels' launch shapes on the device (nb_g1_launch): shared memory per block and resident worlds per SM
    of the forward and the adjoint, the Jacobian's shared memory per block and resident cotangents (Jacobian rows in
    flight, 70 per world) per SM, and the SM count."""
    index = _device_index(device)
    _device(index)
    out = (ctypes.c_longlong * 8)()
    rc = capi.load().nb_g1_launch(index, out)
    if rc:
        raise _fail(f"nb_g1_launch failed (CUDA error {rc})", RuntimeError)
    names = ("forward_smem_bytes", "forward_worlds_per_sm", "adjoint_smem_bytes", "adjoint_worlds_per_sm",
             "jacobian_smem_bytes", "jacobian_rows_per_sm", "sms")
    return dict(zip(names, out[:7]))


def warn_overflow(counts, where="nablaengine_b200"):
    """Warn (RuntimeWarning) when the counters in `counts` saw worlds beyond the per-world capacity, 64 contacts or 192
    constraint rows (the excess is dropped: such a world loses contact forces); returns how many world-steps did. For
    one call: forward()'s info[:, 3] & OVERFLOW_CONTACTS / OVERFLOW_ROWS."""
    ncon = counts.get("fwd_contact_overflow_worlds", 0)
    nrow = counts.get("fwd_row_overflow_worlds", 0)
    if ncon or nrow:
        warnings.warn(f"{where}: world-steps past the contact capacity (64 per world): {ncon}; past the constraint-row "
                      f"capacity (192): {nrow}. Their extra contacts or rows were left out of the solve.",
                      RuntimeWarning, stacklevel=3)
    return ncon + nrow


def set_overflow_warnings(enabled):
    """Switch the capacity warnings on or off (default off, or $NB_OVERFLOW_WARN=1): when on, read_diagnostics warns,
    and at exit the counts nobody read are reported once more. Returns the previous setting."""
    prev, _Settings.overflow_warnings = _Settings.overflow_warnings, bool(enabled)
    return prev


@atexit.register
def _report_unread_overflow():
    if not (_Settings.counters and _Settings.overflow_warnings):
        return
    try:
        for index, state in sorted(_DEVICES.items()):
            warn_overflow(state.read(reset=False), where=f"nablaengine_b200 (cuda:{index})")
    except Exception:  # noqa: BLE001  (CUDA or the interpreter already shutting down)
        pass
