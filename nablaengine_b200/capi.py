"""ctypes binding of libnabla_g1.so (the C ABI of include/nabla_g1.h).

The library is the only compute path: if it is missing or does not export the ABI, load() raises. Nothing here falls
back to a CPU or PyTorch implementation.
"""
import ctypes
import threading
from pathlib import Path

from . import build as _build

HEADER = Path(__file__).resolve().parents[1] / "include" / "nabla_g1.h"
EXPORTS = ("nb_g1_sizes", "nb_g1_work_bytes", "nb_g1_upload", "nb_g1_forward", "nb_g1_forward_stats",
           "nb_g1_adjoint", "nb_g1_jacobian", "nb_g1_kinematics", "nb_g1_kinematics_vjp", "nb_g1_diag_count",
           "nb_g1_diag_forward", "nb_g1_diag_backward", "nb_g1_forward_noalloc", "nb_g1_last_forward",
           "nb_g1_launch", "nb_g1_tape_words", "nb_g1_forward_ex", "nb_g1_adjoint_ex", "nb_g1_jacobian_ex",
           "nb_g1_diag_forward_ex")
ABI_VERSION = 4
NQ, NV, NU, NBODY, MAXCON, NEFC = 36, 35, 29, 31, 64, 192

_LOCK = threading.Lock()
_LIB = []


def declared_symbols():
    """The function names include/nabla_g1.h declares (what the library must export)."""
    import re
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(nb_g1_\w+)\s*\(", text)))


def load(path=None, build_if_missing=True):
    """The loaded library (ctypes.CDLL) with argument types set; builds it first when it is missing and nvcc exists."""
    with _LOCK:
        if _LIB:
            return _LIB[0]
        lib_path = Path(path) if path else _build.LIB
        if not lib_path.exists():
            if not build_if_missing:
                raise RuntimeError(f"{lib_path} is missing: run `python -m nablaengine_b200.build`")
            _build.build()
        lib = ctypes.CDLL(str(lib_path))
        for name in EXPORTS:
            if not hasattr(lib, name):
                raise RuntimeError(f"{lib_path} does not export {name}")
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
        lib.nb_g1_sizes.argtypes, lib.nb_g1_sizes.restype = [vp], None
        lib.nb_g1_work_bytes.argtypes, lib.nb_g1_work_bytes.restype = [i32], i64
        lib.nb_g1_upload.argtypes, lib.nb_g1_upload.restype = [vp, vp], i32
        lib.nb_g1_forward.argtypes = [vp, i32] + [vp] * 6 + [i32, i32] + [vp] * 7
        lib.nb_g1_forward.restype = i32
        lib.nb_g1_forward_stats.argtypes = [vp, i32] + [vp] * 6 + [i32, i32] + [vp] * 5
        lib.nb_g1_forward_stats.restype = i32
        lib.nb_g1_forward_noalloc.argtypes = [vp, i32] + [vp] * 6 + [i32, i32] + [vp] * 6
        lib.nb_g1_forward_noalloc.restype = i32
        lib.nb_g1_adjoint.argtypes = [vp, i32, i32] + [vp] * 10 + [ctypes.c_float, i32, i32]
        lib.nb_g1_adjoint.restype = i32
        lib.nb_g1_jacobian.argtypes = [vp, i32, i32] + [vp] * 6 + [ctypes.c_float, i32, i32]
        lib.nb_g1_jacobian.restype = i32
        lib.nb_g1_kinematics.argtypes, lib.nb_g1_kinematics.restype = [vp, i32] + [vp] * 8, i32
        lib.nb_g1_kinematics_vjp.argtypes, lib.nb_g1_kinematics_vjp.restype = [vp, i32] + [vp] * 12, i32
        lib.nb_g1_diag_count.argtypes, lib.nb_g1_diag_count.restype = [], i64
        lib.nb_g1_diag_forward.argtypes, lib.nb_g1_diag_forward.restype = [vp, vp, i32, i32, i32, vp, vp], i32
        lib.nb_g1_diag_backward.argtypes, lib.nb_g1_diag_backward.restype = [vp, vp, i32] + [vp] * 6, i32
        lib.nb_g1_last_forward.argtypes, lib.nb_g1_last_forward.restype = [vp, i32, vp, vp, vp], i32
        lib.nb_g1_launch.argtypes, lib.nb_g1_launch.restype = [i32, vp], i32
        lib.nb_g1_tape_words.argtypes, lib.nb_g1_tape_words.restype = [i32], i64
        lib.nb_g1_forward_ex.argtypes = lib.nb_g1_forward.argtypes + [i32]
        lib.nb_g1_forward_ex.restype = i32
        lib.nb_g1_adjoint_ex.argtypes = lib.nb_g1_adjoint.argtypes + [i32]
        lib.nb_g1_adjoint_ex.restype = i32
        lib.nb_g1_jacobian_ex.argtypes = lib.nb_g1_jacobian.argtypes + [i32]
        lib.nb_g1_jacobian_ex.restype = i32
        lib.nb_g1_diag_forward_ex.argtypes = lib.nb_g1_diag_forward.argtypes + [i32]
        lib.nb_g1_diag_forward_ex.restype = i32
        sizes = (ctypes.c_longlong * 8)()
        lib.nb_g1_sizes(sizes)
        want = (NQ, NV, NU, NBODY, MAXCON, NEFC)
        if tuple(sizes[:6]) != want or sizes[7] != ABI_VERSION:
            raise RuntimeError(f"{lib_path}: compiled sizes {list(sizes)} do not match {want} / ABI {ABI_VERSION}")
        _LIB.append(lib)
        return lib


def sizes():
    out = (ctypes.c_longlong * 8)()
    load().nb_g1_sizes(out)
    return list(out)


def tape_words(compact=False):
    """Words per world and substep of a tape record: full, or compact (no L_Q: rebuilt by the tape's readers)."""
    return int(load().nb_g1_tape_words(1 if compact else 0))
