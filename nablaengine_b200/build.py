"""Build the CUDA library libnabla_g1.so for sm_100a, in-tree (nablaengine_b200/lib/).

nvcc cross-compiles without a GPU, so this runs anywhere the CUDA toolkit is installed; the built .so travels with
the repository to the GPU machines. `python -m nablaengine_b200.build` rebuilds when a source is newer than the
library or the library was built with other nvcc flags (recorded in a stamp file beside it).
"""
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libnabla_g1.so"
SOURCES = [CSRC / "nb_g1.cu"]
DEPS = SOURCES + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [PKG.parent / "include" / "nabla_g1.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared", "--cudart", "shared"]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libnabla_g1.so")


def _stamp(lib):
    return lib.with_name(lib.name + ".flags")


def _flags_text(extra):
    return " ".join([*ARCH, *FLAGS, *extra])


def stale(lib=LIB, extra=()):
    """True when `lib` is missing, older than a source, or was built with other nvcc flags (the stamp file beside it
    records them)."""
    if not lib.exists():
        return True
    t = lib.stat().st_mtime
    if any(p.stat().st_mtime > t for p in DEPS):
        return True
    stamp = _stamp(lib)
    return not stamp.exists() or stamp.read_text() != _flags_text(extra)


PROFILE_LIB = LIBDIR / "libnabla_g1_prof.so"


def build(force=False, verbose=False, extra=(), out=None):
    """Compile the library when it is missing, older than its sources or built with other flags; returns its path.
    `out` and `extra`: another output path and extra nvcc flags (the phase-profile build: -DNB_PROFILE into
    PROFILE_LIB)."""
    lib = Path(out) if out else LIB
    if not force and not stale(lib, extra):
        return lib
    LIBDIR.mkdir(exist_ok=True)
    tmp = lib.with_suffix(f".tmp{os.getpid()}.so")
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"nvcc failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(r.stderr, flush=True)
    os.replace(tmp, lib)
    _stamp(lib).write_text(_flags_text(extra))
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
