"""Build recipe for the sm_100a library ``leap_b200/lib/libleap_b200.so``.

Every ``leap_b200/csrc/*.cu`` is compiled by nvcc for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/obj`` and linked
into one shared library with the CUDA runtime linked statically.  The
library is built in-tree so that it travels with the repository snapshot.

Run ``python -m leap_b200.build`` (or ``__graft_entry__.build()``).  With
``--clean`` every object and the library are rebuilt from source, so a source
that no longer compiles cannot hide behind an object left from an earlier
build.  ``__graft_entry__.build()`` always builds clean.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(ROOT, "_build", "obj")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libleap_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC,
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand) and not shutil.which(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, extra: list[str], objdir: str = OBJ, force: bool = False) -> str:
    obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
    if force or _stale(obj, [src] + _headers()):
        cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def clean() -> None:
    """Remove the object directory and the linked library."""
    shutil.rmtree(OBJ, ignore_errors=True)
    if os.path.exists(LIB):
        os.remove(LIB)


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _link(objs: list[str], lib: str) -> None:
    cmd = [nvcc(), *ARCH, "-shared", "-o", lib, *objs, "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")


def build_into(objdir: str, lib: str, extra: list[str] | None = None) -> str:
    """Compile every source from scratch into ``objdir`` and link ``lib``.

    Reuses nothing, so it shows whether the current sources build."""
    os.makedirs(objdir, exist_ok=True)
    extra = list(extra or [])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra, objdir, True), sources()))
    _link(objs, lib)
    return lib


def build(verbose: bool = False, extra: list[str] | None = None, fresh: bool = False) -> str:
    """Compile every CUDA source for sm_100a and link the shared library.

    ``fresh`` discards earlier objects first (see :func:`clean`)."""
    if fresh:
        clean()
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    extra = list(extra or [])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), sources()))
    if _stale(LIB, objs):
        _link(objs, LIB)
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    args = sys.argv[1:]
    fresh = "--clean" in args
    build(verbose=True, extra=[a for a in args if a != "--clean"], fresh=fresh)
