"""The CUDA sources build from scratch (no GPU needed: nvcc cross-compiles
sm_100a on the host).

Every ``leap_b200/csrc/*.cu`` is compiled with the library's own flags into a
fresh temporary directory, nothing reused from an earlier build, and linked
into a shared library that must load and export every symbol the public
header declares.  So the CPU suite fails as soon as any source stops
compiling, whatever objects or library an earlier build left in the tree.
"""
import ctypes
import os
import re
import shutil
import tempfile

import pytest

from leap_b200 import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="nvcc is not installed")
def test_every_source_compiles_and_links_from_scratch():
    tmp = tempfile.mkdtemp(prefix="leap_build_")
    try:
        lib = build.build_into(os.path.join(tmp, "obj"), os.path.join(tmp, "libcheck.so"))
        objs = os.listdir(os.path.join(tmp, "obj"))
        assert len(objs) == len(build.sources())
        handle = ctypes.CDLL(lib)
        hdr = open(os.path.join(ROOT, "include", "leap_b200.h")).read()
        names = set(re.findall(r"LEAP_API\s+[\w\s\*]*?\b(leap_\w+)\s*\(", hdr))
        assert names
        for n in sorted(names):
            assert hasattr(handle, n), f"{n} declared but not exported by a fresh build"
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
