"""The C ABI library: loads, exports what include/leap_b200.h declares,
validates arguments, and fails cleanly without a GPU.  No GPU compute."""
import ctypes
import hashlib
import os
import re

import numpy as np
import pytest

from leap_b200 import _native
from leap_b200.attention import rope_table

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    txt = open(os.path.join(ROOT, "include", "leap_b200.h")).read()
    return sorted(set(re.findall(r"LEAP_API\s+[\w\s\*]*?\b(leap_\w+)\s*\(", txt)))


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    decl = declared_symbols()
    assert len(decl) >= 16
    for name in decl:
        assert hasattr(lib, name), f"{name} declared but not exported"
    assert set(decl) == set(_native.SIGNATURES), "bindings out of sync with the header"


def test_built_for_sm100a_only():
    """The library is compiled for sm_100a (checked through the build recipe,
    not by reading the binary)."""
    from leap_b200 import build
    assert build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_version():
    assert b"sm_100a" in _native.lib().leap_version()


def test_rope_table_is_the_reference_table(golden):
    _, man = golden
    for r in man["rope"]:
        c, s = rope_table(r["seq_len"], r["head_dim"], r["theta"])
        assert hashlib.sha256(c.tobytes() + s.tobytes()).hexdigest() == r["sha256"]


def test_invalid_desc_is_rejected():
    lib = _native.lib()
    c, s = rope_table(16, 64)
    fp = ctypes.POINTER(ctypes.c_float)
    h = ctypes.c_void_p()
    # n_heads not a multiple of n_kv_heads
    d = _native.CtxDesc(1, 0, 6, 4, 64, 16, 1, 0, c.ctypes.data_as(fp), s.ctypes.data_as(fp))
    assert lib.leap_ctx_create(ctypes.byref(d), ctypes.byref(h)) == _native.LEAP_ERR_INVALID
    assert b"invalid shape" in lib.leap_last_error()
    # unsupported head_dim
    d = _native.CtxDesc(1, 0, 8, 8, 96, 16, 1, 0, c.ctypes.data_as(fp), s.ctypes.data_as(fp))
    assert lib.leap_ctx_create(ctypes.byref(d), ctypes.byref(h)) == _native.LEAP_ERR_INVALID
    # missing rope table
    d = _native.CtxDesc(1, 0, 8, 8, 64, 16, 1, 0, None, None)
    assert lib.leap_ctx_create(ctypes.byref(d), ctypes.byref(h)) == _native.LEAP_ERR_INVALID
    assert not h.value


def test_null_context_is_an_error():
    lib = _native.lib()
    assert lib.leap_sync(None) == _native.LEAP_ERR_INVALID
    assert lib.leap_attn_decode(None, 0, 0, None, None, None, None) == _native.LEAP_ERR_INVALID
    with pytest.raises(_native.LeapError):
        _native.check(lib.leap_kv_clear(None))


def test_kernel_selectors_validate_their_argument():
    """The process-wide W8A8 kernel selectors take only the kernels they
    name, and report the choices in the message; valid choices need no GPU."""
    lib = _native.lib()
    assert lib.leap_op_set_q8_gemm(2) == _native.LEAP_ERR_INVALID
    assert b"kind::i8" in lib.leap_last_error()
    assert lib.leap_op_set_q8_gemv(3) == _native.LEAP_ERR_INVALID
    assert lib.leap_op_set_q8_gemm(0) == _native.LEAP_OK
    assert lib.leap_op_set_q8_gemm(1) == _native.LEAP_OK  # the library default
    assert lib.leap_op_set_q8_gemv(2) == _native.LEAP_OK  # the library default
    assert lib.leap_set_prefill_impl(None, 3) == _native.LEAP_ERR_INVALID  # needs a context


def test_no_gpu_fails_loudly():
    """Without a GPU the context cannot be created, and says why; there is
    no CPU fallback."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from leap_b200 import AttentionContext, LeapError
    with pytest.raises(LeapError):
        AttentionContext(1, 8, 8, 64, 32, bind_torch_stream=False)


def test_header_compiles_and_links_as_c_and_cpp(tmp_path):
    """An engine's view of the boundary: include/leap_b200.h compiles as C11
    and C++20 and a program calling the entry points links against the
    library (nothing is run)."""
    import shutil
    import subprocess
    prog = r"""
#include "leap_b200.h"
#include <stddef.h>
int use_all(void) {
    leap_ctx *c = NULL; leap_engine *e = NULL; leap_sampler *s = NULL; leap_pp *pp = NULL;
    float q[1] = {0.f}, o[1] = {0.f}; int tok = 0; unsigned long long st = 0;
    int r = leap_attn_decode_host(c, 0, 0, q, q, q, o);
    r |= leap_engine_forward(e, 1, 0, o, &tok);
    r |= leap_sampler_create(32000, 0.8f, 0.9f, 1234ULL, 0, &s);
    r |= leap_sampler_state(s, &st);
    r |= leap_engine_set_sampler(e, s);
    r |= leap_pp_send_next(pp, q, sizeof q, NULL);
    return r;
}
int main(void) { return use_all() == 12345; }
"""
    lib = os.path.join(ROOT, "leap_b200", "lib")
    inc = os.path.join(ROOT, "include")
    for cc, std, ext in (("gcc", "-std=c11", "c"), ("g++", "-std=c++20", "cpp")):
        if not shutil.which(cc):
            pytest.skip(f"{cc} not available")
        src = tmp_path / f"use.{ext}"
        src.write_text(prog)
        out = tmp_path / f"use_{ext}"
        r = subprocess.run([cc, std, "-Wall", "-Werror", f"-I{inc}", str(src), "-o", str(out),
                            f"-L{lib}", "-lleap_b200", f"-Wl,-rpath,{lib}"],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
