"""CPU checkers for the LEAP attention hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs import this package.  The product path (``leap_b200``) never does and
has no CPU fallback.

Two checkers, both loaded with ctypes:

* ``port``  — ``oracle/leap_oracle.c``, a plain-C restatement of the
  reference arithmetic (each function cites the reference file:line it
  follows).  Built by ``make -C oracle port`` (gcc only), so it also builds on
  the GPU box.
* ``ref``   — the reference's OWN code compiled from its sources by
  ``make -C oracle ref``: the attention block / softmax / RoPE-table line
  ranges of ``src/inference/FloatTransformer.cpp`` and
  ``QuantizedTransformer.cpp`` (``libleapref_attn.so``) and the unmodified
  engine behind ``Transformer::create``/``forward``
  (``libleapref_engine*.so``).  Needs the reference sources, so it is built in
  the development container and shipped prebuilt in ``oracle/_ref/``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_ATTN_SO = os.path.join(HERE, "_ref", "libleapref_attn.so")
REF_ENGINE_SO = os.path.join(HERE, "_ref", "libleapref_engine.so")
REF_ENGINE_10K_SO = os.path.join(HERE, "_ref", "libleapref_engine_10k.so")
# the reference engine with its attention block calling libleap_b200.so
REF_ENGINE_GPUATTN_SO = os.path.join(HERE, "_ref", "libleapref_engine_gpuattn.so")

_lock = threading.Lock()
_libs: dict[str, ctypes.CDLL] = {}

_f = ctypes.POINTER(ctypes.c_float)
_i8 = ctypes.POINTER(ctypes.c_int8)
_int = ctypes.c_int


def build_port() -> str:
    """Compile the C restatement if it is missing or stale."""
    src = os.path.join(HERE, "leap_oracle.c")
    if (not os.path.exists(PORT_SO)
            or os.path.getmtime(PORT_SO) < os.path.getmtime(src)):
        subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
    return PORT_SO


def reference_root() -> str | None:
    """Where the reference sources are: ``$LEAP_REFERENCE`` if set, else the
    ``reference_path`` recorded in the repository's ``BASELINE.json``.  None
    when neither names a directory holding ``src/inference``."""
    ref = os.environ.get("LEAP_REFERENCE")
    if not ref:
        try:
            import json
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as fh:
                ref = json.load(fh).get("reference_path")
        except (OSError, ValueError):
            ref = None
    if ref and os.path.isdir(os.path.join(ref, "src", "inference")):
        return ref
    return None


def build_ref() -> bool:
    """Compile the reference's own code (needs the reference sources)."""
    ref = reference_root()
    if ref is None:
        return False
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)
    return True


def build_binding() -> bool:
    """Compile the reference engine bound to the C ABI (needs the reference
    sources and the built libleap_b200.so)."""
    ref = reference_root()
    if ref is None:
        return False
    subprocess.run(["make", "-s", "-C", HERE, "binding", f"REF={ref}"], check=True)
    return True


def has_ref_binding() -> bool:
    return os.path.exists(REF_ENGINE_GPUATTN_SO)


def _load(path: str) -> ctypes.CDLL:
    with _lock:
        lib = _libs.get(path)
        if lib is None:
            lib = ctypes.CDLL(path)
            _libs[path] = lib
        return lib


def port() -> ctypes.CDLL:
    lib = _load(build_port())
    lib.orc_rope_table.argtypes = [_int, _int, ctypes.c_float, _f, _f]
    lib.orc_attn_block.argtypes = [_int, _int, _int, _int, _int, _f, _f, _f,
                                   _f, _f, _f, _f, _int]
    lib.orc_attn_prefill.argtypes = [_int, _int, _int, _int, _int, _int, _f,
                                     _f, _f, _f, _f, _f, _f, _f, _int]
    lib.orc_rmsnorm.argtypes = [_f, _f, _f, _int]
    lib.orc_matmul.argtypes = [_f, _f, _f, _int, _int, _int]
    lib.orc_quantize.argtypes = [_i8, _f, _f, _int, _int]
    lib.orc_qmatmul.argtypes = [_f, _i8, _f, _i8, _f, _int, _int, _int, _int]
    lib.orc_softmax.argtypes = [_f, _int]
    return lib


def has_ref() -> bool:
    return os.path.exists(REF_ATTN_SO)


def ref_attn() -> ctypes.CDLL:
    if not os.path.exists(REF_ATTN_SO):
        raise FileNotFoundError(
            f"{REF_ATTN_SO} missing: run `make -C oracle ref` where the "
            "reference sources are available")
    lib = _load(REF_ATTN_SO)
    lib.leapref_attn_block.argtypes = [_int] * 6 + [_f] * 7
    lib.leapref_rope_table.argtypes = [_int, _int, _int, _int, _f, _f]
    return lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    if a.dtype == np.float32:
        return a.ctypes.data_as(_f)
    if a.dtype == np.int8:
        return a.ctypes.data_as(_i8)
    raise TypeError(a.dtype)


# --------------------------------------------------------------------------
# numpy-level helpers (all arrays float32, C-contiguous)
# --------------------------------------------------------------------------

def rope_table(seq_len: int, head_size: int, theta: float = 500000.0,
               impl: str = "port"):
    """[seq_len, head_size/2] cos and sin tables (FloatTransformer.cpp:56-72)."""
    c = np.empty((seq_len, head_size // 2), np.float32)
    s = np.empty_like(c)
    if impl == "port":
        port().orc_rope_table(seq_len, head_size, theta, _p(c), _p(s))
    else:
        if theta not in (500000.0, 10000.0):
            raise ValueError("the reference code only exists for 500000/10000")
        n_heads = 1
        ref_attn().leapref_rope_table(int(theta == 10000.0), head_size,
                                      n_heads, seq_len, _p(c), _p(s))
    return c, s


def attn_block(q, k_cache, v_cache, pos, n_heads, n_kv_heads, head_size,
               rope_cos, rope_sin, impl: str = "port", threads: int = 1,
               which: int = 0):
    """Run one reference attention block.

    q [n_heads*hs]; k_cache/v_cache [seq_len, kv_dim] for ONE layer with the
    new un-rotated k/v already in row ``pos``.  Arrays are modified in place
    like the reference (q and k row ``pos`` get rotated).  Returns xb.
    """
    seq_len = k_cache.shape[0]
    att = np.empty(n_heads * seq_len, np.float32)
    xb = np.empty(n_heads * head_size, np.float32)
    if impl == "port":
        port().orc_attn_block(n_heads, n_kv_heads, head_size, seq_len, pos,
                              _p(rope_cos), _p(rope_sin), _p(q), _p(k_cache),
                              _p(v_cache), _p(att), _p(xb), threads)
    else:
        ref_attn().leapref_attn_block(which, n_heads, n_kv_heads, head_size,
                                      seq_len, pos, _p(rope_cos),
                                      _p(rope_sin), _p(q), _p(k_cache),
                                      _p(v_cache), _p(att), _p(xb))
    return xb


def decode_case(q, k_new, v_new, k_rows, v_rows, pos, n_heads, n_kv_heads,
                head_size, rope_cos, rope_sin, impl="port", threads=1,
                which=0):
    """Decode attention for one token given the cache rows [0, pos).

    q [n_heads, hs], k_new/v_new [n_kv, hs] un-rotated; k_rows/v_rows
    [pos, n_kv, hs] (already rotated, as the cache holds them).  Returns
    (out [n_heads, hs], rotated k row [n_kv, hs]).  Inputs are not modified.
    """
    kv_dim = n_kv_heads * head_size
    seq_len = pos + 1
    kc = np.zeros((seq_len, kv_dim), np.float32)
    vc = np.zeros((seq_len, kv_dim), np.float32)
    kc[:pos] = k_rows.reshape(pos, kv_dim)
    vc[:pos] = v_rows.reshape(pos, kv_dim)
    kc[pos] = k_new.reshape(kv_dim)
    vc[pos] = v_new.reshape(kv_dim)
    qq = np.ascontiguousarray(q.reshape(-1), dtype=np.float32).copy()
    out = attn_block(qq, kc, vc, pos, n_heads, n_kv_heads, head_size,
                     rope_cos, rope_sin, impl=impl, threads=threads,
                     which=which)
    return out.reshape(n_heads, head_size), kc[pos].reshape(n_kv_heads,
                                                           head_size)


def prefill(q, k, v, k_rows, v_rows, pos0, n_heads, n_kv_heads, head_size,
            rope_cos, rope_sin, threads=1):
    """Causal prefill via the C restatement (block per position in order).

    q [n_tok, n_heads, hs]; k/v [n_tok, n_kv, hs] un-rotated; k_rows/v_rows
    [pos0, n_kv, hs] existing cache rows.  Returns (out, k_cache, v_cache)
    with the caches [pos0+n_tok, n_kv, hs] as the reference leaves them.
    """
    n_tok = q.shape[0]
    kv_dim = n_kv_heads * head_size
    seq_len = pos0 + n_tok
    kc = np.zeros((seq_len, kv_dim), np.float32)
    vc = np.zeros((seq_len, kv_dim), np.float32)
    if pos0:
        kc[:pos0] = k_rows.reshape(pos0, kv_dim)
        vc[:pos0] = v_rows.reshape(pos0, kv_dim)
    qa = np.ascontiguousarray(q, dtype=np.float32)
    ka = np.ascontiguousarray(k, dtype=np.float32)
    va = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty((n_tok, n_heads, head_size), np.float32)
    port().orc_attn_prefill(n_heads, n_kv_heads, head_size, seq_len, pos0,
                            n_tok, _p(rope_cos), _p(rope_sin), _p(qa), _p(ka),
                            _p(va), _p(kc), _p(vc), _p(out), threads)
    return (out, kc.reshape(seq_len, n_kv_heads, head_size),
            vc.reshape(seq_len, n_kv_heads, head_size))


# --------------------------------------------------------------------------
# The unmodified reference engine (Transformer::create / forward), compiled
# from its sources into oracle/_ref (ref_engine_glue.cpp).
# --------------------------------------------------------------------------

class RefEngine:
    """The reference engine on a .bin file: forward(token, pos) -> logits.

    theta_10k selects the copy built with the RoPE literal set to 10000
    (TinyLlama); the shipped reference hard-codes 500000.  gpu_attention
    selects the reference engine built with its attention block bound to
    libleap_b200.so (oracle/ref_binding_attn.cpp; theta 500000)."""

    def __init__(self, path: str, theta_10k: bool = False, gpu_attention: bool = False):
        if gpu_attention:
            # the reference engine whose attention block calls libleap_b200.so
            so = REF_ENGINE_GPUATTN_SO
        else:
            so = REF_ENGINE_10K_SO if theta_10k else REF_ENGINE_SO
        if not os.path.exists(so):
            raise FileNotFoundError(f"{so} missing: run `make -C oracle ref`")
        lib = _load(so)
        lib.leapref_engine_create.restype = ctypes.c_void_p
        lib.leapref_engine_create.argtypes = [ctypes.c_char_p]
        lib.leapref_engine_forward.restype = _f
        lib.leapref_engine_forward.argtypes = [ctypes.c_void_p, _int, _int]
        lib.leapref_engine_config.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
        lib.leapref_engine_clear.argtypes = [ctypes.c_void_p]
        lib.leapref_engine_destroy.argtypes = [ctypes.c_void_p]
        lib.leapref_engine_error.restype = ctypes.c_char_p
        lib.leapref_sample_argmax.argtypes = [_f, _int]
        self.lib = lib
        self.h = lib.leapref_engine_create(path.encode())
        if not self.h:
            raise RuntimeError(lib.leapref_engine_error().decode())
        cfg = (ctypes.c_int * 7)()
        lib.leapref_engine_config(self.h, cfg)
        self.config = tuple(cfg)

    def forward(self, token: int, pos: int) -> np.ndarray:
        p = self.lib.leapref_engine_forward(self.h, token, pos)
        if not p:
            raise RuntimeError(self.lib.leapref_engine_error().decode())
        return np.ctypeslib.as_array(p, shape=(self.config[5],)).copy()

    def argmax(self, logits: np.ndarray) -> int:
        a = np.ascontiguousarray(logits, np.float32)
        return int(self.lib.leapref_sample_argmax(_p(a), int(a.size)))

    def clear(self):
        self.lib.leapref_engine_clear(self.h)

    def close(self):
        if self.h:
            self.lib.leapref_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ref_argmax(v) -> int:
    """Greedy token through the reference Sampler (temperature 0)."""
    a = np.ascontiguousarray(v, np.float32)
    lib = _load(REF_ENGINE_SO)
    lib.leapref_sample_argmax.argtypes = [_f, _int]
    return int(lib.leapref_sample_argmax(_p(a), int(a.size)))


def ref_sample(logits, temperature: float, topp: float, state: int) -> int:
    """One draw of the reference Sampler (src/inference/Sampler.cpp:187-232)
    with its RNG state starting at `state` (advance it with random_f32)."""
    a = np.ascontiguousarray(logits, np.float32)
    lib = _load(REF_ENGINE_SO)
    lib.leapref_sample.argtypes = [_f, _int, ctypes.c_float, ctypes.c_float, ctypes.c_ulonglong]
    return int(lib.leapref_sample(_p(a), int(a.size), float(temperature), float(topp), int(state)))


def random_u32(state: int):
    """The reference's xorshift* step (src/inference/Utils.h:18-24):
    returns (value, new state)."""
    m = (1 << 64) - 1
    state ^= state >> 12
    state = (state ^ (state << 25)) & m
    state ^= state >> 27
    return ((state * 0x2545F4914F6CDD1D) & m) >> 32, state


def random_f32(state: int):
    """A float in [0, 1) (src/inference/Utils.h:26-29): (value, new state)."""
    u, state = random_u32(state)
    return float(np.float32(u >> 8) / np.float32(16777216.0)), state


def has_ref_engine() -> bool:
    return os.path.exists(REF_ENGINE_SO) and os.path.exists(REF_ENGINE_10K_SO)


# --------------------------------------------------------------------------
# Support ops of the layer (end-to-end configs): port and reference
# --------------------------------------------------------------------------

def ref_support() -> ctypes.CDLL:
    lib = ref_attn()
    lib.leapref_rmsnorm.argtypes = [_f, _f, _f, _int]
    lib.leapref_matmul.argtypes = [_f, _f, _f, _int, _int]
    lib.leapref_quantize.argtypes = [_int, _i8, _f, _f, _int]
    lib.leapref_dequantize.argtypes = [_int, _f, _i8, _f, _int]
    lib.leapref_qmatmul.argtypes = [_int, _f, _i8, _f, _i8, _f, _int, _int]
    return lib


def rmsnorm(x, w, impl: str = "port"):
    """FloatTransformer.cpp:79-214 on one row."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    o = np.empty_like(x)
    if impl == "port":
        port().orc_rmsnorm(_p(o), _p(x), _p(w), int(x.size))
    else:
        ref_support().leapref_rmsnorm(_p(o), _p(x), _p(w), int(x.size))
    return o


def matmul(x, w, impl: str = "port", threads: int = 1):
    """y[d] = W[d][n] . x (FloatTransformer.cpp:240-382)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    d, n = w.shape
    y = np.empty(d, np.float32)
    if impl == "port":
        port().orc_matmul(_p(y), _p(x), _p(w), n, d, threads)
    else:
        ref_support().leapref_matmul(_p(y), _p(x), _p(w), n, d)
    return y


def quantize(x, gs: int = 64, impl: str = "port"):
    """(q int8[n], s float32[n/gs]) — QuantizedTransformer.cpp:338-357."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q = np.empty(x.size, np.int8)
    s = np.empty(x.size // gs, np.float32)
    if impl == "port":
        port().orc_quantize(_p(q), _p(s), _p(x), int(x.size), gs)
    else:
        ref_support().leapref_quantize(gs, _p(q), _p(s), _p(x), int(x.size))
    return q, s


def qmatmul(xq, xs, wq, ws, gs: int = 64, impl: str = "port", threads: int = 1):
    """W8A8 GEMV y[d] (QuantizedTransformer.cpp:359-652); wq [d][n]."""
    xq = np.ascontiguousarray(xq, np.int8)
    xs = np.ascontiguousarray(xs, np.float32)
    wq = np.ascontiguousarray(wq, np.int8)
    ws = np.ascontiguousarray(ws, np.float32)
    d, n = wq.shape
    y = np.empty(d, np.float32)
    if impl == "port":
        port().orc_qmatmul(_p(y), _p(xq), _p(xs), _p(wq), _p(ws), n, d, gs, threads)
    else:
        ref_support().leapref_qmatmul(gs, _p(y), _p(xq), _p(xs), _p(wq), _p(ws), n, d)
    return y
