"""ctypes binding of the C ABI in ``include/leap_b200.h``.

The shared library ``leap_b200/lib/libleap_b200.so`` is built in-tree by
``leap_b200/build.py`` for sm_100a.  Loading fails loudly when it is missing:
there is no CPU fallback behind this package.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                        "libleap_b200.so")

c_int = ctypes.c_int
c_float_p = ctypes.POINTER(ctypes.c_float)
c_void_p = ctypes.c_void_p
c_int_p = ctypes.POINTER(ctypes.c_int)

LEAP_OK = 0
LEAP_ERR_INVALID = 1
LEAP_ERR_CUDA = 2
LEAP_ERR_DEVICE = 3
LEAP_ERR_NOMEM = 4
LEAP_ERR_COMM = 5


class CtxDesc(ctypes.Structure):
    """``leap_ctx_desc`` (include/leap_b200.h)."""
    _fields_ = [
        ("n_layers", c_int),
        ("layer0", c_int),
        ("n_heads", c_int),
        ("n_kv_heads", c_int),
        ("head_dim", c_int),
        ("max_seq", c_int),
        ("max_batch", c_int),
        ("device", c_int),
        ("rope_cos", c_float_p),
        ("rope_sin", c_float_p),
    ]


class ModelConfigC(ctypes.Structure):
    """``leap_model_config`` (include/leap_b200.h)."""
    _fields_ = [(n, c_int) for n in ("dim", "hidden_dim", "n_layers", "n_heads", "n_kv_heads",
                                     "vocab_size", "seq_len", "quantized", "group_size",
                                     "shared_classifier")]


# name -> (restype, argtypes); every symbol include/leap_b200.h declares
SIGNATURES: dict[str, tuple] = {
    "leap_last_error": (ctypes.c_char_p, []),
    "leap_version": (ctypes.c_char_p, []),
    "leap_rope_table": (c_int, [c_int, c_int, ctypes.c_float, c_float_p, c_float_p]),
    "leap_ctx_create": (c_int, [ctypes.POINTER(CtxDesc), ctypes.POINTER(c_void_p)]),
    "leap_ctx_destroy": (c_int, [c_void_p]),
    "leap_ctx_set_stream": (c_int, [c_void_p, c_void_p]),
    "leap_ctx_use_own_stream": (c_int, [c_void_p]),
    "leap_set_overlap": (c_int, [c_void_p, c_int]),
    "leap_set_decode_impl": (c_int, [c_void_p, c_int]),
    "leap_decode_cluster_capacity": (c_int, [c_void_p, c_int_p]),
    "leap_sync": (c_int, [c_void_p]),
    "leap_ctx_device_bytes": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_size_t)]),
    "leap_kv_clear": (c_int, [c_void_p]),
    "leap_kv_write": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                              c_int]),
    "leap_kv_read": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                             c_int]),
    "leap_attn_decode": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p,
                                 c_void_p]),
    "leap_attn_decode_host": (c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p,
                                      c_void_p, c_void_p]),
    "leap_attn_decode_batched": (c_int, [c_void_p, c_int, c_int, c_int_p, c_int_p,
                                         c_void_p, c_void_p, c_void_p, c_void_p]),
    "leap_attn_prefill": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                  c_void_p, c_void_p, c_void_p]),
    "leap_set_prefill_impl": (c_int, [c_void_p, c_int]),
    "leap_attn_decode_noalloc": (c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p,
                                         c_void_p, c_void_p, c_void_p, ctypes.c_longlong,
                                         c_void_p, c_void_p, c_void_p, c_void_p]),
    "leap_engine_open": (c_int, [ctypes.c_char_p, c_int, c_int, c_int, ctypes.c_float, c_int,
                                 ctypes.POINTER(c_void_p)]),
    "leap_engine_synthetic": (c_int, [ctypes.POINTER(ModelConfigC), ctypes.c_ulonglong, c_int,
                                      c_int, c_int, ctypes.c_float, c_int,
                                      ctypes.POINTER(c_void_p)]),
    "leap_engine_destroy": (c_int, [c_void_p]),
    "leap_engine_config": (c_int, [c_void_p, ctypes.POINTER(ModelConfigC), c_int_p, c_int_p]),
    "leap_engine_device_bytes": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_size_t)]),
    "leap_engine_set_stream": (c_int, [c_void_p, c_void_p]),
    "leap_engine_sync": (c_int, [c_void_p]),
    "leap_engine_clear_kv": (c_int, [c_void_p]),
    "leap_engine_embed": (c_int, [c_void_p, c_int_p, c_int, c_void_p]),
    "leap_engine_embed_device": (c_int, [c_void_p, c_void_p, c_int, c_void_p]),
    "leap_engine_layers": (c_int, [c_void_p, c_int, c_int, c_void_p]),
    "leap_engine_head": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "leap_engine_forward": (c_int, [c_void_p, c_int, c_int, c_float_p, c_int_p]),
    "leap_engine_prefill": (c_int, [c_void_p, c_int_p, c_int, c_int, c_int_p]),
    "leap_op_rmsnorm": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int]),
    "leap_op_rmsnorm_quantize": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                         c_int]),
    "leap_op_quantize": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, ctypes.c_longlong,
                                 c_int]),
    "leap_op_matmul": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int,
                               c_void_p]),
    "leap_op_qmatmul": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                c_int, c_int, c_int, c_int, c_void_p]),
    "leap_op_matmul_fused": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int,
                                     c_int, c_void_p]),
    "leap_op_qmatmul_fused": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                      c_int, c_int, c_void_p]),
    "leap_op_argmax": (c_int, [c_void_p, c_void_p, c_void_p, c_int]),
    "leap_sampler_create": (c_int, [c_int, ctypes.c_float, ctypes.c_float, ctypes.c_ulonglong, c_int,
                                    ctypes.POINTER(c_void_p)]),
    "leap_sampler_destroy": (c_int, [c_void_p]),
    "leap_sampler_sample": (c_int, [c_void_p, c_void_p, c_void_p, c_void_p]),
    "leap_sampler_state": (c_int, [c_void_p, ctypes.POINTER(ctypes.c_ulonglong)]),
    "leap_engine_set_sampler": (c_int, [c_void_p, c_void_p]),
    "leap_pp_unique_id": (c_int, [c_void_p]),
    "leap_pp_init": (c_int, [c_void_p, c_int, c_int, c_int, c_int, ctypes.POINTER(c_void_p)]),
    "leap_pp_send_next": (c_int, [c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "leap_pp_recv_prev": (c_int, [c_void_p, c_void_p, ctypes.c_size_t, c_void_p]),
    "leap_pp_send": (c_int, [c_void_p, c_int, c_void_p, ctypes.c_size_t, c_void_p]),
    "leap_pp_recv": (c_int, [c_void_p, c_int, c_void_p, ctypes.c_size_t, c_void_p]),
    "leap_pp_abort": (c_int, [c_void_p]),
    "leap_pp_destroy": (c_int, [c_void_p]),
    "leap_op_set_q8_gemv": (c_int, [c_int]),
    "leap_op_set_q8_gemm": (c_int, [c_int]),
}

_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


class LeapError(RuntimeError):
    """A non-zero status from the C ABI (the reference raises
    std::runtime_error for the same conditions)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[leap status {status}] {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m leap_b200.build` "
                    "(nvcc, sm_100a). There is no CPU fallback.")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
        return _lib


def check(status: int) -> None:
    if status != LEAP_OK:
        msg = lib().leap_last_error().decode(errors="replace")
        raise LeapError(status, msg)
