"""Host-side wrapper of the attention C ABI.

``AttentionContext`` owns one ``leap_ctx``: the device KV cache of a range of
layers (and of ``max_batch`` sequence slots), the RoPE table, and the split-KV
scratch.  Its methods mirror what the reference's ``run_layer`` does around
attention (src/inference/FloatTransformer.cpp:384-662) and what its
``clear_kv_cache`` does (:74-77).

Device tensors are ``torch.Tensor`` on the context's GPU (torch is used only
for device memory and streams); host arrays are ``numpy.ndarray``.  Errors
raise :class:`LeapError`, the way the reference raises std::runtime_error.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._native import CtxDesc, LeapError, check, lib

__all__ = ["AttentionContext", "LeapError", "rope_table"]


def rope_table(seq_len: int, head_dim: int, theta: float = 500000.0):
    """Reference RoPE table ``[seq_len, head_dim/2]`` (cos, sin), computed by
    the library exactly as the compiled reference does
    (src/inference/FloatTransformer.cpp:56-72)."""
    c = np.empty((seq_len, head_dim // 2), np.float32)
    s = np.empty_like(c)
    fp = ctypes.POINTER(ctypes.c_float)
    check(lib().leap_rope_table(seq_len, head_dim, ctypes.c_float(theta),
                                c.ctypes.data_as(fp), s.ctypes.data_as(fp)))
    return c, s


def _dptr(t) -> int:
    """Device pointer of a contiguous float32 CUDA tensor."""
    import torch
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("expected a CUDA torch.Tensor")
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise TypeError("expected a contiguous float32 tensor")
    return t.data_ptr()


def _hptr(a: np.ndarray) -> int:
    if a.dtype != np.float32 or not a.flags["C_CONTIGUOUS"]:
        raise TypeError("expected a C-contiguous float32 array")
    return a.ctypes.data


class AttentionContext:
    """Device attention state for ``n_layers`` layers and ``max_batch`` slots.

    Parameters follow the reference ``Config`` (src/inference/Config.h):
    ``n_heads``, ``n_kv_heads``, ``head_dim`` (= dim / n_heads), ``max_seq``
    (= seq_len).  ``rope_cos``/``rope_sin`` default to :func:`rope_table`
    with ``theta``.
    """

    def __init__(self, n_layers: int, n_heads: int, n_kv_heads: int, head_dim: int,
                 max_seq: int, max_batch: int = 1, device: int = 0, layer0: int = 0,
                 theta: float = 500000.0, rope_cos=None, rope_sin=None,
                 bind_torch_stream: bool = True):
        if rope_cos is None or rope_sin is None:
            rope_cos, rope_sin = rope_table(max_seq, head_dim, theta)
        self.rope_cos = np.ascontiguousarray(rope_cos, np.float32)
        self.rope_sin = np.ascontiguousarray(rope_sin, np.float32)
        if self.rope_cos.shape != (max_seq, head_dim // 2):
            raise ValueError("rope tables must be [max_seq, head_dim/2]")
        fp = ctypes.POINTER(ctypes.c_float)
        desc = CtxDesc(n_layers, layer0, n_heads, n_kv_heads, head_dim, max_seq,
                       max_batch, device, self.rope_cos.ctypes.data_as(fp),
                       self.rope_sin.ctypes.data_as(fp))
        h = ctypes.c_void_p()
        check(lib().leap_ctx_create(ctypes.byref(desc), ctypes.byref(h)))
        self._h = h
        self.n_layers, self.n_heads, self.n_kv_heads = n_layers, n_heads, n_kv_heads
        self.head_dim, self.max_seq, self.max_batch = head_dim, max_seq, max_batch
        self.device = device
        if bind_torch_stream:
            self.bind_torch_stream()

    # -- lifetime ---------------------------------------------------------
    def close(self) -> None:
        if getattr(self, "_h", None):
            check(lib().leap_ctx_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise LeapError(1, "context is closed")
        return self._h

    # -- streams ----------------------------------------------------------
    def bind_torch_stream(self, stream=None) -> None:
        """Order this context's work on a torch CUDA stream (default: the
        current stream of its device), so torch tensors can be passed
        without extra synchronisation."""
        import torch
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        check(lib().leap_ctx_set_stream(self.handle, ctypes.c_void_p(stream.cuda_stream)))

    def use_own_stream(self) -> None:
        check(lib().leap_ctx_use_own_stream(self.handle))

    def sync(self) -> None:
        check(lib().leap_sync(self.handle))

    def device_bytes(self) -> int:
        n = ctypes.c_size_t()
        check(lib().leap_ctx_device_bytes(self.handle, ctypes.byref(n)))
        return n.value

    # -- cache ------------------------------------------------------------
    def clear_kv_cache(self) -> None:
        """FloatTransformer::clear_kv_cache (FloatTransformer.cpp:74-77)."""
        check(lib().leap_kv_clear(self.handle))

    def kv_write(self, slot: int, layer: int, pos0: int, k, v) -> None:
        """Write rows [pos0, pos0+n) from reference layout [n, n_kv, hd]."""
        if isinstance(k, np.ndarray):
            k = np.ascontiguousarray(k, np.float32)
            v = np.ascontiguousarray(v, np.float32)
            n = k.shape[0]
            check(lib().leap_kv_write(self.handle, slot, layer, pos0, n, _hptr(k),
                                      _hptr(v), 1))
        else:
            n = k.shape[0]
            check(lib().leap_kv_write(self.handle, slot, layer, pos0, n, _dptr(k),
                                      _dptr(v), 0))

    def kv_read(self, slot: int, layer: int, pos0: int, n: int):
        """Rows [pos0, pos0+n) as host arrays [n, n_kv, hd] (K, V)."""
        k = np.empty((n, self.n_kv_heads, self.head_dim), np.float32)
        v = np.empty_like(k)
        check(lib().leap_kv_read(self.handle, slot, layer, pos0, n, _hptr(k), _hptr(v), 1))
        return k, v

    # -- attention ----------------------------------------------------------
    def decode(self, layer: int, pos: int, q, k_new, v_new, out=None):
        """Fused RoPE + append + attention for one token (device tensors)."""
        import torch
        if out is None:
            out = torch.empty_like(q)
        check(lib().leap_attn_decode(self.handle, layer, pos, _dptr(q), _dptr(k_new),
                                     _dptr(v_new), _dptr(out)))
        return out

    def decode_host(self, layer: int, pos: int, q: np.ndarray, k_new: np.ndarray,
                    v_new: np.ndarray) -> np.ndarray:
        """Same as :meth:`decode` on host arrays; blocks until done."""
        q = np.ascontiguousarray(q, np.float32)
        k_new = np.ascontiguousarray(k_new, np.float32)
        v_new = np.ascontiguousarray(v_new, np.float32)
        out = np.empty((self.n_heads, self.head_dim), np.float32)
        check(lib().leap_attn_decode_host(self.handle, layer, pos, _hptr(q), _hptr(k_new),
                                          _hptr(v_new), _hptr(out)))
        return out

    def decode_batched(self, layer: int, slots, positions, q, k_new, v_new, out=None):
        """Ragged batch: token i of slot slots[i] at positions[i]."""
        import torch
        slots = np.ascontiguousarray(slots, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        if slots.shape != positions.shape or slots.ndim != 1:
            raise ValueError("slots and positions must be equal-length 1-D")
        if out is None:
            out = torch.empty_like(q)
        ip = ctypes.POINTER(ctypes.c_int)
        check(lib().leap_attn_decode_batched(
            self.handle, layer, int(slots.shape[0]), slots.ctypes.data_as(ip),
            positions.ctypes.data_as(ip), _dptr(q), _dptr(k_new), _dptr(v_new),
            _dptr(out)))
        return out

    def prefill(self, slot: int, layer: int, pos0: int, q, k, v, out=None):
        """Causal prefill of q.shape[0] tokens starting at pos0."""
        import torch
        if out is None:
            out = torch.empty_like(q)
        check(lib().leap_attn_prefill(self.handle, slot, layer, pos0, int(q.shape[0]),
                                      _dptr(q), _dptr(k), _dptr(v), _dptr(out)))
        return out

    def set_decode_impl(self, impl: int) -> None:
        """0 = auto, 1 = split-KV, 2 = cluster kernel, 3 = wide split-KV,
        4 = split-KV with a separate combine launch."""
        check(lib().leap_set_decode_impl(self.handle, impl))

    def cluster_capacity(self) -> int:
        n = ctypes.c_int()
        check(lib().leap_decode_cluster_capacity(self.handle, ctypes.byref(n)))
        return n.value

    def set_overlap(self, enable: bool) -> None:
        """Let a decode launch stream its K/V while the previous kernel
        finishes (programmatic dependent launch); on by default."""
        check(lib().leap_set_overlap(self.handle, int(bool(enable))))

    def set_prefill_impl(self, impl: int) -> None:
        """0 = tensor-core 3xTF32 kernel pipelined across warp roles,
        1 = CUDA-core FP32 kernel, 2 = tensor-core 3xTF32 kernel, one tile at
        a time, 3 = the pipelined kernel with its two correction products in
        BF16 (the default)."""
        check(lib().leap_set_prefill_impl(self.handle, impl))
