"""The transformer engine on B200, with the reference's Transformer API.

``Transformer`` mirrors ``Inference::Transformer``
(src/inference/Transformer.h:48-81): ``create(path)``, ``forward(token, pos,
flags)`` returning logits, ``clear_kv_cache()``; a model's layer range can be
restricted for pipeline stages (the split of Transformer.h:17-23).  Greedy
generation follows ``generate`` in src/inference/main.cpp:64-108 at
temperature 0 (``Sampler::sample`` -> argmax, src/inference/Sampler.cpp:199-202).
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._native import LeapError, ModelConfigC, check, lib
from .modelfile import ModelConfig

FLAG_NO_REPLY = 0    # src/inference/Transformer.h:45
FLAG_NEED_REPLY = 1  # src/inference/Transformer.h:46

__all__ = ["Transformer", "FLAG_NO_REPLY", "FLAG_NEED_REPLY"]

_ip = ctypes.POINTER(ctypes.c_int)
_fp = ctypes.POINTER(ctypes.c_float)


class Transformer:
    """Weights and KV cache of layers [layer_begin, layer_end) on one GPU."""

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle
        c = ModelConfigC()
        lb, le = ctypes.c_int(), ctypes.c_int()
        check(lib().leap_engine_config(handle, ctypes.byref(c), ctypes.byref(lb), ctypes.byref(le)))
        self.config = ModelConfig(c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads,
                                  c.vocab_size, c.seq_len)
        self.quantized = bool(c.quantized)
        self.group_size = c.group_size
        self.shared_classifier = bool(c.shared_classifier)
        self.layer_begin, self.layer_end = lb.value, le.value
        self._logits = np.empty(self.config.vocab_size, np.float32)

    # -- construction ---------------------------------------------------------
    @staticmethod
    def create(checkpoint_path: str, device: int = 0, rope_theta: float = 0.0,
               layer_range=None, max_chunk: int = 512) -> "Transformer":
        """Transformer::create (src/inference/TransformerFactory.cpp:59)."""
        lb, le = layer_range if layer_range is not None else (0, -1)
        h = ctypes.c_void_p()
        check(lib().leap_engine_open(checkpoint_path.encode(), device, lb, le,
                                     ctypes.c_float(rope_theta), max_chunk, ctypes.byref(h)))
        return Transformer(h)

    @staticmethod
    def synthetic(config: ModelConfig, quantized: bool, seed: int = 0, group_size: int = 64,
                  device: int = 0, rope_theta: float = 0.0, layer_range=None,
                  max_chunk: int = 512) -> "Transformer":
        """N(0, 0.02) weights generated on the device (no file)."""
        lb, le = layer_range if layer_range is not None else (0, -1)
        c = ModelConfigC(*config.as_tuple(), int(quantized), group_size if quantized else 0, 1)
        h = ctypes.c_void_p()
        check(lib().leap_engine_synthetic(ctypes.byref(c), seed, device, lb, le,
                                          ctypes.c_float(rope_theta), max_chunk,
                                          ctypes.byref(h)))
        return Transformer(h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            check(lib().leap_engine_destroy(self._h))
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
    def handle(self):
        if not self._h:
            raise LeapError(1, "engine is closed")
        return self._h

    def device_bytes(self) -> int:
        n = ctypes.c_size_t()
        check(lib().leap_engine_device_bytes(self.handle, ctypes.byref(n)))
        return n.value

    # -- the reference API ---------------------------------------------------
    def forward(self, token: int, pos: int, flags: int = FLAG_NEED_REPLY):
        """Logits for the next position (a copy of the engine's buffer).  With
        FLAG_NO_REPLY only the cache is advanced and None is returned, as the
        reference master does for prompt tokens (FloatTransformer.cpp:789-790)."""
        if flags == FLAG_NO_REPLY:
            nxt = ctypes.c_int()
            check(lib().leap_engine_forward(self.handle, token, pos, None, ctypes.byref(nxt)))
            return None
        nxt = ctypes.c_int()
        check(lib().leap_engine_forward(self.handle, token, pos,
                                        self._logits.ctypes.data_as(_fp), ctypes.byref(nxt)))
        self.last_token = nxt.value
        return self._logits.copy()

    def set_sampler(self, sampler) -> None:
        """Next tokens from `sampler` (a leap_b200.Sampler on this engine's
        device) instead of the greedy argmax; None restores argmax.  The
        engine keeps a reference, not ownership."""
        self._sampler = sampler
        check(lib().leap_engine_set_sampler(self.handle,
                                            sampler.handle if sampler is not None else None))

    def forward_argmax(self, token: int, pos: int) -> int:
        """Next token: the greedy argmax, or the draw of the sampler set."""
        nxt = ctypes.c_int()
        check(lib().leap_engine_forward(self.handle, token, pos, None, ctypes.byref(nxt)))
        return nxt.value

    def prefill(self, tokens, pos0: int = 0) -> int:
        """Run a prompt through the cache in chunks; returns the greedy token
        that follows it."""
        t = np.ascontiguousarray(tokens, np.int32)
        nxt = ctypes.c_int()
        check(lib().leap_engine_prefill(self.handle, t.ctypes.data_as(_ip), int(t.size), pos0,
                                        ctypes.byref(nxt)))
        return nxt.value

    def generate(self, prompt, steps: int, batched_prompt: bool = True):
        """Greedy decode of `steps` tokens after `prompt` (main.cpp:64-108 at
        temperature 0).  Returns the generated tokens."""
        prompt = list(prompt)
        if batched_prompt:
            tok = self.prefill(prompt, 0)
        else:
            for p, t in enumerate(prompt[:-1]):
                self.forward(t, p, FLAG_NO_REPLY)
            tok = self.forward_argmax(prompt[-1], len(prompt) - 1)
        out = [tok]
        pos = len(prompt)
        for _ in range(steps - 1):
            tok = self.forward_argmax(tok, pos)
            out.append(tok)
            pos += 1
        return out

    def clear_kv_cache(self) -> None:
        """Transformer::clear_kv_cache (FloatTransformer.cpp:74-77)."""
        check(lib().leap_engine_clear_kv(self.handle))

    # -- stage operations on device tensors (pipeline) -------------------------
    def bind_torch_stream(self, stream=None) -> None:
        import torch
        if stream is None:
            stream = torch.cuda.current_stream()
        check(lib().leap_engine_set_stream(self.handle, ctypes.c_void_p(stream.cuda_stream)))

    def sync(self) -> None:
        check(lib().leap_engine_sync(self.handle))

    def embed(self, tokens, x) -> None:
        t = np.ascontiguousarray(tokens, np.int32)
        check(lib().leap_engine_embed(self.handle, t.ctypes.data_as(_ip), int(t.size),
                                      x.data_ptr()))

    def embed_device(self, tokens, x) -> None:
        """Embed int32 token ids that are already on the device."""
        check(lib().leap_engine_embed_device(self.handle, tokens.data_ptr(), int(tokens.numel()),
                                             x.data_ptr()))

    def layers(self, pos0: int, x) -> None:
        check(lib().leap_engine_layers(self.handle, pos0, int(x.shape[0]), x.data_ptr()))

    def head(self, x, logits=None, token=None) -> None:
        check(lib().leap_engine_head(self.handle, x.data_ptr(),
                                     logits.data_ptr() if logits is not None else None,
                                     token.data_ptr() if token is not None else None))
