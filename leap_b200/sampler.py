"""The reference's Sampler on the GPU (src/inference/Sampler.h:12-33).

``Sampler(vocab_size, temperature, topp, rng_seed)`` keeps the reference's
constructor and ``sample(logits)``: temperature 0 is the greedy argmax,
otherwise softmax(logits / temperature) and one draw of the reference's
xorshift* generator per call, multinomial (topp outside (0, 1)) or top-p.
Logits are a CUDA tensor (not modified); ``sample`` returns a host int,
``sample_device`` leaves the token in device memory, stream-ordered.
"""
from __future__ import annotations

import ctypes

from ._native import check, lib


class Sampler:
    def __init__(self, vocab_size: int, temperature: float, topp: float, rng_seed: int,
                 device: int = 0):
        h = ctypes.c_void_p()
        check(lib().leap_sampler_create(int(vocab_size), float(temperature), float(topp),
                                        int(rng_seed) & ((1 << 64) - 1), int(device),
                                        ctypes.byref(h)))
        self.handle = h
        self.vocab_size = int(vocab_size)
        self.device = int(device)

    def sample_device(self, logits, out=None):
        """One draw on the current torch stream; returns a 1-element int32
        CUDA tensor holding the token."""
        import torch
        if logits.dtype != torch.float32 or not logits.is_cuda or not logits.is_contiguous():
            raise ValueError("logits must be a contiguous float32 CUDA tensor")
        if logits.numel() != self.vocab_size:
            raise ValueError(f"logits has {logits.numel()} values, vocab is {self.vocab_size}")
        if out is None:
            out = torch.empty(1, dtype=torch.int32, device=logits.device)
        stream = torch.cuda.current_stream(logits.device)
        check(lib().leap_sampler_sample(self.handle, ctypes.c_void_p(stream.cuda_stream),
                                        ctypes.c_void_p(logits.data_ptr()),
                                        ctypes.c_void_p(out.data_ptr())))
        return out

    def sample(self, logits) -> int:
        """Sampler::sample(logits) -> token id."""
        return int(self.sample_device(logits).item())

    @property
    def state(self) -> int:
        """The generator state after the draws so far (the reference's rng_state)."""
        v = ctypes.c_ulonglong()
        check(lib().leap_sampler_state(self.handle, ctypes.byref(v)))
        return int(v.value)

    def close(self) -> None:
        if getattr(self, "handle", None):
            check(lib().leap_sampler_destroy(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
