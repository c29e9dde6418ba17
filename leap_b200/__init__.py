"""leap_b200 — B200-native attention hot path for LEAP.

The per-layer GQA attention block of LEAP's CPU engines
(src/inference/FloatTransformer.cpp:404-662 and
src/inference/QuantizedTransformer.cpp:680-923), re-designed for sm_100a:
fused RoPE + KV append + split-KV decode attention, ragged batched decode,
and causal prefill, behind the C ABI declared in ``include/leap_b200.h``.
"""
from ._native import LIB_PATH, LeapError
from .attention import AttentionContext, rope_table

__all__ = ["AttentionContext", "LeapError", "rope_table", "LIB_PATH"]
__version__ = "0.1.0"
from .engine import FLAG_NEED_REPLY, FLAG_NO_REPLY, Transformer  # noqa: E402
from .modelfile import ModelConfig  # noqa: E402
from .sampler import Sampler  # noqa: E402

__all__ += ["Transformer", "ModelConfig", "FLAG_NEED_REPLY", "FLAG_NO_REPLY", "Sampler"]
