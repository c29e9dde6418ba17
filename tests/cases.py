"""Seeded synthetic inputs shared by the golden-fixture script and the tests.

All inputs are N(0,1) float32 from ``numpy.random.default_rng(seed)``, drawn
in a fixed order, matching the BASELINE configs' input description
("q/k/v and the cached K/V are N(0,1) fp32 from a seed").  The cache rows
0..pos-1 stand for already-rotated keys, as the cache holds them.
"""
from __future__ import annotations

import hashlib

import numpy as np

# (name, n_heads, n_kv_heads, head_dim)
SHAPES = {
    "l8b": (32, 8, 128),     # Llama-3-8B attention: kv_mul 4
    "tl": (32, 4, 64),       # TinyLlama: kv_mul 8, hd 64
    "l70b": (64, 8, 128),    # Llama-3-70B attention: kv_mul 8
    "mha128": (8, 8, 128),   # kv_mul 1
    "g2_64": (16, 8, 64),    # kv_mul 2
}

# Decode golden cases: every shape at positions that hit the reference's
# 4-key unrolled loop and its tail (:507, :595), tile and split edges.
DECODE_POSITIONS = {
    "l8b": [0, 1, 3, 4, 5, 31, 32, 33, 67, 255, 1000],
    "tl": [0, 2, 63, 64, 65, 300],
    "l70b": [0, 7, 129, 513],
    "mha128": [0, 9, 100],
    "g2_64": [0, 5, 77],
}

# Prefill golden cases: (shape, pos0, n_tok)
PREFILL_CASES = [("l8b", 0, 24), ("l8b", 13, 20), ("tl", 0, 40), ("l70b", 5, 12)]


def decode_inputs(shape: str, pos: int, seed: int):
    h, kv, hd = SHAPES[shape]
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((h, hd), dtype=np.float32)
    k_new = rng.standard_normal((kv, hd), dtype=np.float32)
    v_new = rng.standard_normal((kv, hd), dtype=np.float32)
    k_rows = rng.standard_normal((pos, kv, hd), dtype=np.float32)
    v_rows = rng.standard_normal((pos, kv, hd), dtype=np.float32)
    return q, k_new, v_new, k_rows, v_rows


def prefill_inputs(shape: str, pos0: int, n_tok: int, seed: int):
    h, kv, hd = SHAPES[shape]
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_tok, h, hd), dtype=np.float32)
    k = rng.standard_normal((n_tok, kv, hd), dtype=np.float32)
    v = rng.standard_normal((n_tok, kv, hd), dtype=np.float32)
    k_rows = rng.standard_normal((pos0, kv, hd), dtype=np.float32)
    v_rows = rng.standard_normal((pos0, kv, hd), dtype=np.float32)
    return q, k, v, k_rows, v_rows


def case_seed(kind: str, shape: str, a: int, b: int = 0) -> int:
    """Stable seed per case."""
    h = hashlib.sha256(f"{kind}/{shape}/{a}/{b}".encode()).digest()
    return int.from_bytes(h[:4], "little")


def fingerprint(*arrays) -> str:
    """SHA-256 over the bytes of the inputs (detects a changed generator)."""
    m = hashlib.sha256()
    for a in arrays:
        m.update(np.ascontiguousarray(a).tobytes())
    return m.hexdigest()[:16]


def ragged_contexts(n_seq: int = 64, seed: int = 1, lo: int = 512, hi: int = 8192):
    """Config 3's context lengths: uniform in [lo, hi] from seed 1."""
    return np.random.default_rng(seed).integers(lo, hi + 1, n_seq)


def rel_err(got: np.ndarray, ref: np.ndarray) -> float:
    """max|got-ref| / max|ref| — the north_star's tolerance measure."""
    return float(np.abs(got.astype(np.float64) - ref).max() / np.abs(ref).max())
