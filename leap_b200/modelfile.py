"""LEAP model files (.bin): header parsing and seeded synthetic writers.

Layouts follow the reference exporter and loader:

* v1 FP32 — ``src/export/Export.cpp:17-93``: magic ``0x616B3432``, int32
  version 1, the 7-int ``Config`` (``src/inference/Config.h:5-13``), a
  shared-classifier byte, zero padding to 256 bytes, then attention norms,
  FFN norms, final norm, token embeddings, wq, wk, wv, wo, w1, w2, w3 (each
  for all layers in turn) and the classifier if not shared.  The reference
  loader ties the classifier whenever ``vocab_size > 0``
  (``src/inference/TransformerFactory.cpp:115-118``), so these files are
  written tied.
* v2 W8A8 — ``Export.cpp:95-274``: the same header plus an int32 group size,
  FP32 norms, then per tensor ``int8[numel]`` followed by
  ``float32[numel / group_size]`` for the embeddings, wq..w3 per layer, and
  the classifier if not shared.  Quantization follows
  ``src/export/Utils.cpp:58-85``: ``s = max|w| / 127``,
  ``q = round_half_away(w * (1/s))``.

Synthetic weights are N(0, 0.02) from ``numpy.random.default_rng`` seeded per
tensor (tensors above 64M elements per 16M-element block), RMSNorm weights
1.0 — the BASELINE configs' description.  Blocks are generated and quantized
on a thread pool (numpy releases the GIL in both), so multi-GB files take
seconds to a few minutes; the bytes do not depend on the thread count.
"""
from __future__ import annotations

import concurrent.futures as cf
import dataclasses
import hashlib
import os
import struct

import numpy as np

MAGIC = 0x616B3432


@dataclasses.dataclass
class ModelConfig:
    dim: int
    hidden_dim: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    seq_len: int

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def as_tuple(self):
        return (self.dim, self.hidden_dim, self.n_layers, self.n_heads, self.n_kv_heads,
                self.vocab_size, self.seq_len)


def read_header(path: str):
    """(ModelConfig, quantized, group_size, shared_classifier, header_bytes),
    as TransformerFactory.cpp:59-118 reads it."""
    with open(path, "rb") as f:
        b = f.read(256)
    (magic,) = struct.unpack_from("<i", b, 0)
    quantized, gs, shared = 0, 0, 0
    if magic == MAGIC:
        (version,) = struct.unpack_from("<i", b, 4)
        cfg = struct.unpack_from("<7i", b, 8)
        if version == 1:
            hdr = 256
        elif version == 2:
            quantized = 1
            shared = b[36]
            (gs,) = struct.unpack_from("<i", b, 37)
            hdr = 256
        else:
            raise ValueError(f"Bad file version {version}")
    else:
        cfg = struct.unpack_from("<7i", b, 0)
        hdr = 28
    cfg = list(cfg)
    if not quantized:
        shared = 1 if cfg[5] > 0 else 0
        cfg[5] = abs(cfg[5])
    return ModelConfig(*cfg), quantized, gs, shared, hdr


def _rng(seed: int, name: str):
    h = hashlib.sha256(f"{seed}/{name}".encode()).digest()
    return np.random.default_rng(int.from_bytes(h[:8], "little"))


def _normal(seed, name, shape, std=0.02):
    return (_rng(seed, name).standard_normal(shape, dtype=np.float32) * np.float32(std))


def _quantize_block(w: np.ndarray, gs: int):
    g = w.reshape(-1, gs)
    wmax = np.abs(g).max(axis=1).astype(np.float32)
    s = (wmax / np.float32(127.0)).astype(np.float32)
    inv = np.where(s != 0, np.float32(1.0) / np.where(s != 0, s, np.float32(1)), np.float32(0))
    v = (g * inv[:, None].astype(np.float32)).astype(np.float32)
    q = (np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))).astype(np.int8)
    return q.reshape(-1), s


def quantize_q80(w: np.ndarray, gs: int):
    """src/export/Utils.cpp:58-85 on a flat float32 array: per group of `gs`,
    s = max|w| / 127 and q = round-half-away-from-zero(w * (1/s)), all in
    float32.  Worked in 1M-element pieces so the temporaries stay in cache."""
    w = w.reshape(-1)
    piece = (1 << 20) // gs * gs
    if w.size <= piece:
        return _quantize_block(w, gs)
    q = np.empty(w.size, np.int8)
    s = np.empty(w.size // gs, np.float32)
    for a in range(0, w.size, piece):
        qa, sa = _quantize_block(w[a:a + piece], gs)
        q[a:a + qa.size] = qa
        s[a // gs:a // gs + sa.size] = sa
    return q, s


_BIG = 1 << 26    # tensors above this many elements are seeded per block
_BLOCK = 1 << 24  # elements per block of a big tensor


def _blocks(name: str, numel: int):
    """(rng name, element count) of each seeded block of a tensor, in order."""
    if numel <= _BIG:
        return [(name, numel)]
    return [(f"{name}#{i}", min(_BLOCK, numel - a)) for i, a in enumerate(range(0, numel, _BLOCK))]


def _threads() -> int:
    return max(1, min(32, os.cpu_count() or 1))


def _write_tensors(f, items, seed: int, quant_gs: int = 0) -> None:
    """Write each (name, shape) tensor of `items` in order: FP32, or (with
    quant_gs) its int8 codes followed by its float32 group scales."""
    jobs = []
    for name, shape in items:
        numel = int(np.prod(shape))
        for bname, n in _blocks(name, numel):
            jobs.append((name, bname, n))

    def make(job):
        _, bname, n = job
        w = _normal(seed, bname, (n,))
        return quantize_q80(w, quant_gs) if quant_gs else w

    pending_scales: list[np.ndarray] = []
    current = None
    nt = _threads()
    with cf.ThreadPoolExecutor(max_workers=nt) as ex:
        window = []
        it = iter(jobs)

        def refill():
            for job in it:
                window.append((job, ex.submit(make, job)))
                if len(window) >= 2 * nt:
                    break
        refill()
        while window:
            job, fut = window.pop(0)
            res = fut.result()
            refill()
            name = job[0]
            if quant_gs:
                if current is not None and name != current:
                    for sc in pending_scales:
                        f.write(sc.tobytes())
                    pending_scales = []
                current = name
                f.write(res[0].tobytes())
                pending_scales.append(res[1])
            else:
                f.write(res.tobytes())
    for sc in pending_scales:
        f.write(sc.tobytes())


def _tensors(cfg: ModelConfig, seed: int):
    """(name, shape) in file order for the per-layer weight matrices."""
    L, d, h, kv = cfg.n_layers, cfg.dim, cfg.hidden_dim, cfg.kv_dim
    order = []
    for kind, shape in (("wq", (d, d)), ("wk", (kv, d)), ("wv", (kv, d)), ("wo", (d, d)),
                        ("w1", (h, d)), ("w2", (d, h)), ("w3", (h, d))):
        for l in range(L):
            order.append((f"{kind}.{l}", shape))
    return order


def write_v1(path: str, cfg: ModelConfig, seed: int = 0) -> None:
    """Synthetic FP32 model (tied classifier)."""
    with open(path, "wb") as f:
        hdr = struct.pack("<Ii", MAGIC, 1) + struct.pack("<7i", *cfg.as_tuple()) + bytes([1])
        f.write(hdr + bytes(256 - len(hdr)))
        ones = np.ones(cfg.dim, np.float32)
        for _ in range(2 * cfg.n_layers + 1):
            f.write(ones.tobytes())
        _write_tensors(f, [("tok", (cfg.vocab_size, cfg.dim))] + _tensors(cfg, seed), seed)


def write_v2(path: str, cfg: ModelConfig, seed: int = 0, group_size: int = 64) -> None:
    """Synthetic W8A8 model (tied classifier)."""
    with open(path, "wb") as f:
        hdr = (struct.pack("<Ii", MAGIC, 2) + struct.pack("<7i", *cfg.as_tuple()) + bytes([1])
               + struct.pack("<i", group_size))
        f.write(hdr + bytes(256 - len(hdr)))
        ones = np.ones(cfg.dim, np.float32)
        for _ in range(2 * cfg.n_layers + 1):
            f.write(ones.tobytes())
        _write_tensors(f, [("tok", (cfg.vocab_size, cfg.dim))] + _tensors(cfg, seed), seed,
                       quant_gs=group_size)


def write_timing_file(path: str, cfg: ModelConfig, quantized: bool, group_size: int = 64,
                      seed: int = 0) -> None:
    """A model file of `cfg`'s shape for TIMING only: every tensor is filled
    from one repeated 16 MB block of N(0, 0.02) values (W8A8: their int8
    codes and scales), which writes multi-GB files in seconds.  The engines'
    work per token does not depend on the weight values."""
    rng = np.random.default_rng(seed)
    block = (rng.standard_normal(1 << 22, dtype=np.float32) * np.float32(0.02))
    bq, bs = quantize_q80(block, group_size)

    def fill(f, numel, kind):
        src = {"f32": block, "q": bq, "s": bs}[kind]
        while numel > 0:
            n = min(numel, src.size)
            f.write(src[:n].tobytes())
            numel -= n

    with open(path, "wb") as f:
        if quantized:
            hdr = (struct.pack("<Ii", MAGIC, 2) + struct.pack("<7i", *cfg.as_tuple()) + bytes([1])
                   + struct.pack("<i", group_size))
        else:
            hdr = struct.pack("<Ii", MAGIC, 1) + struct.pack("<7i", *cfg.as_tuple()) + bytes([1])
        f.write(hdr + bytes(256 - len(hdr)))
        ones = np.ones(cfg.dim, np.float32).tobytes()
        for _ in range(2 * cfg.n_layers + 1):
            f.write(ones)
        shapes = [("tok", (cfg.vocab_size, cfg.dim))] + _tensors(cfg, seed)
        for name, shape in shapes:
            numel = int(np.prod(shape))
            if quantized:
                fill(f, numel, "q")
                fill(f, numel // group_size, "s")
            else:
                fill(f, numel, "f32")
