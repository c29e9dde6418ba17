"""Generate the golden fixtures from the reference's OWN compiled code.

Run in a container that has the reference sources (``make -C oracle ref``
builds ``oracle/_ref/libleapref_attn.so`` from the line ranges of
src/inference/FloatTransformer.cpp / QuantizedTransformer.cpp):

    python tests/golden/make_golden.py

Writes ``tests/golden/golden.npz`` (outputs only; inputs are regenerated
from the seeds in tests/cases.py and checked by fingerprint) and
``tests/golden/manifest.json``.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import oracle  # noqa: E402
from cases import (DECODE_POSITIONS, PREFILL_CASES, SHAPES, case_seed,  # noqa: E402
                   decode_inputs, fingerprint, prefill_inputs)

THETA = 500000.0


def main() -> None:
    if not oracle.build_ref():
        raise SystemExit("reference sources not found; cannot make golden fixtures")
    out: dict[str, np.ndarray] = {}
    manifest: dict = {"theta": THETA, "decode": [], "prefill": [], "rope": []}

    # --- RoPE tables (a1): hashes of the reference's own tables ------------
    for theta in (500000.0, 10000.0):
        for hd in (64, 128):
            c, s = oracle.rope_table(8192, hd, theta, impl="ref")
            manifest["rope"].append({
                "theta": theta, "head_dim": hd, "seq_len": 8192,
                "sha256": hashlib.sha256(c.tobytes() + s.tobytes()).hexdigest(),
            })
            out[f"rope/{int(theta)}/{hd}/rows"] = np.concatenate(
                [c[[0, 1, 2047, 8191]], s[[0, 1, 2047, 8191]]])

    tables = {hd: oracle.rope_table(8192, hd, THETA, impl="ref") for hd in (64, 128)}

    # --- decode (a2-a6): one block per case --------------------------------
    for shape, plist in DECODE_POSITIONS.items():
        h, kv, hd = SHAPES[shape]
        c, s = tables[hd]
        for pos in plist:
            seed = case_seed("decode", shape, pos)
            q, kn, vn, kr, vr = decode_inputs(shape, pos, seed)
            o, krow = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s,
                                         impl="ref", which=0)
            o_q, krow_q = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s,
                                             impl="ref", which=1)
            key = f"decode/{shape}/{pos}"
            out[key + "/out"] = o
            out[key + "/krow"] = krow
            manifest["decode"].append({
                "shape": shape, "pos": pos, "seed": seed,
                "inputs": fingerprint(q, kn, vn, kr, vr),
                "w8a8_twin_identical": bool((o == o_q).all() and (krow == krow_q).all()),
            })

    # --- prefill (a10): the reference block run per position in order -------
    lib = oracle.ref_attn()
    fp = oracle._f
    for shape, pos0, n_tok in PREFILL_CASES:
        h, kv, hd = SHAPES[shape]
        c, s = tables[hd]
        seed = case_seed("prefill", shape, pos0, n_tok)
        q, k, v, kr, vr = prefill_inputs(shape, pos0, n_tok, seed)
        seq_len = pos0 + n_tok
        kc = np.zeros((seq_len, kv * hd), np.float32)
        vc = np.zeros((seq_len, kv * hd), np.float32)
        kc[:pos0] = kr.reshape(pos0, kv * hd)
        vc[:pos0] = vr.reshape(pos0, kv * hd)
        res = np.empty((n_tok, h, hd), np.float32)
        att = np.empty(h * seq_len, np.float32)
        for i in range(n_tok):
            p = pos0 + i
            kc[p] = k[i].reshape(-1)
            vc[p] = v[i].reshape(-1)
            qq = np.ascontiguousarray(q[i].reshape(-1)).copy()
            xb = np.empty(h * hd, np.float32)
            lib.leapref_attn_block(0, h, kv, hd, seq_len, p, c.ctypes.data_as(fp),
                                   s.ctypes.data_as(fp), qq.ctypes.data_as(fp),
                                   kc.ctypes.data_as(fp), vc.ctypes.data_as(fp),
                                   att.ctypes.data_as(fp), xb.ctypes.data_as(fp))
            res[i] = xb.reshape(h, hd)
        key = f"prefill/{shape}/{pos0}/{n_tok}"
        out[key + "/out"] = res
        out[key + "/kcache"] = kc[pos0:].reshape(n_tok, kv, hd)
        manifest["prefill"].append({"shape": shape, "pos0": pos0, "n_tok": n_tok,
                                    "seed": seed, "inputs": fingerprint(q, k, v, kr, vr)})

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    print(f"wrote {len(out)} arrays")


if __name__ == "__main__":
    main()
