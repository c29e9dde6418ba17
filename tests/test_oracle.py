"""The CPU oracle (oracle/leap_oracle.c) pinned against the reference.

The fixtures in tests/golden/ were produced by the reference's OWN code
(oracle/_ref, compiled from src/inference/*.cpp line ranges) by
tests/golden/make_golden.py.  These tests need no GPU.
"""
import hashlib

import numpy as np
import pytest

import oracle
from cases import (SHAPES, decode_inputs, fingerprint, prefill_inputs, rel_err)


def test_rope_table_bit_exact(golden):
    data, man = golden
    for r in man["rope"]:
        c, s = oracle.rope_table(r["seq_len"], r["head_dim"], r["theta"], impl="port")
        h = hashlib.sha256(c.tobytes() + s.tobytes()).hexdigest()
        assert h == r["sha256"], f"rope table differs for {r}"
        rows = data[f"rope/{int(r['theta'])}/{r['head_dim']}/rows"]
        np.testing.assert_array_equal(
            rows, np.concatenate([c[[0, 1, 2047, 8191]], s[[0, 1, 2047, 8191]]]))


@pytest.fixture(scope="module")
def tables():
    return {hd: oracle.rope_table(8192, hd, 500000.0) for hd in (64, 128)}


def test_decode_port_matches_reference(golden, tables):
    data, man = golden
    worst = 0.0
    for case in man["decode"]:
        shape, pos, seed = case["shape"], case["pos"], case["seed"]
        h, kv, hd = SHAPES[shape]
        q, kn, vn, kr, vr = decode_inputs(shape, pos, seed)
        assert fingerprint(q, kn, vn, kr, vr) == case["inputs"], "input generator changed"
        c, s = tables[hd]
        out, krow = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s)
        key = f"decode/{shape}/{pos}"
        # the rotated k row written to the cache is bit-exact
        np.testing.assert_array_equal(krow, data[key + "/krow"])
        e = rel_err(out, data[key + "/out"])
        worst = max(worst, e)
        assert e <= 1e-5, f"{key}: rel err {e}"
    assert worst < 1e-5


def test_decode_port_threads_agree(tables):
    h, kv, hd = SHAPES["l8b"]
    q, kn, vn, kr, vr = decode_inputs("l8b", 300, 7)
    c, s = tables[hd]
    o1, _ = oracle.decode_case(q, kn, vn, kr, vr, 300, h, kv, hd, c, s, threads=1)
    o4, _ = oracle.decode_case(q, kn, vn, kr, vr, 300, h, kv, hd, c, s, threads=4)
    np.testing.assert_array_equal(o1, o4)


def test_prefill_port_matches_reference(golden, tables):
    data, man = golden
    for case in man["prefill"]:
        shape, pos0, n_tok, seed = case["shape"], case["pos0"], case["n_tok"], case["seed"]
        h, kv, hd = SHAPES[shape]
        q, k, v, kr, vr = prefill_inputs(shape, pos0, n_tok, seed)
        assert fingerprint(q, k, v, kr, vr) == case["inputs"]
        c, s = tables[hd]
        out, kc, _ = oracle.prefill(q, k, v, kr, vr, pos0, h, kv, hd, c, s)
        key = f"prefill/{shape}/{pos0}/{n_tok}"
        np.testing.assert_array_equal(kc[pos0:], data[key + "/kcache"])
        assert rel_err(out, data[key + "/out"]) <= 1e-5


def test_w8a8_twin_is_the_same_block(golden):
    """QuantizedTransformer.cpp:680-923 computes exactly what
    FloatTransformer.cpp:404-662 does (recorded from the reference)."""
    _, man = golden
    assert all(c["w8a8_twin_identical"] for c in man["decode"])


def test_tolerance_check_catches_a_planted_error(golden, tables):
    """Plant a mistake in the oracle's output (on the CPU) and check that the
    parity measure used by the GPU tests rejects it."""
    data, man = golden
    case = man["decode"][5]
    h, kv, hd = SHAPES[case["shape"]]
    q, kn, vn, kr, vr = decode_inputs(case["shape"], case["pos"], case["seed"])
    c, s = tables[hd]
    out, _ = oracle.decode_case(q, kn, vn, kr, vr, case["pos"], h, kv, hd, c, s)
    ref = data[f"decode/{case['shape']}/{case['pos']}/out"]
    bad = out.copy()
    bad[3, 17] += 1e-3 * np.abs(ref).max()
    assert rel_err(bad, ref) > 1e-4


@pytest.mark.skipif(not oracle.has_ref(), reason="reference build not present")
def test_reference_live_matches_port(tables):
    """Live check against the compiled reference block (not only fixtures)."""
    h, kv, hd = SHAPES["l8b"]
    c, s = tables[hd]
    for pos in (0, 6, 129):
        q, kn, vn, kr, vr = decode_inputs("l8b", pos, 1234 + pos)
        o1, k1 = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s, impl="port")
        o2, k2 = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s, impl="ref")
        np.testing.assert_array_equal(k1, k2)
        assert rel_err(o1, o2) <= 1e-5
