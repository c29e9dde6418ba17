"""Ragged batched decode against the oracle applied to
each sequence (the reference has no batched path; its block per sequence is
the semantics)."""
import numpy as np
import pytest
import torch

import oracle
from cases import SHAPES, ragged_contexts, rel_err
from leap_b200 import AttentionContext, LeapError

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def tables():
    return {hd: oracle.rope_table(8192, hd, 500000.0) for hd in (64, 128)}


def _batch_inputs(shape, ctxs, seed):
    h, kv, hd = SHAPES[shape]
    rng = np.random.default_rng(seed)
    n = len(ctxs)
    q = rng.standard_normal((n, h, hd), dtype=np.float32)
    kn = rng.standard_normal((n, kv, hd), dtype=np.float32)
    vn = rng.standard_normal((n, kv, hd), dtype=np.float32)
    rows = [(rng.standard_normal((int(c) - 1, kv, hd), dtype=np.float32),
             rng.standard_normal((int(c) - 1, kv, hd), dtype=np.float32)) for c in ctxs]
    return q, kn, vn, rows


def _check(shape, ctxs, slots, max_batch, max_seq, tables, seed=3, layers=1, layer=0):
    h, kv, hd = SHAPES[shape]
    q, kn, vn, rows = _batch_inputs(shape, ctxs, seed)
    positions = np.asarray(ctxs, np.int32) - 1
    with AttentionContext(layers, h, kv, hd, max_seq, max_batch=max_batch) as ctx:
        for i, (kr, vr) in enumerate(rows):
            if len(kr):
                ctx.kv_write(int(slots[i]), layer, 0, kr, vr)
        out = ctx.decode_batched(layer, slots, positions, torch.from_numpy(q).cuda(),
                                 torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda())
        ctx.sync()
        out = out.cpu().numpy()
        c, s = tables[hd]
        for i, (kr, vr) in enumerate(rows):
            ref, kref = oracle.decode_case(q[i], kn[i], vn[i], kr, vr, int(positions[i]), h, kv,
                                           hd, c, s, threads=8)
            assert rel_err(out[i], ref) <= TOL, f"sequence {i}"
            kk, vv = ctx.kv_read(int(slots[i]), layer, int(positions[i]), 1)
            np.testing.assert_array_equal(kk[0], kref)
            np.testing.assert_array_equal(vv[0], vn[i])


def test_batched_config3_ragged_64(cuda, tables):
    """64 sequences, ctx ~ U[512, 8192] from seed 1,
    Llama-3-8B heads, fused RoPE + append."""
    ctxs = ragged_contexts(64, seed=1)
    _check("l8b", ctxs, np.arange(64), 64, 8192, tables)


def test_batched_permuted_slots_and_short(cuda, tables):
    ctxs = [1, 2, 33, 100, 257, 5]
    slots = np.array([5, 0, 7, 2, 3, 6])
    _check("tl", ctxs, slots, 8, 300, tables, seed=9, layers=3, layer=2)


def test_batched_more_than_one_launch(cuda, tables):
    """More sequences than one launch table holds (128) -> several launches."""
    rng = np.random.default_rng(4)
    ctxs = rng.integers(1, 60, 150)
    _check("g2_64", ctxs, np.arange(150), 150, 64, tables, seed=10)


def test_batched_rejects_repeated_slot(cuda):
    h, kv, hd = SHAPES["tl"]
    with AttentionContext(1, h, kv, hd, 32, max_batch=4) as ctx:
        q = torch.zeros(2, h, hd, device="cuda:0")
        k = torch.zeros(2, kv, hd, device="cuda:0")
        with pytest.raises(LeapError):
            ctx.decode_batched(0, [1, 1], [3, 4], q, k, k)
        with pytest.raises(LeapError):
            ctx.decode_batched(0, [0, 4], [3, 4], q, k, k)
