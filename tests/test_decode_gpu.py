"""Decode attention on the GPU, through the C ABI, against the oracle.

Tolerance (north_star): max|out - ref| <= 1e-4 * max|ref| for FP32 decode.
The new k row written to the cache must equal the reference's rotated row
bit for bit (RoPE uses separately rounded products, like the reference).
"""
import numpy as np
import pytest
import torch

import oracle
from cases import SHAPES, decode_inputs, rel_err
from leap_b200 import AttentionContext, LeapError

pytestmark = pytest.mark.gpu
TOL = 1e-4


@pytest.fixture(scope="module")
def tables():
    return {hd: oracle.rope_table(8192, hd, 500000.0) for hd in (64, 128)}


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to("cuda:0")


def _run(ctx, layer, pos, q, kn, vn, kr, vr):
    if pos:
        ctx.kv_write(0, layer, 0, kr, vr)
    out = ctx.decode(layer, pos, _dev(q), _dev(kn), _dev(vn))
    ctx.sync()
    kk, vv = ctx.kv_read(0, layer, pos, 1)
    return out.cpu().numpy(), kk[0], vv[0]


# split-KV with last-CTA combine (the auto choice here), cluster kernel, wide
# split-KV, split-KV with a separate combine launch
IMPLS = [1, 2, 3, 4]


@pytest.mark.parametrize("impl", IMPLS)
def test_decode_golden(cuda, golden, impl):
    data, man = golden
    ctxs = {}
    for case in man["decode"]:
        shape, pos = case["shape"], case["pos"]
        h, kv, hd = SHAPES[shape]
        if shape not in ctxs:
            ctxs[shape] = AttentionContext(1, h, kv, hd, 1100)
            ctxs[shape].set_decode_impl(impl)
        q, kn, vn, kr, vr = decode_inputs(shape, pos, case["seed"])
        out, krow, vrow = _run(ctxs[shape], 0, pos, q, kn, vn, kr, vr)
        key = f"decode/{shape}/{pos}"
        e = rel_err(out, data[key + "/out"])
        assert e <= TOL, f"{key}: rel err {e:.3g}"
        np.testing.assert_array_equal(krow, data[key + "/krow"])
        np.testing.assert_array_equal(vrow, vn)
    for c in ctxs.values():
        c.close()


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("ctx_len", [1024, 4096, 8192])
def test_decode_config2_l8b(cuda, tables, ctx_len, impl):
    """Llama-3-8B heads, one query at ctx 1024/4096/8192."""
    h, kv, hd = SHAPES["l8b"]
    pos = ctx_len - 1
    q, kn, vn, kr, vr = decode_inputs("l8b", pos, 2000 + ctx_len)
    with AttentionContext(1, h, kv, hd, 8192) as ctx:
        ctx.set_decode_impl(impl)
        out, krow, _ = _run(ctx, 0, pos, q, kn, vn, kr, vr)
    c, s = tables[hd]
    ref, kref = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s, threads=8)
    assert rel_err(out, ref) <= TOL
    np.testing.assert_array_equal(krow, kref)


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("shape", ["tl", "l70b", "mha128", "g2_64"])
def test_decode_shapes_long(cuda, tables, shape, impl):
    """Every head layout at a context long enough for many splits."""
    h, kv, hd = SHAPES[shape]
    pos = 5000
    q, kn, vn, kr, vr = decode_inputs(shape, pos, 77)
    with AttentionContext(1, h, kv, hd, 6000) as ctx:
        ctx.set_decode_impl(impl)
        out, krow, _ = _run(ctx, 0, pos, q, kn, vn, kr, vr)
    c, s = tables[hd]
    ref, kref = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s, threads=8)
    assert rel_err(out, ref) <= TOL
    np.testing.assert_array_equal(krow, kref)


@pytest.mark.parametrize("impl", IMPLS)
def test_decode_split_and_tile_edges(cuda, tables, impl):
    """Positions on both sides of tile (32/64 rows) and split boundaries,
    and contexts shorter than the cluster (some CTAs own no rows)."""
    h, kv, hd = SHAPES["l8b"]
    c, s = tables[hd]
    with AttentionContext(1, h, kv, hd, 4096) as ctx:
        ctx.set_decode_impl(impl)
        for pos in (2, 14, 15, 16, 31, 32, 33, 63, 64, 65, 223, 224, 225, 447, 448, 1023,
                    1024, 2047, 2048, 4095):
            q, kn, vn, kr, vr = decode_inputs("l8b", pos, 31 + pos)
            out, krow, _ = _run(ctx, 0, pos, q, kn, vn, kr, vr)
            ref, kref = oracle.decode_case(q, kn, vn, kr, vr, pos, h, kv, hd, c, s, threads=8)
            assert rel_err(out, ref) <= TOL, pos
            np.testing.assert_array_equal(krow, kref)


@pytest.mark.parametrize("impl", IMPLS)
def test_decode_consecutive_steps(cuda, tables, impl):
    """Token-by-token decode: the cache grows through the kernel's own
    appends, as forward() does in the reference (main.cpp:80-89)."""
    h, kv, hd = SHAPES["tl"]
    c, s = tables[hd]
    rng = np.random.default_rng(5)
    n = 70
    kc = np.zeros((n, kv * hd), np.float32)
    vc = np.zeros((n, kv * hd), np.float32)
    with AttentionContext(2, h, kv, hd, 128) as ctx:
        ctx.set_decode_impl(impl)
        for pos in range(n):
            q = rng.standard_normal((h, hd), dtype=np.float32)
            kn = rng.standard_normal((kv, hd), dtype=np.float32)
            vn = rng.standard_normal((kv, hd), dtype=np.float32)
            out = ctx.decode(1, pos, _dev(q), _dev(kn), _dev(vn)).cpu().numpy()
            # the oracle's running cache: new row written, then rotated in
            # place by the block, as in the reference
            kc[pos] = kn.reshape(-1)
            vc[pos] = vn.reshape(-1)
            ref = oracle.attn_block(q.reshape(-1).copy(), kc, vc, pos, h, kv, hd, c, s)
            assert rel_err(out, ref.reshape(h, hd)) <= TOL, pos
        ctx.sync()
        kk, vv = ctx.kv_read(0, 1, 0, n)
        np.testing.assert_array_equal(kk.reshape(n, -1), kc)
        np.testing.assert_array_equal(vv.reshape(n, -1), vc)
        # layer 0 was never touched
        k0, _ = ctx.kv_read(0, 0, 0, n)
        assert not k0.any()


@pytest.mark.parametrize("impl", IMPLS)
@pytest.mark.parametrize("overlap", [True, False])
def test_decode_layer_chain_overlap(cuda, tables, overlap, impl):
    """Launch overlap: layer l's decode takes layer l-1's output as its q
    (so it must read q only after the previous kernel completed), layers
    alternate, and every step grows the caches; checked step by step."""
    h, kv, hd = SHAPES["l8b"]
    c, s = tables[hd]
    n_layers, n_steps, pos0 = 4, 6, 700
    rng = np.random.default_rng(17)
    kc = [np.zeros((pos0 + n_steps, kv * hd), np.float32) for _ in range(n_layers)]
    vc = [np.zeros((pos0 + n_steps, kv * hd), np.float32) for _ in range(n_layers)]
    with AttentionContext(n_layers, h, kv, hd, pos0 + n_steps) as ctx:
        ctx.set_overlap(overlap)
        ctx.set_decode_impl(impl)
        for layer in range(n_layers):
            kr = rng.standard_normal((pos0, kv, hd), dtype=np.float32)
            vr = rng.standard_normal((pos0, kv, hd), dtype=np.float32)
            ctx.kv_write(0, layer, 0, kr, vr)
            kc[layer][:pos0] = kr.reshape(pos0, -1)
            vc[layer][:pos0] = vr.reshape(pos0, -1)
        for step in range(n_steps):
            pos = pos0 + step
            x = rng.standard_normal((h, hd), dtype=np.float32)
            xd = _dev(x)
            news = []
            outs = []
            for layer in range(n_layers):
                kn = rng.standard_normal((kv, hd), dtype=np.float32)
                vn = rng.standard_normal((kv, hd), dtype=np.float32)
                xd = ctx.decode(layer, pos, xd, _dev(kn), _dev(vn))  # no sync between layers
                news.append((kn, vn))
                outs.append(xd)
            got = [o.cpu().numpy() for o in outs]
            for layer in range(n_layers):
                kn, vn = news[layer]
                kc[layer][pos] = kn.reshape(-1)
                vc[layer][pos] = vn.reshape(-1)
                # the oracle is fed the GPU's own input for this layer, so
                # errors do not compound through the chain; it rotates the
                # running cache row in place like the reference
                ref_in = x if layer == 0 else got[layer - 1]
                ref = oracle.attn_block(ref_in.reshape(-1).copy(), kc[layer], vc[layer], pos, h,
                                        kv, hd, c, s).reshape(h, hd)
                assert rel_err(got[layer], ref) <= TOL, (step, layer)
        ctx.sync()
        for layer in range(n_layers):
            kk, _ = ctx.kv_read(0, layer, pos0, n_steps)
            np.testing.assert_array_equal(kk.reshape(n_steps, -1), kc[layer][pos0:])


def test_decode_host_entry_point_matches_device(cuda):
    h, kv, hd = SHAPES["l8b"]
    pos = 3000
    q, kn, vn, kr, vr = decode_inputs("l8b", pos, 11)
    with AttentionContext(1, h, kv, hd, 4096) as ctx:
        ctx.kv_write(0, 0, 0, kr, vr)
        a = ctx.decode(0, pos, _dev(q), _dev(kn), _dev(vn)).cpu().numpy()
        b = ctx.decode_host(0, pos, q, kn, vn)
        b2 = ctx.decode_host(0, pos, q, kn, vn)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(b, b2)


def test_decode_argument_errors(cuda):
    h, kv, hd = SHAPES["l8b"]
    with AttentionContext(2, h, kv, hd, 64) as ctx:
        q = torch.zeros(h * hd + 1, device="cuda:0")
        k = torch.zeros(kv, hd, device="cuda:0")
        with pytest.raises(LeapError):
            ctx.decode(0, 64, q[:-1], k, k)        # pos == max_seq
        with pytest.raises(LeapError):
            ctx.decode(2, 0, q[:-1], k, k)         # layer out of range
        with pytest.raises(LeapError):
            ctx.decode(0, 0, q[1:], k, k)          # misaligned pointer
        ctx.sync()


def test_clear_kv_cache(cuda):
    h, kv, hd = SHAPES["tl"]
    with AttentionContext(1, h, kv, hd, 64) as ctx:
        ctx.kv_write(0, 0, 0, np.ones((10, kv, hd), np.float32), np.ones((10, kv, hd), np.float32))
        ctx.clear_kv_cache()
        ctx.sync()
        k, v = ctx.kv_read(0, 0, 0, 10)
        assert not k.any() and not v.any()


def test_cluster_capacity_query(cuda):
    """The context reports how many 16-CTA decode clusters fit at once (7 on
    the B200s measured here: one GPC has fewer than 16 usable SMs), and auto
    mode picks the cluster kernel only when every kv head's cluster fits."""
    h, kv, hd = SHAPES["l8b"]
    with AttentionContext(1, h, kv, hd, 64) as ctx:
        assert ctx.cluster_capacity() >= 1
