"""leap_attn_decode_noalloc: decode attention for callers that cannot allocate.

Some callers cannot call cudaMalloc — their device memory is owned by one
allocator or a fixed arena, or they are inside a region that must not change
the device's allocations — so they cannot create a context.  They pass their
own cache and buffers, and the library keeps its split-KV scratch in an array
compiled into it.  This test calls that entry point through the C ABI twice
in a row (the second call reads the row the first one appended) and checks
its output and appended rows against the regular context-based entry point
on the same inputs, within the decode tolerance, and that the calls change
no device allocation.

The file name puts it last in collection, so a run stopped at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from cases import SHAPES, decode_inputs, rel_err
from leap_b200 import AttentionContext, rope_table
from leap_b200._native import check, lib

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _noalloc(stream, h, kv, hd, pos, cos_d, sin_d, kc, vc, q, kn, vn, out):
    check(lib().leap_attn_decode_noalloc(
        ctypes.c_void_p(stream), h, kv, hd, pos, cos_d.data_ptr(), sin_d.data_ptr(),
        kc.data_ptr(), vc.data_ptr(), ctypes.c_longlong(kc.shape[1] * hd), q.data_ptr(),
        kn.data_ptr(), vn.data_ptr(), out.data_ptr()))


def test_noalloc_decode_matches_context_decode(cuda):
    h, kv, hd = SHAPES["l8b"]
    pos = 3000
    max_seq = 3072
    dev = cuda
    q, kn, vn, kr, vr = decode_inputs("l8b", pos, 4242)
    rng = np.random.default_rng(99)
    q2 = rng.standard_normal((h, hd), dtype=np.float32)
    kn2 = rng.standard_normal((kv, hd), dtype=np.float32)
    vn2 = rng.standard_normal((kv, hd), dtype=np.float32)
    c, s = rope_table(max_seq, hd)

    # the caller's own memory (the test harness allocates it; the entry
    # point under test allocates nothing)
    kc = torch.zeros(kv, max_seq, hd, device=dev)
    vc = torch.zeros(kv, max_seq, hd, device=dev)
    kc[:, :pos] = torch.from_numpy(kr.transpose(1, 0, 2).copy()).to(dev)
    vc[:, :pos] = torch.from_numpy(vr.transpose(1, 0, 2).copy()).to(dev)
    cos_d = torch.from_numpy(c).to(dev)
    sin_d = torch.from_numpy(s).to(dev)
    ins = [torch.from_numpy(x).to(dev) for x in (q, kn, vn, q2, kn2, vn2)]
    outs = [torch.empty(h, hd, device=dev) for _ in range(2)]
    stream = torch.cuda.current_stream(dev).cuda_stream
    torch.cuda.synchronize(dev)

    # first call on this device does its one-time set-up
    _noalloc(stream, h, kv, hd, pos, cos_d, sin_d, kc, vc, ins[0], ins[1], ins[2], outs[0])
    torch.cuda.synchronize(dev)
    free_before = torch.cuda.mem_get_info(dev)[0]
    _noalloc(stream, h, kv, hd, pos + 1, cos_d, sin_d, kc, vc, ins[3], ins[4], ins[5], outs[1])
    torch.cuda.synchronize(dev)
    assert torch.cuda.mem_get_info(dev)[0] == free_before, "the call changed device allocations"
    got = [o.cpu().numpy() for o in outs]
    rows = kc[:, pos:pos + 2].permute(1, 0, 2).cpu().numpy()
    vrows = vc[:, pos:pos + 2].permute(1, 0, 2).cpu().numpy()

    # the same two steps through the existing context entry point
    with AttentionContext(1, h, kv, hd, max_seq, rope_cos=c, rope_sin=s) as ctx:
        ctx.kv_write(0, 0, 0, kr, vr)
        r1 = ctx.decode(0, pos, ins[0], ins[1], ins[2])
        r2 = ctx.decode(0, pos + 1, ins[3], ins[4], ins[5])
        ctx.sync()
        ref = [r1.cpu().numpy(), r2.cpu().numpy()]
        kk, vv = ctx.kv_read(0, 0, pos, 2)

    for i in range(2):
        assert rel_err(got[i], ref[i]) <= TOL, f"call {i + 1}"
    np.testing.assert_array_equal(rows, kk)
    np.testing.assert_array_equal(vrows, vv)


def test_noalloc_rejects_what_does_not_fit(cuda):
    h, kv, hd = SHAPES["l8b"]
    t = torch.zeros(16, device=cuda)
    # head_stride too small for pos
    with pytest.raises(Exception):
        check(lib().leap_attn_decode_noalloc(None, h, kv, hd, 100, t.data_ptr(), t.data_ptr(),
                                             t.data_ptr(), t.data_ptr(),
                                             ctypes.c_longlong(100 * hd), t.data_ptr(),
                                             t.data_ptr(), t.data_ptr(), t.data_ptr()))
    # a context whose split-KV partials exceed the fixed scratch is refused
    # before anything is launched (pointers are never dereferenced)
    big = 1 << 20
    with pytest.raises(Exception, match="scratch"):
        check(lib().leap_attn_decode_noalloc(None, h, kv, hd, big - 1, t.data_ptr(), t.data_ptr(),
                                             t.data_ptr(), t.data_ptr(),
                                             ctypes.c_longlong(big * hd), t.data_ptr(),
                                             t.data_ptr(), t.data_ptr(), t.data_ptr()))
