"""GPU: the support ops of the layer against the C restatement of the
reference functions they replace, each called through its C-ABI entry point
(leap_op_*), which launches the same kernel the engine launches.

Bit-exact: activation quantize (QuantizedTransformer.cpp:338-357), the W8A8
GEMV/GEMM (:359-652, 4-row blocks) and argmax (Sampler.cpp:20-120).
Tolerance: FP32 GEMV/GEMM (FloatTransformer.cpp:240-382) and rmsnorm
(:79-214), whose sums the GPU associates differently: per output
4 sqrt(n) eps sum|w x| (GEMV/GEMM) and 1e-6 of max|ref| (rmsnorm).
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
import refsrc
from leap_b200._native import LeapError, check, lib

pytestmark = pytest.mark.gpu


def _s():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _quantize_dev(x_d, gs=64):
    n = x_d.numel()
    q = torch.empty(n, dtype=torch.int8, device=x_d.device)
    s = torch.empty(n // gs, dtype=torch.float32, device=x_d.device)
    check(lib().leap_op_quantize(_s(), q.data_ptr(), s.data_ptr(), x_d.data_ptr(), n, gs))
    return q, s


@pytest.mark.parametrize("n", [64, 4096, 14336, 28672 * 3])
def test_quantize_bit_exact(cuda, n):
    r = np.random.default_rng(n)
    x = (r.standard_normal(n) * 3).astype(np.float32)
    if n > 256:
        x[:64] = 0                       # an all-zero group (scale 0)
        x[64:128] = np.float32(1e-30)    # a tiny group
        x[200] = np.float32(-1e4)        # one large value
    q, s = _quantize_dev(_dev(x))
    torch.cuda.synchronize()
    q0, s0 = oracle.quantize(x)
    assert np.array_equal(q.cpu().numpy(), q0)
    assert np.array_equal(s.cpu().numpy().view(np.uint32), s0.view(np.uint32))


def _qmm(xq, xs, wq, ws, n, d, T, res=None):
    y = torch.empty((T, d), dtype=torch.float32, device="cuda")
    check(lib().leap_op_qmatmul(_s(), y.data_ptr(), xq.data_ptr(), xs.data_ptr(), wq.data_ptr(),
                                ws.data_ptr(), n, d, T, 64,
                                res.data_ptr() if res is not None else None))
    return y


@pytest.fixture(params=[0, 1, 2], ids=["sliced", "regs", "stream"])
def q8_gemv(request):
    check(lib().leap_op_set_q8_gemv(request.param))
    yield request.param
    check(lib().leap_op_set_q8_gemv(2))  # the library default


@pytest.mark.parametrize("n,d", [(2048, 256), (4096, 6144), (14336, 4096), (8192, 1024),
                                 (28672, 256), (65536, 64), (5632, 37), (4096, 3), (256, 9),
                                 (4160, 100), (4160, 4001), (6208, 3601)])
def test_qmatmul_gemv_bit_exact(cuda, q8_gemv, n, d):
    r = np.random.default_rng(n * 7 + d)
    x = r.standard_normal(n).astype(np.float32)
    w = (r.standard_normal((d, n)) * 0.02).astype(np.float32)
    wq, ws = oracle.quantize(w.reshape(-1))
    xq_d, xs_d = _quantize_dev(_dev(x))
    y = _qmm(xq_d, xs_d, _dev(wq), _dev(ws), n, d, 1)
    torch.cuda.synchronize()
    xq, xs = oracle.quantize(x)
    ref = oracle.qmatmul(xq, xs, wq.reshape(d, n), ws.reshape(d, n // 64), threads=8)
    assert np.array_equal(y.cpu().numpy()[0], ref)
    # with a residual, as the engine's x += W.v uses it (y aliases res)
    res = _dev(np.arange(d, dtype=np.float32))
    wq_d, ws_d = _dev(wq), _dev(ws)  # kept alive until the kernel has run
    check(lib().leap_op_qmatmul(_s(), res.data_ptr(), xq_d.data_ptr(), xs_d.data_ptr(),
                                wq_d.data_ptr(), ws_d.data_ptr(), n, d, 1, 64, res.data_ptr()))
    torch.cuda.synchronize()
    assert np.array_equal(res.cpu().numpy(), (np.arange(d, dtype=np.float32) + ref))


@pytest.mark.parametrize("n,d", [(4096, 6144), (4096, 4096), (2048, 300), (320, 77), (64, 9),
                                 (8192, 1000), (14336, 64)])
@pytest.mark.parametrize("norm", [True, False], ids=["rmsnorm", "quantize"])
def test_qmatmul_fused_equals_separate_ops(cuda, n, d, norm):
    """leap_op_qmatmul_fused (the engine's decode-step GEMV with the norm and
    quantization in its prologue where x fits the spare stages, else the
    separate kernels) gives the bits of leap_op_rmsnorm_quantize /
    leap_op_quantize followed by leap_op_qmatmul, with and without a
    residual aliasing y; and the oracle's arithmetic for the quantize form."""
    r = np.random.default_rng(n * 5 + d + norm)
    x = (r.standard_normal(n) * 3).astype(np.float32)
    x[:64] = 0  # an all-zero group (scale 0)
    nw = (1 + 0.1 * r.standard_normal(n)).astype(np.float32)
    w = (r.standard_normal((d, n)) * 0.02).astype(np.float32)
    wq, ws = oracle.quantize(w.reshape(-1))
    x_d, nw_d, wq_d, ws_d = _dev(x), _dev(nw), _dev(wq), _dev(ws)
    q = torch.empty(n, dtype=torch.int8, device="cuda")
    sc = torch.empty(n // 64, dtype=torch.float32, device="cuda")
    if norm:
        check(lib().leap_op_rmsnorm_quantize(_s(), q.data_ptr(), sc.data_ptr(), x_d.data_ptr(),
                                             nw_d.data_ptr(), 1, n))
    else:
        q, sc = _quantize_dev(x_d)
    ref = _qmm(q, sc, wq_d, ws_d, n, d, 1)[0]
    nwp = nw_d.data_ptr() if norm else None
    y = torch.empty(d, dtype=torch.float32, device="cuda")
    check(lib().leap_op_qmatmul_fused(_s(), y.data_ptr(), x_d.data_ptr(), nwp, wq_d.data_ptr(),
                                      ws_d.data_ptr(), n, d, None))
    res = _dev(np.arange(d, dtype=np.float32))
    check(lib().leap_op_qmatmul_fused(_s(), res.data_ptr(), x_d.data_ptr(), nwp, wq_d.data_ptr(),
                                      ws_d.data_ptr(), n, d, res.data_ptr()))
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), ref.cpu().numpy())
    assert np.array_equal(res.cpu().numpy(), np.arange(d, dtype=np.float32) + ref.cpu().numpy())
    if not norm:
        xq, xs = oracle.quantize(x)
        want = oracle.qmatmul(xq, xs, wq.reshape(d, n), ws.reshape(d, n // 64), threads=8)
        assert np.array_equal(y.cpu().numpy(), want)


@pytest.mark.parametrize("n,d", [(2048, 2560), (4096, 6144), (320, 77), (64, 9), (5632, 100),
                                 (28672, 16)])
def test_matmul_fused_equals_separate_ops(cuda, n, d):
    """leap_op_matmul_fused (the FP32 decode step's GEMV with the RMSNorm in
    its prologue where x and the norm weight fit shared memory, else the
    separate kernels) gives the bits of leap_op_rmsnorm followed by
    leap_op_matmul, with and without a residual aliasing y."""
    r = np.random.default_rng(n * 3 + d)
    x = (r.standard_normal(n) * 3).astype(np.float32)
    nw = (1 + 0.1 * r.standard_normal(n)).astype(np.float32)
    w = (r.standard_normal((d, n)) * 0.02).astype(np.float32)
    x_d, nw_d, w_d = _dev(x), _dev(nw), _dev(w)
    xb = torch.empty(n, dtype=torch.float32, device="cuda")
    check(lib().leap_op_rmsnorm(_s(), xb.data_ptr(), x_d.data_ptr(), nw_d.data_ptr(), 1, n))
    ref = torch.empty(d, dtype=torch.float32, device="cuda")
    check(lib().leap_op_matmul(_s(), ref.data_ptr(), xb.data_ptr(), w_d.data_ptr(), n, d, 1, None))
    y = torch.empty(d, dtype=torch.float32, device="cuda")
    check(lib().leap_op_matmul_fused(_s(), y.data_ptr(), x_d.data_ptr(), nw_d.data_ptr(),
                                     w_d.data_ptr(), n, d, None))
    res = _dev(np.arange(d, dtype=np.float32))
    check(lib().leap_op_matmul_fused(_s(), res.data_ptr(), x_d.data_ptr(), nw_d.data_ptr(),
                                     w_d.data_ptr(), n, d, res.data_ptr()))
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), ref.cpu().numpy())
    want = (np.arange(d, dtype=np.float32) + ref.cpu().numpy()).astype(np.float32)
    assert np.array_equal(res.cpu().numpy(), want)


@pytest.mark.parametrize("T", [2, 33, 100])
def test_qmatmul_gemm_equals_gemv_rows(cuda, T):
    n, d = 4096, 1024 + 64
    r = np.random.default_rng(T)
    x = r.standard_normal((T, n)).astype(np.float32)
    w = (r.standard_normal((d, n)) * 0.02).astype(np.float32)
    res = r.standard_normal((T, d)).astype(np.float32)
    wq, ws = oracle.quantize(w.reshape(-1))
    wq_d, ws_d = _dev(wq), _dev(ws)
    xq_d, xs_d = _quantize_dev(_dev(x))
    y = _qmm(xq_d, xs_d, wq_d, ws_d, n, d, T, _dev(res))
    rows = [_qmm(xq_d[t * n:(t + 1) * n], xs_d[t * n // 64:(t + 1) * n // 64], wq_d, ws_d,
                 n, d, 1, _dev(res[t])) for t in range(T)]
    torch.cuda.synchronize()
    y = y.cpu().numpy()
    for t in range(T):
        assert np.array_equal(y[t], rows[t].cpu().numpy()[0])
    # and against the port, with the residual added after the group chain
    xq, xs = oracle.quantize(x[-1])
    ref = oracle.qmatmul(xq, xs, wq.reshape(d, n), ws.reshape(d, n // 64), threads=8)
    assert np.array_equal(y[-1], (res[-1] + ref).astype(np.float32))


@pytest.mark.parametrize("n,d,T", [(4096, 6144, 64), (14336, 4096, 100), (4096, 200, 130),
                                   (256, 128, 2), (8192, 1024, 512)])
def test_qmatmul_gemm_tensor_core_equals_dp4a(cuda, n, d, T):
    """The tcgen05 kind::i8 GEMM (impl 1, the default) and the CUDA-core
    dp4a GEMM (impl 0) give the same bits, with and without a residual, on
    ragged row and token tiles; sampled outputs equal the port's chain."""
    r = np.random.default_rng(n + d + T)
    x = r.standard_normal((T, n)).astype(np.float32)
    w = (r.standard_normal((d, n)) * 0.02).astype(np.float32)
    res = r.standard_normal((T, d)).astype(np.float32)
    wq, ws = oracle.quantize(w.reshape(-1))
    wq_d, ws_d = _dev(wq), _dev(ws)
    xq_d, xs_d = _quantize_dev(_dev(x))
    res_d = _dev(res)
    out = {}
    try:
        for impl in (0, 1):
            check(lib().leap_op_set_q8_gemm(impl))
            out[impl] = (_qmm(xq_d, xs_d, wq_d, ws_d, n, d, T).cpu().numpy(),
                         _qmm(xq_d, xs_d, wq_d, ws_d, n, d, T, res_d).cpu().numpy())
    finally:
        check(lib().leap_op_set_q8_gemm(1))  # the library default
    assert np.array_equal(out[1][0], out[0][0])
    assert np.array_equal(out[1][1], out[0][1])
    for t in sorted({0, T // 2, T - 1}):
        xq, xs = oracle.quantize(x[t])
        ref = oracle.qmatmul(xq, xs, wq.reshape(d, n), ws.reshape(d, n // 64), threads=8)
        assert np.array_equal(out[1][0][t], ref)
        assert np.array_equal(out[1][1][t], (res[t] + ref).astype(np.float32))


def test_qmatmul_gemm_impl_selection(cuda):
    with pytest.raises(LeapError):
        check(lib().leap_op_set_q8_gemm(2))
    check(lib().leap_op_set_q8_gemm(1))


def _mm(x_d, w_d, n, d, T, res=None):
    y = torch.empty((T, d), dtype=torch.float32, device="cuda")
    check(lib().leap_op_matmul(_s(), y.data_ptr(), x_d.data_ptr(), w_d.data_ptr(), n, d, T,
                               res.data_ptr() if res is not None else None))
    return y


@pytest.mark.parametrize("n,d,T", [(2048, 256, 1), (2048, 5632, 1), (5632, 2048, 1),
                                   (2048, 32000, 1), (2048, 2560, 7), (5632, 2048, 64),
                                   (2048, 256, 130)])
def test_matmul_f32(cuda, n, d, T):
    r = np.random.default_rng(n + d + T)
    x = r.standard_normal((T, n)).astype(np.float32)
    w = (r.standard_normal((d, n)) * 0.02).astype(np.float32)
    res = r.standard_normal((T, d)).astype(np.float32)
    y = _mm(_dev(x), _dev(w), n, d, T, _dev(res)).cpu().numpy()
    for t in sorted({0, T // 2, T - 1}):
        ref = oracle.matmul(x[t], w, threads=8)
        # both are FP32 sums of n products in different association orders:
        # each is within ~sqrt(n) * eps * sum|w x| of the exact value
        bound = 4 * np.sqrt(n) * np.finfo(np.float32).eps * (np.abs(w) @ np.abs(x[t]))
        err = np.abs((y[t] - res[t]) - ref)
        assert (err <= bound + 2 * np.finfo(np.float32).eps * np.abs(res[t])).all(), (
            t, float(err.max()), float(bound.min()))


@pytest.mark.parametrize("rows,dim", [(1, 2048), (1, 4096), (1, 8192), (37, 2048)])
def test_rmsnorm(cuda, rows, dim):
    r = np.random.default_rng(dim + rows)
    x = (r.standard_normal((rows, dim)) * 4).astype(np.float32)
    w = r.standard_normal(dim).astype(np.float32)
    x_d = _dev(x)
    o = torch.empty_like(x_d)
    check(lib().leap_op_rmsnorm(_s(), o.data_ptr(), x_d.data_ptr(), _dev(w).data_ptr(), rows,
                                dim))
    # in place, as the head uses it
    check(lib().leap_op_rmsnorm(_s(), x_d.data_ptr(), x_d.data_ptr(), _dev(w).data_ptr(), rows,
                                dim))
    o = o.cpu().numpy()
    assert np.array_equal(o, x_d.cpu().numpy())
    for i in sorted({0, rows - 1}):
        ref = oracle.rmsnorm(x[i], w)
        assert np.abs(o[i] - ref).max() <= 1e-6 * np.abs(ref).max()


@pytest.mark.parametrize("rows,dim", [(1, 2048), (1, 4096), (1, 8192), (9, 4096), (3, 14336 // 4)])
def test_rmsnorm_quantize_equals_rmsnorm_then_quantize(cuda, rows, dim):
    if dim % 64:
        pytest.skip("W8A8 rows are multiples of 64")
    r = np.random.default_rng(rows * dim)
    x = (r.standard_normal((rows, dim)) * 3).astype(np.float32)
    w = (1 + 0.1 * r.standard_normal(dim)).astype(np.float32)
    x_d, w_d = _dev(x), _dev(w)
    o = torch.empty_like(x_d)
    check(lib().leap_op_rmsnorm(_s(), o.data_ptr(), x_d.data_ptr(), w_d.data_ptr(), rows, dim))
    q1, s1 = _quantize_dev(o.reshape(-1))
    q2 = torch.empty(rows * dim, dtype=torch.int8, device="cuda")
    s2 = torch.empty(rows * dim // 64, dtype=torch.float32, device="cuda")
    check(lib().leap_op_rmsnorm_quantize(_s(), q2.data_ptr(), s2.data_ptr(), x_d.data_ptr(),
                                         w_d.data_ptr(), rows, dim))
    torch.cuda.synchronize()
    assert torch.equal(q1, q2)
    assert torch.equal(s1.view(torch.int32), s2.view(torch.int32))
    # and the quantization of the oracle's rmsnorm agrees but for last-bit
    # rounding of the norm (codes within 1)
    q0, _ = oracle.quantize(oracle.rmsnorm(x[0], w))
    assert np.abs(q0.astype(int) - q2.cpu().numpy()[:dim].astype(int)).max() <= 1


def _lane_order_argmax(v):
    """The reference scan (Sampler.cpp:20-120) keeps one running maximum per
    lane of 8 with a strict >, then reduces the lanes in order, and scans the
    n % 8 tail last: ties go to the lowest lane, then the lowest index."""
    n8 = v.size & ~7
    best = max(range(v.size), key=lambda i: (v[i], -(i & 7 if i < n8 else 8), -i))
    return best


ARGMAX_CASES = [(1, []), (7, [2, 5]), (32000, [9, 16]), (32000, [15, 8, 31999]),
                (128256, [17, 90, 128255]), (32003, [32001, 31999])]


def argmax_input(n, ties):
    r = np.random.default_rng(n + len(ties))
    v = r.standard_normal(n).astype(np.float32)
    if ties:
        v[ties] = v.max() + 1
    return v


def argmax_case_key(n, ties):
    return "argmax/" + "_".join(str(x) for x in [n] + list(ties))


@pytest.mark.parametrize("n,ties", ARGMAX_CASES)
def test_argmax_reference_tie_order(cuda, n, ties):
    """The reference Sampler's argmax (live, or its recorded answer)."""
    v = argmax_input(n, ties)
    tok = torch.empty(1, dtype=torch.int32, device="cuda")
    check(lib().leap_op_argmax(_s(), tok.data_ptr(), _dev(v).data_ptr(), n))
    want = (oracle.ref_argmax(v) if refsrc.live()
            else int(refsrc.recorded(argmax_case_key(n, ties))))
    assert int(tok.item()) == want == _lane_order_argmax(v)


def test_op_argument_errors(cuda):
    x = torch.zeros(100, device="cuda")
    q = torch.zeros(100, dtype=torch.int8, device="cuda")
    with pytest.raises(LeapError):
        check(lib().leap_op_quantize(_s(), q.data_ptr(), x.data_ptr(), x.data_ptr(), 100, 64))
    with pytest.raises(LeapError):
        check(lib().leap_op_qmatmul(_s(), x.data_ptr(), q.data_ptr(), x.data_ptr(), q.data_ptr(),
                                    x.data_ptr(), 128, 1, 1, 32, None))
    with pytest.raises(LeapError):
        check(lib().leap_op_matmul(_s(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 6, 1, 1, None))
