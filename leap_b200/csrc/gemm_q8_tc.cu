// gemm_q8_tc.cu — W8A8 matrix x prompt-chunk product on tcgen05 tensor cores.
//
// y[t][r] (+ res[t][r]) for t < T tokens and r < d weight rows, with the
// reference's W8A8 arithmetic (src/inference/QuantizedTransformer.cpp:359-652):
// per output, over the 64-element groups g in order,
//     val = fma(float(dot_g), w_s[r][g] * x_s[t][g], val)
// where dot_g is the exact int32 dot product of the group's int8 weights and
// int8 activations.  The tensor core forms every dot_g (kind::i8, int32
// accumulate: exact in any order); the fma chain runs in FP32 registers in
// group order, so the outputs are bit-identical to the CUDA-core GEMM and to
// the GEMV run token by token.
//
// CTA = 128 weight rows (the TMEM lanes) x 64 tokens.  Warps:
//   warp 8      TMA producer: 128-byte K slices (two groups) of the weight
//               tile [128 rows] and the activation tile [64 tokens] into a
//               4-stage ring, 128-byte swizzle (the K-major operand layout);
//   warp 9      one elected lane issues two K=32 MMAs per group into one of
//               four TMEM buffers of 64 int32 columns (a fresh accumulator
//               per group, so each group's dot stays separate);
//   warps 0-7   epilogue: warp w reads TMEM lanes 32(w%4).. (its 32 rows) and
//               columns 32(w/4).. (its 32 tokens) of each group's buffer,
//               releases the buffer, and advances its 32 x 32 chains.
// Every hand-off is an mbarrier and every wait is bounded; a wait that gives
// up stops the CTA after what is in flight has landed, and is reported
// through the error word.  No TMA load here uses cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "ctx.h"
#include "engine.h"
#include "tc.cuh"

namespace leap {
namespace eng {
namespace {

constexpr int kQM = 128;                  // weight rows per CTA = TMEM lanes
constexpr int kQN = 64;                   // tokens per CTA
constexpr int kQKc = 128;                 // bytes of K per stage: two groups
constexpr int kQS = 4;                    // stages
constexpr int kQNB = 4;                   // TMEM group buffers of kQN columns
constexpr int kQEpi = 8;                  // epilogue warps
constexpr int kQThreads = 32 * (kQEpi + 2);
constexpr int kQGB = 8;                   // groups per scale block
constexpr uint32_t kQABytes = kQM * kQKc;             // 16 KB
constexpr uint32_t kQBBytes = kQN * kQKc;             // 8 KB
constexpr uint32_t kQStageBytes = kQABytes + kQBBytes;  // multiple of 1024
constexpr uint32_t kQXsWarp = kQGB * 32 * 4;          // a warp's x scales [8][32]
constexpr size_t kQSmem = size_t(kQS) * kQStageBytes + kQEpi * kQXsWarp + 1024;
constexpr uint32_t kQTmemCols = kQNB * kQN;           // 256
static_assert(kQStageBytes % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");

// 32-bit instruction descriptor for kind::i8: D S32 (bits 4-5 = 2), A and B
// signed 8-bit (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17,
// M >> 4 at bit 24 (the layout of tc::idesc_tf32).
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) |
           (uint32_t(M >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] . B[smem desc]^T, int8 x int8 -> int32
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
        :
        : "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 2-D tiled TMA load of box (x, y) of `map` into this CTA's shared memory,
// completing its bytes on `bar`.  x is a byte offset, a multiple of 128.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// float(i) for |i| < 2^22, exactly: i added to the integer image of
// kMagic = 1.5 * 2^23 lands on the float kMagic + i (unit spacing there), and
// subtracting kMagic leaves i.  A group dot is at most 64 * 128 * 128 = 2^20
// in magnitude.  An integer add and a (packed) float add instead of a
// conversion instruction.
constexpr float kMagic = 12582912.0f;
__device__ __forceinline__ float magic_image(int i) { return __int_as_float(i + 0x4B400000); }

__global__ void __launch_bounds__(kQThreads, 2)
gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                  float *y, const float *__restrict__ xs, const float *__restrict__ ws, int n,
                  int d, int T, const float *res, int *err) {
    extern __shared__ unsigned char smraw[];
    __shared__ uint64_t full[kQS], empty[kQS], dfull[kQNB], dempty[kQNB], fin;
    __shared__ uint32_t tmem_sh;
    __shared__ int s_fail;
    unsigned char *base = smraw + ((1024u - (smem_addr(smraw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_addr(base);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * kQN, r0 = blockIdx.y * kQM;
    const int ng = n >> 6, nch = (n + kQKc - 1) / kQKc;

    if (tid == 0) {
        for (int s = 0; s < kQS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < kQNB; ++b) {
            mbar_init(&dfull[b], 1);
            mbar_init(&dempty[b], kQEpi);
        }
        mbar_init(&fin, 1);
        s_fail = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tc::alloc(&tmem_sh, kQTmemCols);
        tc::relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_sh;

    if (warp == kQEpi) {
        // ---- TMA producer: K slice c into stage c % kQS ----------------------
        const bool leader = tc::elect_one_sync();
        bool ok = true;
        int c = 0;
        for (; c < nch; ++c) {
            const int s = c % kQS;
            if (c >= kQS)
                ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], uint32_t(c / kQS - 1) & 1u));
            if (!ok) break;
            if (leader) {
                mbar_arrive_expect_tx(&full[s], kQStageBytes);
                tma_load_2d(base + s * kQStageBytes, &tmw, c * kQKc, r0, &full[s]);
                tma_load_2d(base + s * kQStageBytes + kQABytes, &tmx, c * kQKc, t0, &full[s]);
            }
            __syncwarp();
        }
        if (!ok && lane == 0) atomicExch(&s_fail, 1);
        // the copies issued last have landed before shared memory is released
        for (int cc = max(0, c - kQS); cc < c; ++cc)
            (void)mbar_wait(&full[cc % kQS], uint32_t(cc / kQS) & 1u);
    } else if (warp == kQEpi + 1) {
        // ---- MMA issuer: group g = two K=32 products into buffer g % kQNB ----
        const bool leader = tc::elect_one_sync();
        const uint32_t idesc = idesc_i8(kQM, kQN);
        const uint64_t da0 = tc::sw128_kmajor_desc(sbase);
        const uint64_t db0 = tc::sw128_kmajor_desc(sbase + kQABytes);
        bool ok = true;
        for (int g = 0; g < ng; ++g) {
            const int c = g >> 1, s = c % kQS, b = g % kQNB;
            if ((g & 1) == 0) ok = __all_sync(0xffffffffu, mbar_wait(&full[s], uint32_t(c / kQS) & 1u));
            if (ok && g >= kQNB)
                ok = __all_sync(0xffffffffu, mbar_wait(&dempty[b], uint32_t(g / kQNB - 1) & 1u));
            if (!ok) break;
            tc::fence_after_sync();
            if (leader) {
                const uint64_t so = uint64_t(uint32_t(s) * kQStageBytes >> 4);
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {
                    // 32-byte K steps inside the 128-byte swizzled rows
                    const uint64_t ko = uint64_t(((g & 1) * 64 + kk * 32) >> 4);
                    mma_i8_ss(tmem + uint32_t(b * kQN), da0 + so + ko, db0 + so + ko, idesc,
                              kk ? 1u : 0u);
                }
                tc::commit(&dfull[b]);
                if ((g & 1) || g == ng - 1) tc::commit(&empty[s]);
            }
            __syncwarp();
        }
        if (!ok && lane == 0) atomicExch(&s_fail, 1);
        // every product has completed before TMEM and shared memory go
        if (leader) tc::commit(&fin);
        __syncwarp();
        (void)mbar_wait(&fin, 0);
    } else {
        // ---- epilogue: rows r0 + 32 (warp % 4) + lane, tokens t0 + 32 (warp / 4) + i
        const int q = warp & 3, h = warp >> 2;
        const int row = r0 + 32 * q + lane;
        const bool row_ok = row < d;
        const int tok = t0 + 32 * h + lane;  // the token whose x scales this lane loads
        const float *wsr = ws + size_t(row_ok ? row : 0) * ng;
        const float *xsr = xs + size_t(tok < T ? tok : 0) * ng;
        float *sxw = reinterpret_cast<float *>(base + kQS * kQStageBytes + warp * kQXsWarp);  // [8][32]
        const uint32_t tl = tmem + (uint32_t(32 * q) << 16) + uint32_t(32 * h);
        const int nblk = (ng + kQGB - 1) / kQGB;
        // scales of block k: this lane's row (w) and this lane's token (x);
        // ng % 4 == 0, so both are two aligned float4 reads
        auto load_scales = [&](int k, float (&w)[kQGB], float (&x)[kQGB]) {
            const int g0 = k * kQGB;
#pragma unroll
            for (int i = 0; i < kQGB / 4; ++i) {
                const bool in = g0 + 4 * i < ng;
                const float4 wv = (in && row_ok) ? *reinterpret_cast<const float4 *>(wsr + g0 + 4 * i)
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
                const float4 xv = (in && tok < T) ? *reinterpret_cast<const float4 *>(xsr + g0 + 4 * i)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                w[4 * i] = wv.x;
                w[4 * i + 1] = wv.y;
                w[4 * i + 2] = wv.z;
                w[4 * i + 3] = wv.w;
                x[4 * i] = xv.x;
                x[4 * i + 1] = xv.y;
                x[4 * i + 2] = xv.z;
                x[4 * i + 3] = xv.w;
            }
        };
        float2 val[16];  // tokens (2i, 2i + 1)
#pragma unroll
        for (int i = 0; i < 16; ++i) val[i] = make_float2(0.f, 0.f);
        float wcur[kQGB], wnxt[kQGB], xnxt[kQGB];
        load_scales(0, wcur, xnxt);
#pragma unroll
        for (int j = 0; j < kQGB; ++j) sxw[j * 32 + lane] = xnxt[j];
        __syncwarp();
        bool ok = true;
        for (int k = 0; k < nblk && ok; ++k) {
            if (k + 1 < nblk) load_scales(k + 1, wnxt, xnxt);
            const int gend = min(kQGB, ng - k * kQGB);
#pragma unroll
            for (int gg = 0; gg < kQGB; ++gg) {
                if (gg < gend && ok) {
                    const int g = k * kQGB + gg, b = g % kQNB;
                    ok = __all_sync(0xffffffffu, mbar_wait(&dfull[b], uint32_t(g / kQNB) & 1u));
                    if (ok) {
                        tc::fence_after_sync();
                        float dv[32];
                        tc::ld32(tl + uint32_t(b * kQN), dv);
                        tc::wait_ld();
                        tc::fence_before_sync();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&dempty[b]);
                        // token pairs in packed FP32x2 instructions, each
                        // half rounded exactly as the scalar fma / mul
                        const float2 wsg = make_float2(wcur[gg], wcur[gg]);
                        const float2 neg_c = make_float2(-kMagic, -kMagic);
                        const float4 *xr = reinterpret_cast<const float4 *>(sxw + gg * 32);
#pragma unroll
                        for (int i4 = 0; i4 < 8; ++i4) {
                            const float4 x4 = xr[i4];
                            const float2 xp[2] = {make_float2(x4.x, x4.y), make_float2(x4.z, x4.w)};
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int t = 4 * i4 + 2 * e;
                                const float2 dot = __fadd2_rn(
                                    make_float2(magic_image(__float_as_int(dv[t])),
                                                magic_image(__float_as_int(dv[t + 1]))),
                                    neg_c);
                                val[t / 2] = __ffma2_rn(dot, __fmul2_rn(wsg, xp[e]), val[t / 2]);
                            }
                        }
                    }
                }
            }
            __syncwarp();  // every lane is done with block k's x scales
            if (k + 1 < nblk) {
#pragma unroll
                for (int j = 0; j < kQGB; ++j) {
                    sxw[j * 32 + lane] = xnxt[j];
                    wcur[j] = wnxt[j];
                }
            }
            __syncwarp();
        }
        if (ok) {
            if (row_ok) {
#pragma unroll
                for (int t = 0; t < 32; ++t) {
                    const int tt = t0 + 32 * h + t;
                    if (tt < T) {
                        const size_t o = size_t(tt) * d + row;
                        const float v = (t & 1) ? val[t / 2].y : val[t / 2].x;
                        y[o] = res ? __fadd_rn(res[o], v) : v;
                    }
                }
            }
        } else if (lane == 0) {
            atomicExch(&s_fail, 1);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0 && s_fail) report_error(err, kDevWaitTimeout);
    if (warp == 0) tc::dealloc(tmem, kQTmemCols);
}

// cuTensorMapEncodeTiled from the driver, looked up once.
std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int encode_map(CUtensorMap *m, const void *base, int inner_bytes, int rows, int box_rows,
               const char *what) {
    std::call_once(g_encode_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) {
        set_error("gemm_q8_tc: cuTensorMapEncodeTiled is not available from the driver");
        return LEAP_ERR_CUDA;
    }
    const cuuint64_t dims[2] = {cuuint64_t(inner_bytes), cuuint64_t(rows)};
    const cuuint64_t strides[1] = {cuuint64_t(inner_bytes)};
    const cuuint32_t box[2] = {cuuint32_t(kQKc), cuuint32_t(box_rows)};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                                strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("gemm_q8_tc: cuTensorMapEncodeTiled(%s) failed (%d)", what, int(r));
        return LEAP_ERR_CUDA;
    }
    return LEAP_OK;
}

}  // namespace

bool gemm_q8_tc_supported(const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                          int n, int T) {
    const auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    // two-float4 scale reads need ng % 4 == 0 and 16-byte aligned scale rows
    return T >= 2 && n >= 256 && n % 256 == 0 && a16(xq) && a16(wq) && a16(xs) && a16(ws);
}

int gemm_q8_tc(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
               const float *ws, int n, int d, int T, const float *res, int *err) {
    CUtensorMap mw, mx;
    if (int rc = encode_map(&mw, wq, n, d, kQM, "weights")) return rc;
    if (int rc = encode_map(&mx, xq, n, T, kQN, "activations")) return rc;
    const void *fn = reinterpret_cast<const void *>(gemm_q8_tc_kernel);
    if (int rc = set_kernel_smem(fn, kQSmem, "cudaFuncSetAttribute(gemm_q8_tc)")) return rc;
    const dim3 grid(unsigned((T + kQN - 1) / kQN), unsigned((d + kQM - 1) / kQM));
    gemm_q8_tc_kernel<<<grid, kQThreads, kQSmem, st>>>(mw, mx, y, xs, ws, n, d, T, res, err);
    return cuda_status(cudaGetLastError(), "gemm_q8_tc_kernel launch");
}

}  // namespace eng
}  // namespace leap
