// prefill_tc.cu — causal prefill attention on the 5th-generation tensor
// cores (tcgen05, accumulators in TMEM) with an FP32-accurate 3xTF32 split.
//
// Semantics: the reference block (src/inference/FloatTransformer.cpp:
// 404-662) run for pos = pos0 .. pos0+n_tok-1 in order (the reference feeds
// prompts token by token, src/inference/main.cpp:80-89), i.e. causal
// attention of every prompt token over cache rows 0..its position.  The
// append kernel (prefill_attn.cu) has already rotated q (into `qrot`) and
// written the rotated k and raw v of the chunk into the cache.
//
// CTA = 128 query rows (BT tokens x G query heads sharing one kv head) x one
// kv head; thread i owns TMEM lane i = query row i.  TMEM (512 columns):
//   [  0,128) Q hi   [128,256) Q lo      (A operands of S = Q K^T)
//   [256,320) S, then P hi               (A operand of O += P V)
//   [320,384) P lo
//   [384,512) O accumulator
// Shared memory: K hi/lo as [64 keys][128 d] and V^T hi/lo as
// [128 d][64 keys], K-major with the 128-byte swizzle, written by the
// threads from row-major staging tiles that 1-D bulk copies bring in.
// Every product is hi*hi + hi*lo + lo*hi of a TF32 split (about 2^-21
// relative); softmax runs in FP32 registers, one row per thread.
#include "common.cuh"
#include "ctx.h"
#include "tc.cuh"

namespace leap {
namespace {

constexpr int kTcRows = 128;     // query rows per CTA = TMEM lanes
constexpr int kTcKeys = 64;      // keys per tile
constexpr int kTcHd = 128;       // head_dim handled here
constexpr int kTcThreads = 128;
constexpr uint32_t kColQhi = 0, kColQlo = 128, kColS = 256, kColPlo = 320, kColO = 384;
constexpr uint32_t kTmemCols = 512;
constexpr float kTcMaxLag = 8.0f;  // log2 of how far the running max may trail

// shared-memory layout (bytes from a 1024-byte aligned base)
constexpr uint32_t kOffKhi = 0;                    // 4 chunks x 64 rows x 128 B
constexpr uint32_t kOffKlo = 32768;
constexpr uint32_t kOffVThi = 65536;               // 2 chunks x 128 rows x 128 B
constexpr uint32_t kOffVTlo = 98304;
constexpr uint32_t kOffStK = 131072;               // staging K [64][128] fp32
constexpr uint32_t kOffStV = 163840;               // staging V [64][128] fp32
constexpr uint32_t kTcSmemUsed = 196608;
constexpr size_t kTcSmem = kTcSmemUsed + 1024;     // + alignment slack

struct TcArgs {
    const float *qrot;   // [n_tok][n_heads][128], rotated
    const float *kc;     // kv head 0 of (slot, layer); heads head_stride apart
    const float *vc;
    size_t head_stride;
    float *out;          // [n_tok][n_heads][128]
    int *err;
    int pos0, n_tok, n_heads;
    float scale_log2;
};

template <int G>
__global__ void __launch_bounds__(kTcThreads, 1) prefill_tc_kernel(const TcArgs a) {
    constexpr int BT = kTcRows / G;  // tokens per CTA
    extern __shared__ unsigned char smem_raw[];
    __shared__ uint64_t full_bar, s_bar, o_bar;
    __shared__ uint32_t tmem_base_sh;

    const int tid = threadIdx.x, warp = tid >> 5;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_addr(base);
    float *stK = reinterpret_cast<float *>(base + kOffStK);
    float *stV = reinterpret_cast<float *>(base + kOffStV);

    const int kvh = blockIdx.y;
    const int t0 = (gridDim.x - 1 - blockIdx.x) * BT;  // longest rows first
    const int t_last = min(t0 + BT, a.n_tok) - 1;
    const int kv_end = a.pos0 + t_last + 1;
    const int n_kt = (kv_end + kTcKeys - 1) / kTcKeys;
    const float *gK = a.kc + size_t(kvh) * a.head_stride;
    const float *gV = a.vc + size_t(kvh) * a.head_stride;

    // this thread's query row
    const int my_tok = t0 + tid / G;
    const int my_head = kvh * G + tid % G;
    const int qp = a.pos0 + my_tok;
    const bool row_valid = my_tok < a.n_tok;

    if (tid == 0) {
        mbar_init(&full_bar, 1);
        mbar_init(&s_bar, 1);
        mbar_init(&o_bar, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        tc::alloc(&tmem_base_sh, kTmemCols);
        tc::relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base_sh;
    const uint32_t lane_off = uint32_t(warp * 32) << 16;

    auto issue_tile = [&](int j) {
        const int k0 = j * kTcKeys;
        const int nr = min(kTcKeys, kv_end - k0);
        const uint32_t bytes = uint32_t(nr) * kTcHd * 4;
        mbar_arrive_expect_tx(&full_bar, 2 * bytes);
        bulk_g2s(stK, gK + size_t(k0) * kTcHd, bytes, &full_bar);
        bulk_g2s(stV, gV + size_t(k0) * kTcHd, bytes, &full_bar);
    };
    if (tid == 0) issue_tile(0);

    // Q row -> TMEM as hi / lo
    {
        const float *qrow = a.qrot + (size_t(my_tok) * a.n_heads + my_head) * kTcHd;
#pragma unroll 1
        for (int c = 0; c < kTcHd / 32; ++c) {
            float hi[32], lo[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (row_valid) v = *reinterpret_cast<const float4 *>(qrow + c * 32 + 4 * i);
                const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    hi[4 * i + e] = tc::tf32_hi(x[e]);
                    lo[4 * i + e] = x[e] - hi[4 * i + e];
                }
            }
            tc::st32(tmem + lane_off + kColQhi + 32 * c, hi);
            tc::st32(tmem + lane_off + kColQlo + 32 * c, lo);
        }
        tc::wait_st();
    }

    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // Issued / completed counts of the three asynchronous streams (tile
    // copies, S products, O products), tracked identically by every thread
    // so that a wait that gave up can drain what is still in flight.
    int tiles_issued = 1, tiles_done = 0, s_issued = 0, s_done = 0, o_issued = 0, o_done = 0;
    const uint32_t idesc_s = tc::idesc_tf32(kTcRows, kTcKeys);
    const uint32_t idesc_o = tc::idesc_tf32(kTcRows, kTcHd);
    const uint64_t dkhi = tc::sw128_kmajor_desc(sbase + kOffKhi);
    const uint64_t dklo = tc::sw128_kmajor_desc(sbase + kOffKlo);
    const uint64_t dvhi = tc::sw128_kmajor_desc(sbase + kOffVThi);
    const uint64_t dvlo = tc::sw128_kmajor_desc(sbase + kOffVTlo);

#pragma unroll 1
    for (int j = 0; j < n_kt; ++j) {
        const int k0 = j * kTcKeys;
        const int nr = min(kTcKeys, kv_end - k0);
        ok = mbar_wait(&full_bar, j & 1);
        if (ok) ++tiles_done;
        if (ok && j > 0) {
            ok = mbar_wait(&o_bar, (j - 1) & 1);  // PV(j-1) done
            if (ok) ++o_done;
        }
        ok = __syncthreads_and(ok);
        if (!ok) break;
        tc::fence_after_sync();

        // ---- staging -> K hi/lo [keys][d] and V^T hi/lo [d][keys] ----------
#pragma unroll 4
        for (int i = 0; i < kTcKeys * kTcHd / 4 / kTcThreads; ++i) {
            const int f = tid + kTcThreads * i;
            const int n = f >> 5, d = (f & 31) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (n < nr) v = reinterpret_cast<const float4 *>(stK)[f];
            float4 h, w;
            h.x = tc::tf32_hi(v.x); w.x = v.x - h.x;
            h.y = tc::tf32_hi(v.y); w.y = v.y - h.y;
            h.z = tc::tf32_hi(v.z); w.z = v.z - h.z;
            h.w = tc::tf32_hi(v.w); w.w = v.w - h.w;
            const uint32_t off = tc::sw128_offset(n, d, kTcKeys);
            *reinterpret_cast<float4 *>(base + kOffKhi + off) = h;
            *reinterpret_cast<float4 *>(base + kOffKlo + off) = w;
        }
        {
            const int d = tid;  // one V^T row per thread
#pragma unroll 4
            for (int jg = 0; jg < kTcKeys / 4; ++jg) {
                float x[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int n = 4 * jg + e;
                    x[e] = (n < nr) ? stV[n * kTcHd + d] : 0.f;
                }
                float4 h, w;
                h.x = tc::tf32_hi(x[0]); w.x = x[0] - h.x;
                h.y = tc::tf32_hi(x[1]); w.y = x[1] - h.y;
                h.z = tc::tf32_hi(x[2]); w.z = x[2] - h.z;
                h.w = tc::tf32_hi(x[3]); w.w = x[3] - h.w;
                const uint32_t off = tc::sw128_offset(d, 4 * jg, kTcHd);
                *reinterpret_cast<float4 *>(base + kOffVThi + off) = h;
                *reinterpret_cast<float4 *>(base + kOffVTlo + off) = w;
            }
        }
        fence_proxy_async_smem();  // operand writes -> visible to the MMA
        tc::fence_before_sync();
        __syncthreads();
        if (j + 1 < n_kt) ++tiles_issued;
        ++s_issued;

        if (warp == 0) {
            tc::fence_after_sync();
            if (tc::elect_one_sync()) {
                if (j + 1 < n_kt) issue_tile(j + 1);  // staging is free again
                // S = Qhi Khi + Qhi Klo + Qlo Khi   (M 128, N 64, K 128 in 16 steps)
#pragma unroll
                for (int term = 0; term < 3; ++term) {
#pragma unroll
                    for (int kk = 0; kk < kTcHd / 8; ++kk) {
                        const uint64_t bdesc =
                            (term == 1 ? dklo : dkhi) +
                            uint64_t(((kk >> 2) * (kTcKeys * 128) + (kk & 3) * 32) >> 4);
                        tc::mma_tf32_ts(tmem + kColS,
                                        tmem + (term == 2 ? kColQlo : kColQhi) + 8 * kk, bdesc,
                                        idesc_s, (term > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                tc::commit(&s_bar);
            }
            __syncwarp();
        }

        // ---- online softmax of this thread's row -----------------------------
        ok = mbar_wait(&s_bar, j & 1);
        if (ok) ++s_done;
        ok = __syncthreads_and(ok);
        if (!ok) break;
        tc::fence_after_sync();
        float s[2][32];
        tc::ld32(tmem + lane_off + kColS, s[0]);
        tc::ld32(tmem + lane_off + kColS + 32, s[1]);
        tc::wait_ld();
        float mt = m;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const int key = k0 + 32 * h + c;
                s[h][c] = (key <= qp && key < kv_end) ? s[h][c] * a.scale_log2 : -INFINITY;
                mt = fmaxf(mt, s[h][c]);
            }
        // The running max moves (and O in TMEM is rescaled: 4 loads, 128
        // multiplies and 4 stores per thread) only when the tile's max
        // exceeds it by more than 2^8; otherwise the probabilities of this
        // tile are formed against the old max and are at most 256, which
        // FP32 carries without loss.  The result O / l is the same function.
        const bool move = (m == -INFINITY) || (mt > m + kTcMaxLag);
        const float alpha = move ? ((m == -INFINITY) ? 0.f : fast_exp2(m - mt)) : 1.f;
        if (move) m = mt;
        float rs = 0.f;
        float phi[2][32], plo[2][32];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int c = 0; c < 32; ++c) {
                const float p = (s[h][c] == -INFINITY) ? 0.f : fast_exp2(s[h][c] - m);
                rs += p;
                phi[h][c] = tc::tf32_hi(p);
                plo[h][c] = p - phi[h][c];
            }
        l = l * alpha + rs;
        tc::st32(tmem + lane_off + kColS, phi[0]);
        tc::st32(tmem + lane_off + kColS + 32, phi[1]);
        tc::st32(tmem + lane_off + kColPlo, plo[0]);
        tc::st32(tmem + lane_off + kColPlo + 32, plo[1]);
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
            for (int c = 0; c < kTcHd / 32; ++c) {
                float o[32];
                tc::ld32(tmem + lane_off + kColO + 32 * c, o);
                tc::wait_ld();
#pragma unroll
                for (int i = 0; i < 32; ++i) o[i] *= alpha;
                tc::st32(tmem + lane_off + kColO + 32 * c, o);
            }
        }
        tc::wait_st();
        tc::fence_before_sync();
        __syncthreads();
        ++o_issued;

        if (warp == 0) {
            tc::fence_after_sync();
            if (tc::elect_one_sync()) {
                // O += Phi VThi + Phi VTlo + Plo VThi   (M 128, N 128, K 64 in 8 steps)
#pragma unroll
                for (int term = 0; term < 3; ++term) {
#pragma unroll
                    for (int kk = 0; kk < kTcKeys / 8; ++kk) {
                        const uint64_t bdesc =
                            (term == 1 ? dvlo : dvhi) +
                            uint64_t(((kk >> 2) * (kTcHd * 128) + (kk & 3) * 32) >> 4);
                        tc::mma_tf32_ts(tmem + kColO,
                                        tmem + (term == 2 ? kColPlo : kColS) + 8 * kk, bdesc,
                                        idesc_o, (j > 0 || term > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                tc::commit(&o_bar);
            }
            __syncwarp();
        }
    }

    if (ok) {
        ok = mbar_wait(&o_bar, (n_kt - 1) & 1);
        if (ok) ++o_done;
        ok = __syncthreads_and(ok);
    }
    if (ok) {
        tc::fence_after_sync();
        const float inv = 1.f / l;
        float *dst = a.out + (size_t(my_tok) * a.n_heads + my_head) * kTcHd;
#pragma unroll 1
        for (int c = 0; c < kTcHd / 32; ++c) {
            float o[32];
            tc::ld32(tmem + lane_off + kColO + 32 * c, o);
            tc::wait_ld();
            if (row_valid) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 v;
                    v.x = o[4 * i + 0] * inv;
                    v.y = o[4 * i + 1] * inv;
                    v.z = o[4 * i + 2] * inv;
                    v.w = o[4 * i + 3] * inv;
                    *reinterpret_cast<float4 *>(dst + 32 * c + 4 * i) = v;
                }
            }
        }
    } else {
        // A wait gave up: give what is still in flight a bounded chance to
        // land before the TMEM and shared memory are released, and report.
        while (tiles_done < tiles_issued && mbar_wait(&full_bar, tiles_done & 1)) ++tiles_done;
        while (s_done < s_issued && mbar_wait(&s_bar, s_done & 1)) ++s_done;
        while (o_done < o_issued && mbar_wait(&o_bar, o_done & 1)) ++o_done;
        if (tid == 0) report_error(a.err, kDevWaitTimeout);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::dealloc(tmem, kTmemCols);
}

template <int G>
int launch_tc_g(leap_ctx *c, const TcArgs &a) {
    const void *fn = reinterpret_cast<const void *>(prefill_tc_kernel<G>);
    if (const int st = set_kernel_smem(fn, kTcSmem, "cudaFuncSetAttribute(prefill_tc)")) return st;
    constexpr int BT = kTcRows / G;
    dim3 grid((a.n_tok + BT - 1) / BT, c->n_kv);
    prefill_tc_kernel<G><<<grid, kTcThreads, kTcSmem, c->stream>>>(a);
    return cuda_status(cudaGetLastError(), "prefill_tc_kernel launch");
}

}  // namespace

int launch_prefill_tc(leap_ctx *c, const float *qrot, const float *kc, const float *vc,
                      float *out, int pos0, int n_tok) {
    if (c->hd != kTcHd) {
        set_error("tensor-core prefill handles head_dim 128");
        return LEAP_ERR_INVALID;
    }
    TcArgs a;
    a.qrot = qrot;
    a.kc = kc;
    a.vc = vc;
    a.head_stride = c->head_stride;
    a.out = out;
    a.err = c->d_err;
    a.pos0 = pos0;
    a.n_tok = n_tok;
    a.n_heads = c->n_heads;
    a.scale_log2 = kLog2e / sqrtf(float(kTcHd));
    switch (c->group) {
        case 1: return launch_tc_g<1>(c, a);
        case 2: return launch_tc_g<2>(c, a);
        case 4: return launch_tc_g<4>(c, a);
        case 8: return launch_tc_g<8>(c, a);
        default:
            set_error("unsupported kv_mul %d", c->group);
            return LEAP_ERR_INVALID;
    }
}

}  // namespace leap
