// prefill_tc_pipe.cu — causal prefill attention on tcgen05 tensor cores,
// 3xTF32, software-pipelined across three roles.
//
// Semantics as prefill_tc.cu (the reference block run for pos0..pos0+n-1 in
// order, src/inference/FloatTransformer.cpp:404-662 and main.cpp:80-89):
// the append kernel has rotated q into `qrot` and written the chunk's rotated
// k and raw v into the cache.  This kernel overlaps the three kinds of work
// that prefill_tc.cu runs one after another for every key tile:
//
//   warps 0-3  (128 threads, TMEM lanes = the CTA's 128 query rows): online
//              softmax of S(j) in FP32 registers, P(j) hi/lo back to TMEM;
//   warps 4-11 (256 threads): convert the FP32 K/V tile j+2 staged by bulk
//              copies into TF32 hi/lo operand tiles (K-major, 128-byte
//              swizzle; V transposed);
//   warp 12    (one elected lane): issue every tcgen05.mma, whichever is
//              ready first (S(j+1) = Q K(j+1)^T runs while the softmax works
//              on S(j); O += P(j) V(j) as soon as P(j) is in TMEM);
//   warp 13    (one elected lane): a staging buffer's next bulk copies as soon
//              as the converters free it (apart from the MMA issue, which
//              blocks while the tensor core's queue is full).
//
// Key tiles are 32 keys so that everything can be double-buffered:
//   TMEM (512 columns): Q hi [0,128) Q lo [128,256) O [256,384)
//                       S/P hi buffer b at 384+64b, P lo at 384+64b+32;
//   shared memory: per buffer b, K hi/lo [32][128] and V^T hi/lo [128][32]
//                  (4 x 16 KB) and FP32 staging K, V [32][128] (2 x 16 KB).
// Products are hi*hi + hi*lo + lo*hi (3xTF32, ~2^-21 relative).  With BFC the
// two correction products (hi*lo, lo*hi) run as BF16 kind::f16 products of
// K = 16 instead (the hi and lo parts rounded to BF16, ~2^-19 relative per
// product, FP32's exponent range): 40 instead of 60 tensor-core instructions
// per 32-key tile, in the same TMEM columns and shared-memory tiles:
//   TMEM: Q hi (TF32) [0,128), Q hi (BF16 pairs) [128,192), Q lo (BF16 pairs)
//         [192,256); P hi (TF32) over S, P hi | P lo (BF16 pairs) at +32 / +48;
//   K operands: hi (TF32, 16 KB), hi (BF16, 8 KB), lo (BF16, 8 KB);
//   V^T operands: hi (TF32, 16 KB), hi | lo (BF16) in the two halves of each
//         128-byte row (16 KB).
// The running max moves only when a row's max grows by more than 2^8 (see
// prefill_tc.cu).
// All hand-offs are mbarriers; every wait is bounded and a timeout sets the
// error word after draining what is in flight.
#include "common.cuh"
#include "ctx.h"
#include "tc.cuh"

namespace leap {
namespace {

constexpr int kPRows = 128;                  // query rows per CTA = TMEM lanes
constexpr int kPKeys = 32;                   // keys per tile
constexpr int kPHd = 128;
constexpr int kPConv = 8;                    // converter warps
constexpr int kPThreads = 32 * (4 + kPConv + 2);  // softmax, convert, MMA, copy warps
constexpr uint32_t kPColQhi = 0, kPColQlo = 128, kPColO = 256, kPColS = 384;
constexpr uint32_t kPTmemCols = 512;
constexpr float kPMaxLag = 8.0f;

// shared memory (bytes from a 1024-aligned base), buffer b = 0/1
constexpr uint32_t kPOpBytes = kPKeys * kPHd * 4;             // 16 KB: one operand tile
__host__ __device__ constexpr uint32_t kPOffKhi(int b) { return uint32_t(b) * 4 * kPOpBytes; }
__host__ __device__ constexpr uint32_t kPOffKlo(int b) { return kPOffKhi(b) + kPOpBytes; }
__host__ __device__ constexpr uint32_t kPOffVThi(int b) { return kPOffKhi(b) + 2 * kPOpBytes; }
__host__ __device__ constexpr uint32_t kPOffVTlo(int b) { return kPOffKhi(b) + 3 * kPOpBytes; }
__host__ __device__ constexpr uint32_t kPOffStK(int b) { return 8 * kPOpBytes + uint32_t(b) * 2 * kPOpBytes; }
__host__ __device__ constexpr uint32_t kPOffStV(int b) { return kPOffStK(b) + kPOpBytes; }
constexpr uint32_t kPSmemUsed = 12 * kPOpBytes;               // 192 KB
constexpr size_t kPSmem = kPSmemUsed + 1024;

struct PArgs {
    const float *qrot;   // [n_tok][n_heads][128], rotated
    const float *kc;     // kv head 0 of (slot, layer); heads head_stride apart
    const float *vc;
    size_t head_stride;
    float *out;          // [n_tok][n_heads][128]
    int *err;
    int pos0, n_tok, n_heads;
    float scale_log2;
};

struct PBars {
    uint64_t q_ready;        // Q hi/lo in TMEM (4 softmax warps)
    uint64_t st_full[2];     // staging b holds tile j (bulk-copy bytes)
    uint64_t st_empty[2];    // converters done with staging b (4 warps)
    uint64_t k_full[2];      // K operand tiles b hold tile j (converter warps)
    uint64_t v_full[2];      // V^T operand tiles b hold tile j (converter warps)
    uint64_t ph_free[2];     // PV(j)'s P-hi terms done: S columns of buffer b free (commit)
    uint64_t op_empty[2];    // PV(j) done: V operands b and S/P buffer b free (commit)
    uint64_t s_full[2];      // S(j) done (commit)
    uint64_t p_full[2];      // P(j) in TMEM, O rescaled if needed (4 warps)
};

__device__ __forceinline__ uint32_t par(int j) { return uint32_t(j >> 1) & 1u; }

template <int G, bool BFC>
__global__ void __launch_bounds__(kPThreads, 1) prefill_tc_pipe_kernel(const PArgs a) {
    constexpr int BT = kPRows / G;  // tokens per CTA
    extern __shared__ unsigned char smem_raw[];
    __shared__ PBars bars;
    __shared__ uint32_t tmem_base_sh;
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    unsigned char *base = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_addr(base);

    // Blocks are dispatched in linear order (x fastest): x = kv head, y = the
    // query block counted from the end, so the whole grid runs longest-first.
    const int kvh = blockIdx.x;
    const int t0 = (gridDim.y - 1 - blockIdx.y) * BT;
    const int t_last = min(t0 + BT, a.n_tok) - 1;
    const int kv_end = a.pos0 + t_last + 1;
    const int n_kt = (kv_end + kPKeys - 1) / kPKeys;
    const float *gK = a.kc + size_t(kvh) * a.head_stride;
    const float *gV = a.vc + size_t(kvh) * a.head_stride;

    if (tid == 0) {
        mbar_init(&bars.q_ready, 4);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars.st_full[b], 1);
            mbar_init(&bars.st_empty[b], kPConv);
            mbar_init(&bars.k_full[b], kPConv);
            mbar_init(&bars.v_full[b], kPConv);
            mbar_init(&bars.ph_free[b], 1);
            mbar_init(&bars.op_empty[b], 1);
            mbar_init(&bars.s_full[b], 1);
            mbar_init(&bars.p_full[b], 4);
        }
        s_fail = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        tc::alloc(&tmem_base_sh, kPTmemCols);
        tc::relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_base_sh;

    if (warp < 4) {
        // ================= softmax warps: row `tid` of the CTA =================
        const uint32_t lane_off = uint32_t(warp * 32) << 16;
        const int my_tok = t0 + tid / G;
        const int my_head = kvh * G + tid % G;
        const int qp = a.pos0 + my_tok;
        const bool row_valid = my_tok < a.n_tok;
        {
            const float *qrow = a.qrot + (size_t(my_tok) * a.n_heads + my_head) * kPHd;
            // The row's four 128-byte lines are requested into L1 at once, so
            // only the first chunk below waits a full round trip.
            if (row_valid) {
#pragma unroll
                for (int c = 0; c < kPHd / 32; ++c)
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(qrow + 32 * c));
            }
#pragma unroll 1
            for (int c = 0; c < kPHd / 32; ++c) {
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
                tc::st32(tmem + lane_off + kPColQhi + 32 * c, hi);
                if (BFC) {
                    uint32_t h16[16], l16[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        h16[i] = tc::pack_bf16x2(hi[2 * i], hi[2 * i + 1]);
                        l16[i] = tc::pack_bf16x2(lo[2 * i], lo[2 * i + 1]);
                    }
                    tc::st16u(tmem + lane_off + kPColQlo + 16 * c, h16);
                    tc::st16u(tmem + lane_off + kPColQlo + 64 + 16 * c, l16);
                } else {
                    tc::st32(tmem + lane_off + kPColQlo + 32 * c, lo);
                }
            }
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.q_ready);
        }
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < n_kt && ok; ++j) {
            const int b = j & 1;
            const int k0 = j * kPKeys;
            ok = __all_sync(0xffffffffu, mbar_wait(&bars.s_full[b], par(j)));
            if (!ok) break;
            tc::fence_after_sync();
            const uint32_t scol = kPColS + 64u * b;
            float s[32];
            tc::ld32(tmem + lane_off + scol, s);
            tc::wait_ld();
            // Raw scores; masked keys become -inf.  Only the diagonal tiles
            // (and a last tile past kv_end) mask anything, so a warp whose
            // 32 rows all see the whole tile skips the test.  Max and sum run
            // as four independent chains so the tile is latency-light.
            float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
            if (__all_sync(0xffffffffu, k0 + kPKeys - 1 <= qp && k0 + kPKeys <= kv_end)) {
#pragma unroll
                for (int c = 0; c < 32; ++c) mx[c & 3] = fmaxf(mx[c & 3], s[c]);
            } else {
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const int key = k0 + c;
                    if (!(key <= qp && key < kv_end)) s[c] = -INFINITY;
                    mx[c & 3] = fmaxf(mx[c & 3], s[c]);
                }
            }
            // scale_log2 > 0, so the scaled max is the max of the scaled scores
            const float mt =
                fmaxf(m, fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * a.scale_log2);
            const bool move = (m == -INFINITY) || (mt > m + kPMaxLag);
            const float alpha = move ? ((m == -INFINITY) ? 0.f : fast_exp2(m - mt)) : 1.f;
            if (move) m = mt;
            // Key 0 is in every row's first tile, so m is finite from here
            // on and a masked score gives exp2(-inf) = +0.
            // Key pairs in packed FP32x2 instructions (each half rounded as
            // the scalar fma / add); the four sum chains are the pairs' halves.
            const float2 scl2 = make_float2(a.scale_log2, a.scale_log2);
            const float2 nm2 = make_float2(-m, -m);
            float2 rsp[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
            float phi[32], plo[32];
#pragma unroll
            for (int c2 = 0; c2 < 16; ++c2) {
                const float2 e = __ffma2_rn(make_float2(s[2 * c2], s[2 * c2 + 1]), scl2, nm2);
                const float2 p = make_float2(fast_exp2(e.x), fast_exp2(e.y));
                rsp[c2 & 1] = __fadd2_rn(rsp[c2 & 1], p);
                phi[2 * c2] = tc::tf32_hi(p.x);
                phi[2 * c2 + 1] = tc::tf32_hi(p.y);
                const float2 lo = __fadd2_rn(p, make_float2(-phi[2 * c2], -phi[2 * c2 + 1]));
                plo[2 * c2] = lo.x;
                plo[2 * c2 + 1] = lo.y;
            }
            l = l * alpha + ((rsp[0].x + rsp[0].y) + (rsp[1].x + rsp[1].y));
            tc::st32(tmem + lane_off + scol, phi);
            if (BFC) {
                float p16[32];  // BF16 pairs: P hi in cells 0-15, P lo in 16-31
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    p16[i] = __uint_as_float(tc::pack_bf16x2(phi[2 * i], phi[2 * i + 1]));
                    p16[16 + i] = __uint_as_float(tc::pack_bf16x2(plo[2 * i], plo[2 * i + 1]));
                }
                tc::st32(tmem + lane_off + scol + 32, p16);
            } else {
                tc::st32(tmem + lane_off + scol + 32, plo);
            }
            // O holds PV(0..j-1): rescale rows whose max moved, once PV(j-1)
            // has landed (PV(j) is issued only after this warp's arrival below)
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                ok = __all_sync(0xffffffffu, mbar_wait(&bars.op_empty[b ^ 1], par(j - 1)));
                if (!ok) break;
                tc::fence_after_sync();
#pragma unroll 1
                for (int c = 0; c < kPHd / 32; ++c) {
                    float o[32];
                    tc::ld32(tmem + lane_off + kPColO + 32 * c, o);
                    tc::wait_ld();
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= alpha;
                    tc::st32(tmem + lane_off + kPColO + 32 * c, o);
                }
            }
            tc::wait_st();
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.p_full[b]);
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars.op_empty[(n_kt - 1) & 1], par(n_kt - 1)));
        if (ok) {
            tc::fence_after_sync();
            const float inv = 1.f / l;
            float *dst = a.out + (size_t(my_tok) * a.n_heads + my_head) * kPHd;
#pragma unroll 1
            for (int c = 0; c < kPHd / 32; ++c) {
                float o[32];
                tc::ld32(tmem + lane_off + kPColO + 32 * c, o);
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
        } else if (lane == 0) {
            atomicExch(&s_fail, 1);
        }
    } else if (warp < 4 + kPConv) {
        // ================= converter warps: staging -> TF32 hi/lo operands ======
        // K of tile j goes into buffer j%2 as soon as S(j-2) has read that
        // buffer's K, so it overlaps PV(j-2); V waits for PV(j-2).
        const int ct = tid - 128;  // 0 .. 32*kPConv-1
        bool ok = true;
        for (int j = 0; j < n_kt && ok; ++j) {
            const int b = j & 1;
            const int nr = min(kPKeys, kv_end - j * kPKeys);
            ok = mbar_wait(&bars.st_full[b], par(j));
            if (ok && j >= 2) ok = mbar_wait(&bars.s_full[b], par(j - 2));
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            const float *stK = reinterpret_cast<const float *>(base + kPOffStK(b));
            const float *stV = reinterpret_cast<const float *>(base + kPOffStV(b));
#pragma unroll
            for (int i = 0; i < kPKeys * kPHd / 4 / (32 * kPConv); ++i) {  // K: float4s
                const int f = ct + 32 * kPConv * i;
                const int n = f >> 5, d = (f & 31) * 4;
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (n < nr) v = reinterpret_cast<const float4 *>(stK)[f];
                float4 h, w;
                h.x = tc::tf32_hi(v.x); w.x = v.x - h.x;
                h.y = tc::tf32_hi(v.y); w.y = v.y - h.y;
                h.z = tc::tf32_hi(v.z); w.z = v.z - h.z;
                h.w = tc::tf32_hi(v.w); w.w = v.w - h.w;
                const uint32_t off = tc::sw128_offset(n, d, kPKeys);
                *reinterpret_cast<float4 *>(base + kPOffKhi(b) + off) = h;
                if (BFC) {
                    const uint32_t o16 = tc::sw128_offset_b16(n, d, kPKeys);
                    *reinterpret_cast<uint2 *>(base + kPOffKlo(b) + o16) =
                        make_uint2(tc::pack_bf16x2(h.x, h.y), tc::pack_bf16x2(h.z, h.w));
                    *reinterpret_cast<uint2 *>(base + kPOffKlo(b) + kPOpBytes / 2 + o16) =
                        make_uint2(tc::pack_bf16x2(w.x, w.y), tc::pack_bf16x2(w.z, w.w));
                } else {
                    *reinterpret_cast<float4 *>(base + kPOffKlo(b) + off) = w;
                }
            }
            fence_proxy_async_smem();  // K operand writes -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.k_full[b]);
            if (j >= 2) ok = __all_sync(0xffffffffu, mbar_wait(&bars.op_empty[b], par(j - 2)));
            if (!ok) break;
            {
                // V^T row d, a 1/kVParts share of its keys per thread
                constexpr int kVParts = 32 * kPConv / kPHd;
                constexpr int kVGroups = kPKeys / 4 / kVParts;
                const int d = ct % kPHd;
                const int jg0 = (ct / kPHd) * kVGroups;
#pragma unroll
                for (int jg = jg0; jg < jg0 + kVGroups; ++jg) {
                    float x[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int n = 4 * jg + e;
                        x[e] = (n < nr) ? stV[n * kPHd + d] : 0.f;
                    }
                    float4 h, w;
                    h.x = tc::tf32_hi(x[0]); w.x = x[0] - h.x;
                    h.y = tc::tf32_hi(x[1]); w.y = x[1] - h.y;
                    h.z = tc::tf32_hi(x[2]); w.z = x[2] - h.z;
                    h.w = tc::tf32_hi(x[3]); w.w = x[3] - h.w;
                    const uint32_t off = tc::sw128_offset(d, 4 * jg, kPHd);
                    *reinterpret_cast<float4 *>(base + kPOffVThi(b) + off) = h;
                    if (BFC) {
                        // keys 0-31 of row d: hi in bytes 0-63, lo in 64-127
                        *reinterpret_cast<uint2 *>(base + kPOffVTlo(b) +
                                                   tc::sw128_offset_b16(d, 4 * jg, kPHd)) =
                            make_uint2(tc::pack_bf16x2(h.x, h.y), tc::pack_bf16x2(h.z, h.w));
                        *reinterpret_cast<uint2 *>(base + kPOffVTlo(b) +
                                                   tc::sw128_offset_b16(d, kPKeys + 4 * jg, kPHd)) =
                            make_uint2(tc::pack_bf16x2(w.x, w.y), tc::pack_bf16x2(w.z, w.w));
                    } else {
                        *reinterpret_cast<float4 *>(base + kPOffVTlo(b) + off) = w;
                    }
                }
            }
            fence_proxy_async_smem();  // V operand writes -> visible to the tensor core
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&bars.st_empty[b]);
                mbar_arrive(&bars.v_full[b]);
            }
        }
        if (!ok && lane == 0) atomicExch(&s_fail, 1);
    } else if (warp == 4 + kPConv + 1) {
        // ================= copy producer: staging buffer j%2 <- tile j =========
        // Tile j+2 is requested the moment the converters have taken tile j.
        const bool leader = tc::elect_one_sync();
        bool ok = true;
        int staged = 0;
        for (; staged < n_kt; ++staged) {
            const int j = staged, b = j & 1;
            if (j >= 2) ok = __all_sync(0xffffffffu, mbar_wait(&bars.st_empty[b], par(j - 2)));
            if (!ok) break;
            const int k0 = j * kPKeys;
            const uint32_t bytes = uint32_t(min(kPKeys, kv_end - k0)) * kPHd * 4;
            if (leader) {
                mbar_arrive_expect_tx(&bars.st_full[b], 2 * bytes);
                bulk_g2s(base + kPOffStK(b), gK + size_t(k0) * kPHd, bytes, &bars.st_full[b]);
                bulk_g2s(base + kPOffStV(b), gV + size_t(k0) * kPHd, bytes, &bars.st_full[b]);
            }
            __syncwarp();
        }
        if (!ok && leader) atomicExch(&s_fail, 1);
        // the last copy into each buffer has landed before shared memory goes
        for (int b = 0; b < 2; ++b) {
            const int lt = staged - 1 - ((staged - 1 - b) & 1);
            if (lt >= 0) (void)mbar_wait(&bars.st_full[b], par(lt));
        }
    } else {  // warp 4 + kPConv
        // ================= MMA issuer ==========================================
        // The whole warp runs the schedule (waits are warp-uniform); one
        // elected lane issues, with descriptors precomputed per buffer.
        const bool leader = tc::elect_one_sync();
        auto wait_all = [&](uint64_t *bar, uint32_t parity) {
            return __all_sync(0xffffffffu, mbar_wait(bar, parity));
        };
        const uint32_t idesc_s = tc::idesc_tf32(kPRows, kPKeys);
        const uint32_t idesc_o = tc::idesc_tf32(kPRows, kPHd);
        const uint32_t idesc_s16 = tc::idesc_bf16(kPRows, kPKeys);
        const uint32_t idesc_o16 = tc::idesc_bf16(kPRows, kPHd);
        const uint64_t dkhi[2] = {tc::sw128_kmajor_desc(sbase + kPOffKhi(0)),
                                  tc::sw128_kmajor_desc(sbase + kPOffKhi(1))};
        const uint64_t dvhi[2] = {tc::sw128_kmajor_desc(sbase + kPOffVThi(0)),
                                  tc::sw128_kmajor_desc(sbase + kPOffVThi(1))};
        constexpr uint64_t kLoStep = kPOpBytes >> 4;  // hi -> lo tile of the same buffer
        int s_issued = 0, pv_issued = 0;
        bool ok = wait_all(&bars.q_ready, 0);
        auto issue_s = [&](int j) {  // S(j) = Qhi Khi + Qhi Klo + Qlo Khi  (M 128, N 32, K 128)
            const int b = j & 1;
            const uint32_t scol = kPColS + 64u * b;
            const uint64_t dk = b ? dkhi[1] : dkhi[0];
            if (leader) {
                if (BFC) {
#pragma unroll
                    for (int kk = 0; kk < kPHd / 8; ++kk)  // Qhi Khi, TF32, K = 8
                        tc::mma_tf32_ts(tmem + scol, tmem + kPColQhi + 8 * kk,
                                        dk + uint64_t(((kk >> 2) * (kPKeys * 128) + (kk & 3) * 32) >> 4),
                                        idesc_s, kk > 0 ? 1u : 0u);
                    // BF16 K tiles follow the TF32 hi tile: hi at +16 KB, lo at +24 KB
#pragma unroll
                    for (int term = 1; term < 3; ++term) {
#pragma unroll
                        for (int kk = 0; kk < kPHd / 16; ++kk) {  // K = 16 per product
                            const uint64_t bdesc = dk + kLoStep + (term == 1 ? kLoStep / 2 : 0) +
                                uint64_t(((kk >> 2) * (kPKeys * 128) + (kk & 3) * 32) >> 4);
                            // term 1: Qhi Klo; term 2: Qlo Khi (A: BF16 pairs, 8 columns per product)
                            tc::mma_bf16_ts(tmem + scol, tmem + kPColQlo + (term == 2 ? 64 : 0) + 8 * kk,
                                            bdesc, idesc_s16, 1u);
                        }
                    }
                } else {
#pragma unroll
                    for (int term = 0; term < 3; ++term) {
#pragma unroll
                        for (int kk = 0; kk < kPHd / 8; ++kk) {
                            const uint64_t bdesc = dk + (term == 1 ? kLoStep : 0) +
                                                   uint64_t(((kk >> 2) * (kPKeys * 128) + (kk & 3) * 32) >> 4);
                            tc::mma_tf32_ts(tmem + scol, tmem + (term == 2 ? kPColQlo : kPColQhi) + 8 * kk,
                                            bdesc, idesc_s, (term > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                }
                tc::commit(&bars.s_full[b]);
            }
            __syncwarp();
        };
        // O += P(j) V(j): the two terms that read P hi (Phi Vhi, Phi Vlo)
        // first, then Plo Vhi.  The commit between them frees the S columns
        // (where P hi lives) for S(j+2), which then queues on the tensor core
        // behind the P-lo products instead of waiting for the pipe to drain.
        auto issue_pv = [&](int j) {
            const int b = j & 1;
            const uint32_t scol = kPColS + 64u * b;
            const uint64_t dv = b ? dvhi[1] : dvhi[0];
            if (leader) {
                if (BFC) {
#pragma unroll
                    for (int kk = 0; kk < kPKeys / 8; ++kk)  // Phi Vhi, TF32
                        tc::mma_tf32_ts(tmem + kPColO, tmem + scol + 8 * kk, dv + uint64_t(kk * 2),
                                        idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
                    tc::commit(&bars.ph_free[b]);
#pragma unroll
                    for (int term = 1; term < 3; ++term) {
#pragma unroll
                        for (int kk = 0; kk < kPKeys / 16; ++kk) {
                            // term 1: Phi (cells +32) . Vlo (bytes 64-127);
                            // term 2: Plo (cells +48) . Vhi (bytes 0-63)
                            const uint64_t bdesc = dv + kLoStep + uint64_t(((term == 1 ? 64 : 0) + 32 * kk) >> 4);
                            tc::mma_bf16_ts(tmem + kPColO, tmem + scol + (term == 1 ? 32 : 48) + 8 * kk,
                                            bdesc, idesc_o16, 1u);
                        }
                    }
                } else {
#pragma unroll
                    for (int term = 0; term < 3; ++term) {
                        if (term == 2) tc::commit(&bars.ph_free[b]);
#pragma unroll
                        for (int kk = 0; kk < kPKeys / 8; ++kk) {
                            const uint64_t bdesc = dv + (term == 1 ? kLoStep : 0) + uint64_t(kk * 2);
                            tc::mma_tf32_ts(tmem + kPColO, tmem + scol + (term == 2 ? 32 : 0) + 8 * kk,
                                            bdesc, idesc_o, (j > 0 || term > 0 || kk > 0) ? 1u : 0u);
                        }
                    }
                }
                tc::commit(&bars.op_empty[b]);
            }
            __syncwarp();
        };
        // Issue whichever step is ready: S(j) once tile j's K operands are
        // converted and PV(j-2)'s P-hi terms have released buffer j%2's S
        // columns; PV(j) once the softmax has written P(j) and tile j's V
        // operands are converted.  Every test is of the next phase of its
        // barrier only (the one before it was observed), so parities cannot
        // alias.  No progress for kMaxWaitNs ends the loop.
        unsigned long long t_idle = global_ns();
        uint32_t idle_polls = 0;
        while (ok && pv_issued < n_kt) {
            bool progress = false;
            if (s_issued < n_kt && s_issued <= pv_issued + 1) {
                const int j = s_issued, b = j & 1;
                bool ready = mbar_test(&bars.k_full[b], par(j));
                if (ready && j >= 2) ready = mbar_test(&bars.ph_free[b], par(j - 2));
                if (__all_sync(0xffffffffu, ready)) {
                    tc::fence_after_sync();
                    issue_s(j);
                    ++s_issued;
                    progress = true;
                }
            }
            if (pv_issued < s_issued) {
                const int j = pv_issued;
                if (__all_sync(0xffffffffu, mbar_test(&bars.p_full[j & 1], par(j)) &&
                                                mbar_test(&bars.v_full[j & 1], par(j)))) {
                    tc::fence_after_sync();
                    issue_pv(j);
                    ++pv_issued;
                    progress = true;
                }
            }
            if (progress) {
                idle_polls = 0;
            } else if ((++idle_polls & 255) == 0) {
                const unsigned long long t = global_ns();
                if (idle_polls == 256) t_idle = t;
                else if (t - t_idle > kMaxWaitNs || idle_polls >= kMaxWaitPolls) ok = false;
            }
        }
        if (!ok && leader) atomicExch(&s_fail, 1);
        // nothing may still be in flight when the CTA releases TMEM and shared
        // memory: wait (bounded) for the last operation on every barrier
        for (int b = 0; b < 2; ++b) {
            const int ls = s_issued - 1 - ((s_issued - 1 - b) & 1);      // last S into b
            if (ls >= 0) (void)mbar_wait(&bars.s_full[b], par(ls));
            const int lp = pv_issued - 1 - ((pv_issued - 1 - b) & 1);    // last PV on b
            if (lp >= 0) (void)mbar_wait(&bars.ph_free[b], par(lp));
            if (lp >= 0) (void)mbar_wait(&bars.op_empty[b], par(lp));
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0 && s_fail) report_error(a.err, kDevWaitTimeout);
    if (warp == 0) tc::dealloc(tmem, kPTmemCols);
}

template <int G, bool BFC>
int launch_pipe_g(leap_ctx *c, const PArgs &a) {
    const void *fn = reinterpret_cast<const void *>(prefill_tc_pipe_kernel<G, BFC>);
    if (const int st = set_kernel_smem(fn, kPSmem, "cudaFuncSetAttribute(prefill_tc_pipe)")) return st;
    constexpr int BT = kPRows / G;
    dim3 grid(c->n_kv, (a.n_tok + BT - 1) / BT);
    prefill_tc_pipe_kernel<G, BFC><<<grid, kPThreads, kPSmem, c->stream>>>(a);
    return cuda_status(cudaGetLastError(), "prefill_tc_pipe_kernel launch");
}

}  // namespace

int launch_prefill_tc_pipe(leap_ctx *c, const float *qrot, const float *kc, const float *vc,
                           float *out, int pos0, int n_tok, bool bf16_corrections) {
    if (c->hd != kPHd) {
        set_error("tensor-core prefill handles head_dim 128");
        return LEAP_ERR_INVALID;
    }
    PArgs a;
    a.qrot = qrot;
    a.kc = kc;
    a.vc = vc;
    a.head_stride = c->head_stride;
    a.out = out;
    a.err = c->d_err;
    a.pos0 = pos0;
    a.n_tok = n_tok;
    a.n_heads = c->n_heads;
    a.scale_log2 = kLog2e / sqrtf(float(kPHd));
    switch (c->group * 2 + (bf16_corrections ? 1 : 0)) {
        case 2: return launch_pipe_g<1, false>(c, a);
        case 3: return launch_pipe_g<1, true>(c, a);
        case 4: return launch_pipe_g<2, false>(c, a);
        case 5: return launch_pipe_g<2, true>(c, a);
        case 8: return launch_pipe_g<4, false>(c, a);
        case 9: return launch_pipe_g<4, true>(c, a);
        case 16: return launch_pipe_g<8, false>(c, a);
        case 17: return launch_pipe_g<8, true>(c, a);
        default:
            set_error("unsupported kv_mul %d", c->group);
            return LEAP_ERR_INVALID;
    }
}

}  // namespace leap
