// decode_attn.cu — fused RoPE + KV append + split-KV GQA decode attention.
//
// Replaces the reference's attention block (src/inference/
// FloatTransformer.cpp:404-662, twin QuantizedTransformer.cpp:680-923):
//   * RoPE of q (all heads) and of the new k row  (:404-494)
//   * the new rotated k and raw v written into cache row `pos` (:397-402)
//   * scores q.k * 1/sqrt(hd) over rows 0..pos   (:497-630)
//   * softmax (:632, :216-238) and the weighted V sum (:634-661).
//
// Design (HBM-bound, CUDA cores, no tensor cores):
//   * one CTA per (sequence, split of the context, kv head); the CTA packs
//     the kv_mul query heads that share that kv head, so every K/V byte
//     crosses HBM once (the reference re-reads K/V once per query head);
//   * K and V tiles of 16 KB each move global -> shared with 1-D bulk
//     copies (TMA engine) into a 3-stage mbarrier pipeline; the cache is
//     head-major, so a tile of positions is one contiguous range;
//   * a row of K/V is read by a group of LPR lanes, each holding a slice
//     of dims for all G query heads; scores are reduced with xor-shuffles;
//   * online softmax per lane group, merged across groups in shared memory;
//   * splits of one (sequence, kv head) are combined by the CTA that
//     finishes last (atomic ticket), so there is no second launch.
#include <cfloat>
#include <cstdio>

#include "common.cuh"
#include "ctx.h"

namespace leap {
namespace {

// CTA shapes (SH), three stages of K+V tiles each:
//   0: 128 threads, 16 KB tiles, two CTAs per SM;
//   1: 256 threads, 32 KB tiles, one CTA per SM (half as many splits).
constexpr int kStages = 3;
constexpr int kEarlyStages = 2;  // stages filled before the dependency wait
constexpr int kMaxSplitsPerSeq = 256;
constexpr float kRescaleLog2 = 8.f;  // see the online softmax in the tile loop

template <int HD, int G, int SH>
struct Cfg {
    static constexpr int THREADS = SH == 0 ? 128 : 256;
    static constexpr int MINB = SH == 1 ? 1 : 2;     // resident CTAs per SM
    static constexpr int WARPS = THREADS / 32;
    static constexpr int TILE_BYTES = SH == 1 ? 32768 : 16384;  // per tensor per stage
    static constexpr int kLpr0 = G * HD / 64;
    static constexpr int LPR = kLpr0 < 8 ? 8 : (kLpr0 > 32 ? 32 : kLpr0);
    static constexpr int RPW = 32 / LPR;             // rows per warp pass
    static constexpr int NGRP = WARPS * RPW;        // row groups per CTA
    static constexpr int DPL = HD / LPR;             // dims per lane
    static constexpr int C4 = DPL / 4;               // float4 chunks per lane
    static constexpr int TILE = TILE_BYTES / (HD * 4);
    static constexpr int RPG = TILE / NGRP;          // rows per group per tile
    static constexpr int NV4 = G * HD / 4;           // float4 outputs per CTA
    static constexpr int MLS = 2 * (G < 2 ? 2 : G);  // floats per split's (M, L) record
    static constexpr size_t kSmem = size_t(2) * kStages * TILE * HD * sizeof(float);
    static_assert(DPL % 4 == 0 && C4 >= 1, "lane slice must be float4s");
    static_assert(TILE % NGRP == 0, "tile rows must split over groups");
    // CTA merge buffer [NGRP][G][HD] and combine tables reuse the stages
    static_assert(size_t(NGRP) * G * HD * sizeof(float) <= kSmem, "merge smem");
    // combine staging: (M, L) table + weights + at least one partial
    static_assert((size_t(kMaxSplitsPerSeq) * (MLS + G) + G * HD) * sizeof(float) <= kSmem,
                  "combine smem");
};

struct DecodeArgs {
    const float *q;      // [n_seq][n_kv*G][HD]
    const float *k_new;  // [n_seq][n_kv][HD]
    const float *v_new;
    float *out;          // [n_seq][n_kv*G][HD]
    float *k_cache;
    float *v_cache;
    const float *rope_cos;  // [max_seq][HD/2]
    const float *rope_sin;
    size_t head_stride, layer_off, slot_stride;  // floats
    float *part_o;       // [parts][G*HD]
    float *part_ml;      // [parts][MLS]: (M, L) per head, padded to 16 bytes
    unsigned *counters;  // [kMaxSeqPerLaunch][n_kv]
    int *err;
    int *err_host;       // non-null: error codes also go to this host-mapped word
    int n_kv;
    float scale_log2;    // log2(e) / sqrt(HD)
};

// TAIL: the last CTA of a (sequence, kv head) combines its splits (ticket);
// otherwise every CTA only publishes its partial and decode_combine_kernel,
// launched right after, combines them.
template <int HD, int G, int SH, bool TAIL>
__global__ void __launch_bounds__(Cfg<HD, G, SH>::THREADS, Cfg<HD, G, SH>::MINB)
decode_attn_kernel(const DecodeArgs a, const DecodeSeq tab) {
    using C = Cfg<HD, G, SH>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float *sK = reinterpret_cast<float *>(smem_raw);      // [kStages][TILE][HD]
    float *sV = sK + kStages * C::TILE * HD;
    __shared__ uint64_t full_bar[kStages];
    __shared__ float red_m[C::NGRP][G], red_l[C::NGRP][G];
    __shared__ uint64_t comb_bar, comb_bar_o;  // (M, L) table; partial outputs
    __shared__ int s_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int j = lane % C::LPR;                   // lane within its row group
    const int grp = warp * C::RPW + lane / C::LPR;  // row group

    // ---- which (sequence, split, kv head) ---------------------------------
    // One sequence: blocks are handed out in linear order, and the last few
    // start only once the previous kernel's combining CTAs leave their SMs
    // (with no tiles staged before the dependency wait).  So the linear order
    // is remapped to put every kv head's last split, the short one, at the
    // end: the late blocks get the least work (14.996 -> 14.85 us per launch
    // at ctx 8192).  Batches keep (split, kv head) = (x, y).
    int bx = blockIdx.x;
    int kvh_sel = blockIdx.y;
    if (tab.n_seq == 1) {
        const int T = gridDim.x;
        const int b = blockIdx.y * T + blockIdx.x;
        const int n_full = gridDim.y * (T - 1);  // blocks of the non-last splits
        if (b >= n_full) {
            bx = T - 1;
            kvh_sel = b - n_full;
        } else {
            bx = b % (T - 1);
            kvh_sel = b / (T - 1);
        }
    }
    int lo = 0, hi = tab.n_seq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tab.split0[mid] <= bx) lo = mid; else hi = mid - 1;
    }
    const int seq = lo;
    const int split = bx - tab.split0[seq];
    const int nsplit = tab.split0[seq + 1] - tab.split0[seq];
    const int kvh = kvh_sel;
    const int pos = tab.pos[seq];
    const int row_begin = split * tab.chunk;
    const int row_end = min(row_begin + tab.chunk, pos + 1);
    const int n_tiles = (row_end - row_begin + C::TILE - 1) / C::TILE;
    const bool last_split = (split == nsplit - 1);

    const size_t head_off = size_t(tab.slot[seq]) * a.slot_stride + a.layer_off +
                            size_t(kvh) * a.head_stride;
    float *gK = a.k_cache + head_off;
    float *gV = a.v_cache + head_off;

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&full_bar[s], 1);
        mbar_init(&comb_bar, 1);
        mbar_init(&comb_bar_o, 1);
        fence_mbar_init();
    }
    __syncthreads();

    // Stage the first tiles: kEarlyStages of them before the dependency wait
    // (they overlap the previous kernel's tail), the rest after it.  Filling
    // every stage early was measured slower: those copies compete with the
    // previous kernel's split-KV combine, which is on the critical path.
    auto stage_tile = [&](int t) {
        const int r0 = row_begin + t * C::TILE;
        const uint32_t bytes = min(C::TILE, row_end - r0) * HD * 4;
        mbar_arrive_expect_tx(&full_bar[t % kStages], 2 * bytes);
        bulk_g2s(sK + (t % kStages) * C::TILE * HD, gK + size_t(r0) * HD, bytes,
                 &full_bar[t % kStages]);
        bulk_g2s(sV + (t % kStages) * C::TILE * HD, gV + size_t(r0) * HD, bytes,
                 &full_bar[t % kStages]);
    };
    if (tid == 0)
        for (int t = 0; t < min(kEarlyStages, n_tiles); ++t) stage_tile(t);
    // Up to here only this layer's cache rows were read, which the previous
    // kernel of the stream never writes (the host launches with overlap only
    // then).  Inputs, scratch and outputs may still be in use by it.
    grid_dependency_wait();
    grid_launch_dependents();
    if (tid == 0)
        for (int t = kEarlyStages; t < min(kStages, n_tiles); ++t) stage_tile(t);

    // ---- rotated q slice: heads kvh*G .. +G, dims of this lane's chunks ---
    const int qh0 = kvh * G;
    const float *qs = a.q + (size_t(seq) * a.n_kv * G + qh0) * HD;
    const float *rc = a.rope_cos + size_t(pos) * (HD / 2);
    const float *rs = a.rope_sin + size_t(pos) * (HD / 2);
    float q[G][C::DPL];
#pragma unroll
    for (int i = 0; i < C::C4; ++i) {
        const int c4 = j + C::LPR * i;
        const float2 cc = *reinterpret_cast<const float2 *>(rc + 2 * c4);
        const float2 ss = *reinterpret_cast<const float2 *>(rs + 2 * c4);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float4 x = *reinterpret_cast<const float4 *>(qs + g * HD + 4 * c4);
            const float2 r0 = rope_pair(x.x, x.y, cc.x, ss.x);
            const float2 r1 = rope_pair(x.z, x.w, cc.y, ss.y);
            q[g][4 * i + 0] = r0.x;
            q[g][4 * i + 1] = r0.y;
            q[g][4 * i + 2] = r1.x;
            q[g][4 * i + 3] = r1.y;
        }
    }

    float m[G], l[G], o[G][C::DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < C::DPL; ++d) o[g][d] = 0.f;
    }

    // ---- main loop over tiles --------------------------------------------
    // Tile by tile: wait, scores, softmax update and V sum, then release the
    // stage for the refill.  (Forming the scores of tile t+1 alongside the V
    // sum of tile t was measured slower: at the dependency release every
    // stage is full and no copy is in flight until the first stage is
    // released, so that release must come as early as possible.)

    // Wait (this thread) for tile tt; if it holds row `pos`, rotate k, append
    // k and v to the cache, and patch the staged tile (the copy may have read
    // the old row) — that needs the whole CTA.  False if the wait gave up.
    auto tile_ready = [&](int tt) -> bool {
        bool r = mbar_wait(&full_bar[tt % kStages], (tt / kStages) & 1);
        const int r0 = row_begin + tt * C::TILE;
        if (last_split && pos < r0 + C::TILE) {
            r = __syncthreads_and(r);
            if (!r) return false;
            const int rr = pos - r0;
            float *tK = sK + (tt % kStages) * C::TILE * HD;
            float *tV = sV + (tt % kStages) * C::TILE * HD;
            const float *kn = a.k_new + (size_t(seq) * a.n_kv + kvh) * HD;
            const float *vn = a.v_new + (size_t(seq) * a.n_kv + kvh) * HD;
            for (int d = 2 * tid; d < HD; d += 2 * C::THREADS) {
                const float2 kk = *reinterpret_cast<const float2 *>(kn + d);
                const float2 vv = *reinterpret_cast<const float2 *>(vn + d);
                const float2 kr = rope_pair(kk.x, kk.y, rc[d / 2], rs[d / 2]);
                *reinterpret_cast<float2 *>(tK + rr * HD + d) = kr;
                *reinterpret_cast<float2 *>(tV + rr * HD + d) = vv;
                *reinterpret_cast<float2 *>(gK + size_t(pos) * HD + d) = kr;
                *reinterpret_cast<float2 *>(gV + size_t(pos) * HD + d) = vv;
            }
            __syncthreads();
        }
        return r;
    };

    // Scaled scores (log2 units) of this lane group's rows of tile tt;
    // -inf beyond the split.
    auto tile_scores = [&](int tt, float (&sc)[C::RPG][G]) {
        const int r0 = row_begin + tt * C::TILE;
        const float *tK = sK + (tt % kStages) * C::TILE * HD;
#pragma unroll
        for (int rr = 0; rr < C::RPG; ++rr) {
            const int row = rr * C::NGRP + grp;
            const bool valid = (r0 + row) < row_end;
            float acc[G];
#pragma unroll
            for (int g = 0; g < G; ++g) acc[g] = 0.f;
            if (valid) {
                const float *kr = tK + row * HD;
#pragma unroll
                for (int i = 0; i < C::C4; ++i) {
                    const float4 kk =
                        *reinterpret_cast<const float4 *>(kr + 4 * (j + C::LPR * i));
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        acc[g] = fmaf(q[g][4 * i + 0], kk.x, acc[g]);
                        acc[g] = fmaf(q[g][4 * i + 1], kk.y, acc[g]);
                        acc[g] = fmaf(q[g][4 * i + 2], kk.z, acc[g]);
                        acc[g] = fmaf(q[g][4 * i + 3], kk.w, acc[g]);
                    }
                }
            }
#pragma unroll
            for (int off = C::LPR / 2; off >= 1; off >>= 1) {
#pragma unroll
                for (int g = 0; g < G; ++g)
                    acc[g] += __shfl_xor_sync(0xffffffffu, acc[g], off);
            }
#pragma unroll
            for (int g = 0; g < G; ++g) sc[rr][g] = valid ? acc[g] * a.scale_log2 : -INFINITY;
        }
    };

    // Online softmax update and weighted V sum of tile tt.  The running max m
    // (log2 units) is a lazily moved reference: it moves, and l and o are
    // rescaled, only when a score exceeds it by more than kRescaleLog2, so
    // p = 2^(s - m) <= 2^8.  Exact in real arithmetic; after the first tile
    // it is rarely taken.
    auto tile_accumulate = [&](int tt, const float (&sc)[C::RPG][G]) {
        const int r0 = row_begin + tt * C::TILE;
        const float *tV = sV + (tt % kStages) * C::TILE * HD;
        float mt[G];
        bool grow = false;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            mt[g] = sc[0][g];
#pragma unroll
            for (int rr = 1; rr < C::RPG; ++rr) mt[g] = fmaxf(mt[g], sc[rr][g]);
            grow |= mt[g] > m[g] + kRescaleLog2;
        }
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float mn = fmaxf(m[g], mt[g]);
                const float alpha = (mn == -INFINITY) ? 1.f : fast_exp2(m[g] - mn);
                m[g] = mn;
                l[g] *= alpha;
#pragma unroll
                for (int d = 0; d < C::DPL; ++d) o[g][d] *= alpha;
            }
        }
#pragma unroll
        for (int rr = 0; rr < C::RPG; ++rr) {
            const int row = rr * C::NGRP + grp;
            if ((r0 + row) < row_end) {
                float p[G];
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    p[g] = fast_exp2(sc[rr][g] - m[g]);
                    l[g] += p[g];
                }
                const float *vr = tV + row * HD;
#pragma unroll
                for (int i = 0; i < C::C4; ++i) {
                    const float4 vv =
                        *reinterpret_cast<const float4 *>(vr + 4 * (j + C::LPR * i));
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        o[g][4 * i + 0] = fmaf(p[g], vv.x, o[g][4 * i + 0]);
                        o[g][4 * i + 1] = fmaf(p[g], vv.y, o[g][4 * i + 1]);
                        o[g][4 * i + 2] = fmaf(p[g], vv.z, o[g][4 * i + 2]);
                        o[g][4 * i + 3] = fmaf(p[g], vv.w, o[g][4 * i + 3]);
                    }
                }
            }
        }
    };

    int failed = -1;  // the tile whose wait gave up
    for (int t = 0; t < n_tiles; ++t) {
        const bool landed = tile_ready(t);
        float sc[C::RPG][G];
        tile_scores(t, sc);
        tile_accumulate(t, sc);
        // One CTA barrier per tile: every warp is done with the stage (refill
        // it), and a wait that gave up in any thread ends the loop for all
        // (that tile's values are discarded; its shared reads stayed in
        // bounds).
        if (__syncthreads_or(!landed)) {
            failed = t;
            break;
        }
        if (tid == 0 && t + kStages < n_tiles) stage_tile(t + kStages);
    }

    if (failed >= 0) {
        // A wait gave up: give the copies still in flight a bounded chance
        // to land before this CTA's shared memory is released, then report.
        for (int tt = failed + 1; tt < min(failed + kStages, n_tiles); ++tt)
            (void)mbar_wait(&full_bar[tt % kStages], (tt / kStages) & 1);
        if (tid == 0) report_error(a.err, a.err_host, kDevWaitTimeout);
        return;
    }

    // ---- merge the row groups of this CTA ---------------------------------
    // Each row group stores its raw (m, l, o); every output thread then forms
    // its head's M (max), L and the groups' scale factors itself, L summed in
    // the order of a 32-lane xor butterfly (lanes >= NGRP adding zeros).  One
    // barrier instead of three, and the same bits as a per-head warp
    // reduction with shuffles (14.94 -> 14.77 us per launch at ctx 8192).
    if (j == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            red_m[grp][g] = m[g];
            red_l[grp][g] = l[g];
        }
    }
    float *red_o = sK;  // [NGRP][G][HD]; every warp is done with the stages
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int i = 0; i < C::C4; ++i) {
            const float4 v = make_float4(o[g][4 * i + 0], o[g][4 * i + 1], o[g][4 * i + 2],
                                         o[g][4 * i + 3]);
            *reinterpret_cast<float4 *>(red_o + (grp * G + g) * HD + 4 * (j + C::LPR * i)) = v;
        }
    }
    __syncthreads();

    float *out_seq = a.out + (size_t(seq) * a.n_kv * G + qh0) * HD;
    // Partials of one (sequence, kv head) are contiguous, so the combining
    // CTA fetches them with one bulk copy: index kvh * total + split0 + split.
    const int pfirst = kvh * tab.split0[tab.n_seq] + tab.split0[seq];
    const int pidx = pfirst + split;
    static_assert(C::NGRP <= 32, "butterfly over 32 lanes");
    for (int e = tid; e < C::NV4; e += C::THREADS) {
        const int g = (4 * e) / HD;
        float f[C::NGRP];
        float M = -INFINITY;
#pragma unroll
        for (int k = 0; k < C::NGRP; ++k) {
            f[k] = red_m[k][g];
            M = fmaxf(M, f[k]);
        }
#pragma unroll
        for (int k = 0; k < C::NGRP; ++k) f[k] = (f[k] == -INFINITY) ? 0.f : fast_exp2(f[k] - M);
        float t[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            const int kk = k < C::NGRP ? k : 0;  // in-bounds index; the term is 0 beyond NGRP
            t[k] = k < C::NGRP ? __fmul_rn(red_l[kk][g], f[kk]) : 0.f;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
            for (int k = 0; k < off; ++k) t[k] = __fadd_rn(t[k], t[k + off]);
        }
        const float L = t[0];
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int gg = 0; gg < C::NGRP; ++gg) {
            const float4 v = *reinterpret_cast<const float4 *>(red_o + gg * G * HD + 4 * e);
            acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, f[gg]));
            acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, f[gg]));
            acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, f[gg]));
            acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, f[gg]));
        }
        if (nsplit == 1) {
            const float inv = 1.f / L;
            acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
            *reinterpret_cast<float4 *>(out_seq + 4 * e) = acc;
        } else {
            *reinterpret_cast<float4 *>(a.part_o + size_t(pidx) * G * HD + 4 * e) = acc;
            if ((4 * e) % HD == 0) {
                a.part_ml[size_t(pidx) * C::MLS + 2 * g + 0] = M;
                a.part_ml[size_t(pidx) * C::MLS + 2 * g + 1] = L;
            }
        }
    }
    if (nsplit == 1) return;

    // ---- split-KV combine by the last CTA of this (sequence, kv head) -----
    if (!TAIL) return;  // decode_combine_kernel takes it from here
    __syncthreads();
    if (tid == 0) {
        // publish this CTA's partial (release, cumulative over the CTA's
        // stores ordered by the barrier) and learn whether it is the last
        fence_proxy_async_global();
        unsigned *cnt = a.counters + seq * a.n_kv + kvh;
        const unsigned ticket = atom_add_acq_rel_gpu(cnt, 1u);
        s_last = (ticket == unsigned(nsplit - 1));
        if (s_last) *cnt = 0u;  // ready for the next launch (stream-ordered)
    }
    __syncthreads();
    if (!s_last) return;

    // Stage the (M, L) table and the partial outputs in shared memory with
    // bulk copies (one round trip per chunk of partials), then combine.
    float *sML = sK;                                     // [nsplit][MLS]
    float *cW = sML + nsplit * C::MLS;                   // [nsplit][G] weights
    float *sO = cW + ((nsplit * G + 3) & ~3);            // [cap][G*HD]
    const int cap = int((C::kSmem / sizeof(float) - size_t(sO - sK)) / (G * HD));
    const int n0 = min(cap, nsplit);
    // The (M, L) table and the partials arrive on separate barriers, so the
    // weights are formed while the partials are still on their way.
    uint32_t cphase = 0;
    if (tid == 0) {
        fence_proxy_async_global();
        const uint32_t ml_bytes = uint32_t(nsplit) * C::MLS * 4;
        const uint32_t o_bytes = uint32_t(n0) * G * HD * 4;
        mbar_arrive_expect_tx(&comb_bar, ml_bytes);
        bulk_g2s(sML, a.part_ml + size_t(pfirst) * C::MLS, ml_bytes, &comb_bar);
        mbar_arrive_expect_tx(&comb_bar_o, o_bytes);
        bulk_g2s(sO, a.part_o + size_t(pfirst) * G * HD, o_bytes, &comb_bar_o);
    }
    bool cok = mbar_wait(&comb_bar, 0);
    cok = __syncthreads_and(cok);
    if (!cok) {
        (void)mbar_wait(&comb_bar_o, 0);  // let the partials' copy land first
        if (tid == 0) report_error(a.err, a.err_host, kDevWaitTimeout);
        return;
    }
    // one warp per head: max, rescaled sum, normalised weights
    for (int g = warp; g < G; g += C::WARPS) {
        float M = -INFINITY;
        for (int sp = lane; sp < nsplit; sp += 32) M = fmaxf(M, sML[sp * C::MLS + 2 * g]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.f;
        for (int sp = lane; sp < nsplit; sp += 32)
            L += sML[sp * C::MLS + 2 * g + 1] * fast_exp2(sML[sp * C::MLS + 2 * g] - M);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        const float inv = 1.f / L;
        for (int sp = lane; sp < nsplit; sp += 32)
            cW[sp * G + g] = fast_exp2(sML[sp * C::MLS + 2 * g] - M) * inv;
    }
    cok = mbar_wait(&comb_bar_o, cphase);  // the first chunk of partials
    cok = __syncthreads_and(cok);  // also: every weight is in cW
    if (!cok) {
        if (tid == 0) report_error(a.err, a.err_host, kDevWaitTimeout);
        return;
    }
    cphase ^= 1u;
    constexpr int kPerThread = (C::NV4 + C::THREADS - 1) / C::THREADS;
    float4 acc[kPerThread];
#pragma unroll
    for (int r = 0; r < kPerThread; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < nsplit; s0 += cap) {
        const int n = min(cap, nsplit - s0);
        if (s0 > 0) {
            __syncthreads();  // every thread is done with the previous chunk
            if (tid == 0) {
                const uint32_t o_bytes = uint32_t(n) * G * HD * 4;
                mbar_arrive_expect_tx(&comb_bar_o, o_bytes);
                bulk_g2s(sO, a.part_o + size_t(pfirst + s0) * G * HD, o_bytes, &comb_bar_o);
            }
            cok = mbar_wait(&comb_bar_o, cphase);
            cok = __syncthreads_and(cok);
            if (!cok) {
                if (tid == 0) report_error(a.err, a.err_host, kDevWaitTimeout);
                return;
            }
            cphase ^= 1u;
        }
#pragma unroll
        for (int r = 0; r < kPerThread; ++r) {
            const int e = tid + r * C::THREADS;
            if (e < C::NV4) {
                const int g = (4 * e) / HD;
#pragma unroll 8
                for (int i = 0; i < n; ++i) {
                    const float w = cW[(s0 + i) * G + g];
                    const float4 v = *reinterpret_cast<const float4 *>(sO + i * G * HD + 4 * e);
                    acc[r].x = fmaf(w, v.x, acc[r].x);
                    acc[r].y = fmaf(w, v.y, acc[r].y);
                    acc[r].z = fmaf(w, v.z, acc[r].z);
                    acc[r].w = fmaf(w, v.w, acc[r].w);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kPerThread; ++r) {
        const int e = tid + r * C::THREADS;
        if (e < C::NV4) *reinterpret_cast<float4 *>(out_seq + 4 * e) = acc[r];
    }
}

// Split-KV combine as its own launch: one CTA of 4 warps per (sequence,
// query head).  Warp 0 forms M (max of the splits' running maxima), L (sum of
// L_s * 2^(M_s - M)) and the weights w_s = 2^(M_s - M) / L into shared
// memory; then warp k sums w_s times the partials of splits s = k, k+4, ...
// (all of its loads in flight at once) and the four sums are added.
// Launched with programmatic serialization right after the attention kernel;
// it waits for it before reading anything, and lets its own successor launch
// first: the successor (the next layer's attention, a GEMV) reads only
// constant data (its K/V cache, weights) before its own griddepcontrol.wait,
// which returns only once this kernel, and so the attention, has completed.
constexpr int kCombWarps = 4;
constexpr int kCombUnroll = 8;

template <int HD, int G>
__global__ void __launch_bounds__(32 * kCombWarps)
decode_combine_kernel(const DecodeArgs a, const DecodeSeq tab) {
    constexpr int MLS = 2 * (G < 2 ? 2 : G);
    constexpr int V4 = HD / 4;  // float4 per head: 32 or 16 lanes busy
    __shared__ float s_w[kMaxSplitsPerSeq];
    __shared__ float4 s_acc[kCombWarps][32];
    grid_launch_dependents();
    grid_dependency_wait();
    const int seq = blockIdx.x, qh = blockIdx.y, kvh = qh / G, g = qh - kvh * G;
    const int nsplit = tab.split0[seq + 1] - tab.split0[seq];
    if (nsplit <= 1) return;  // the attention kernel wrote this output itself
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t pfirst = size_t(kvh) * tab.split0[tab.n_seq] + tab.split0[seq];
    const float *ml = a.part_ml + pfirst * MLS + 2 * g;
    if (warp == 0) {
        float M = -INFINITY;
        for (int sp = lane; sp < nsplit; sp += 32) M = fmaxf(M, ml[size_t(sp) * MLS]);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
        float L = 0.f;
        for (int sp = lane; sp < nsplit; sp += 32)
            L += ml[size_t(sp) * MLS + 1] * fast_exp2(ml[size_t(sp) * MLS] - M);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
        const float inv = 1.f / L;
        for (int sp = lane; sp < nsplit; sp += 32) s_w[sp] = fast_exp2(ml[size_t(sp) * MLS] - M) * inv;
    }
    // the partials do not depend on the weights: start loading them now
    const float *po = a.part_o + pfirst * (G * HD) + g * HD + 4 * (lane < V4 ? lane : 0);
    float4 v[kCombUnroll];
    int sp0 = warp;
#pragma unroll
    for (int u = 0; u < kCombUnroll; ++u) {
        const int sp = sp0 + u * kCombWarps;
        v[u] = sp < nsplit ? *reinterpret_cast<const float4 *>(po + size_t(sp) * (G * HD))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    __syncthreads();
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (;;) {
#pragma unroll
        for (int u = 0; u < kCombUnroll; ++u) {
            const int sp = sp0 + u * kCombWarps;
            if (sp < nsplit) {
                const float w = s_w[sp];
                acc.x = fmaf(w, v[u].x, acc.x);
                acc.y = fmaf(w, v[u].y, acc.y);
                acc.z = fmaf(w, v[u].z, acc.z);
                acc.w = fmaf(w, v[u].w, acc.w);
            }
        }
        sp0 += kCombUnroll * kCombWarps;
        if (sp0 >= nsplit) break;
#pragma unroll
        for (int u = 0; u < kCombUnroll; ++u) {
            const int sp = sp0 + u * kCombWarps;
            v[u] = sp < nsplit ? *reinterpret_cast<const float4 *>(po + size_t(sp) * (G * HD))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    s_acc[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && lane < V4) {
        float4 r = s_acc[0][lane];
#pragma unroll
        for (int k = 1; k < kCombWarps; ++k) {
            const float4 t = s_acc[k][lane];
            r.x += t.x; r.y += t.y; r.z += t.z; r.w += t.w;
        }
        float *out = a.out + (size_t(seq) * a.n_kv * G + qh) * HD;
        *reinterpret_cast<float4 *>(out + 4 * lane) = r;
    }
}

template <int HD, int G, int SH>
int launch_t(leap_ctx *c, const DecodeArgs &a, const DecodeSeq &tab, int total_splits,
             bool overlap, bool tail) {
    using C = Cfg<HD, G, SH>;
    for (auto fn : {decode_attn_kernel<HD, G, SH, true>, decode_attn_kernel<HD, G, SH, false>}) {
        const int st = set_kernel_smem(reinterpret_cast<const void *>(fn), C::kSmem,
                                       "cudaFuncSetAttribute(decode)");
        if (st != LEAP_OK) return st;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(total_splits, c->n_kv);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = overlap ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const bool combine = !tail && total_splits > tab.n_seq;  // some sequence has splits
    const int st = cuda_status(
        cudaLaunchKernelEx(&cfg, combine ? decode_attn_kernel<HD, G, SH, false>
                                         : decode_attn_kernel<HD, G, SH, true>, a, tab),
        "decode_attn_kernel launch");
    if (st != LEAP_OK || !combine) return st;
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3(tab.n_seq, c->n_kv * G);
    cc.blockDim = dim3(32 * kCombWarps);
    cc.stream = c->stream;
    cudaLaunchAttribute cattr[1];
    cattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    cattr[0].val.programmaticStreamSerializationAllowed = 1;  // it waits before reading
    cc.attrs = cattr;
    cc.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cc, decode_combine_kernel<HD, G>, a, tab),
                       "decode_combine_kernel launch");
}

}  // namespace

int plan_decode(const leap_ctx *c, DecodeSeq &tab, int shape) {
    const int per_sm = shape == 1 ? 1 : 2;
    // At most 1024 rows (4 MB of K+V at head_dim 128) per CTA: long splits
    // amortise each CTA's prologue and partial; launches that fit one wave
    // are split finer anyway (below).
    const long cap_rows = 1024L * 128 / c->hd;
    long total = 0;
    int max_ctx = 0;
    for (int i = 0; i < tab.n_seq; ++i) {
        const int ctx = tab.pos[i] + 1;
        total += ctx;
        if (ctx > max_ctx) max_ctx = ctx;
    }
    const long rows = total * c->n_kv;
    const long target = long(per_sm) * c->num_sms;  // one wave
    long chunk = (rows + target - 1) / target;
    if (chunk > cap_rows) chunk = cap_rows;
    const long min_chunk = (max_ctx + kMaxSplitsPerSeq - 1) / kMaxSplitsPerSeq;
    if (chunk < min_chunk) chunk = min_chunk;
    // Chunks are whole 8-row groups (a CTA's last tile may be partial).  When
    // the work fits one wave, grow the chunk until the per-sequence ceilings
    // no longer push the CTA count past it.
    chunk = (chunk + 7) / 8 * 8;
    auto n_ctas = [&](long ch) {
        long n = 0;
        for (int i = 0; i < tab.n_seq; ++i) n += (tab.pos[i] + ch) / ch;
        return n * c->n_kv;
    };
    while (chunk < cap_rows && n_ctas(chunk) > target) chunk += 8;
    tab.chunk = int(chunk);
    int acc = 0;
    for (int i = 0; i < tab.n_seq; ++i) {
        tab.split0[i] = acc;
        acc += int((tab.pos[i] + chunk) / chunk);  // ceil((pos+1)/chunk)
    }
    tab.split0[tab.n_seq] = acc;
    return acc;
}

int max_decode_parts(int hd, int n_kv, int max_batch, int max_seq_pad, int num_sms) {
    // An upper bound on plan_decode's CTA count: a chunk shorter than 256
    // rows (hd 128) only occurs when the launch fits one wave (2 per SM).
    const long cap_rows = 262144L / (hd * 4 * 2);
    const long nb = max_batch < kMaxSeqPerLaunch ? max_batch : kMaxSeqPerLaunch;
    long a = (nb * max_seq_pad * long(n_kv) + cap_rows - 1) / cap_rows;
    if (a < 2L * num_sms) a = 2L * num_sms;
    return int(a + nb * n_kv * 2 + 64);
}

namespace {
template <int SH>
int launch_width(leap_ctx *c, const DecodeArgs &a, const DecodeSeq &tab, int total, bool overlap,
                 bool tail) {
    switch (c->hd * 100 + c->group) {
        case 12801: return launch_t<128, 1, SH>(c, a, tab, total, overlap, tail);
        case 12802: return launch_t<128, 2, SH>(c, a, tab, total, overlap, tail);
        case 12804: return launch_t<128, 4, SH>(c, a, tab, total, overlap, tail);
        case 12808: return launch_t<128, 8, SH>(c, a, tab, total, overlap, tail);
        case 6401: return launch_t<64, 1, SH>(c, a, tab, total, overlap, tail);
        case 6402: return launch_t<64, 2, SH>(c, a, tab, total, overlap, tail);
        case 6404: return launch_t<64, 4, SH>(c, a, tab, total, overlap, tail);
        case 6408: return launch_t<64, 8, SH>(c, a, tab, total, overlap, tail);
        default:
            set_error("unsupported head_dim %d / kv_mul %d", c->hd, c->group);
            return LEAP_ERR_INVALID;
    }
}
}  // namespace

int launch_decode(leap_ctx *c, int layer, const DecodeSeq &seqs, const float *q,
                  const float *k_new, const float *v_new, float *out) {
    // Overlap with the previous kernel only if this context's previous
    // operation did not write this layer (the early K/V prefetch must not
    // read rows that kernel may still be appending).
    const bool overlap = c->overlap && c->last_written_layer != leap_ctx::kWroteAll &&
                         c->last_written_layer != layer;
    // decode_impl 2 forces the cluster kernel (16 CTAs per kv head, split
    // reduction in distributed shared memory); auto never picks it unless
    // every head's cluster fits at once.
    const bool use_cluster =
        c->decode_impl == 2 ||
        (c->decode_impl == 0 && seqs.n_seq == 1 && c->cluster_capacity >= c->n_kv);
    if (use_cluster) {
        const int st = launch_decode_cluster(c, layer, seqs, q, k_new, v_new, out, overlap);
        if (st == LEAP_OK) c->last_written_layer = layer;
        return st;
    }
    // Split-KV CTA shape: 128 threads, two CTAs per SM (measured fastest at
    // ctx 1k-8k); impl 3 selects 256 threads, one per SM (half the splits).
    const int shape = c->decode_impl == 3 ? 1 : 0;
    // impl 4: the splits are combined by a second launch; else by the last CTA
    const bool tail = c->decode_impl != 4;
    DecodeSeq tab = seqs;
    plan_decode(c, tab, shape);
    const int total = tab.split0[tab.n_seq];
    if (long(total) * c->n_kv > c->max_parts) {
        set_error("decode plan needs %d partials, scratch holds %d", total * c->n_kv,
                  c->max_parts);
        return LEAP_ERR_INVALID;
    }
    DecodeArgs a;
    a.q = q;
    a.k_new = k_new;
    a.v_new = v_new;
    a.out = out;
    a.k_cache = c->k_cache;
    a.v_cache = c->v_cache;
    a.rope_cos = c->rope_cos;
    a.rope_sin = c->rope_sin;
    a.head_stride = c->head_stride;
    a.layer_off = size_t(layer) * c->layer_stride;
    a.slot_stride = c->slot_stride;
    // alternate scratch sets so an overlapped launch never shares the
    // previous launch's partials or tickets
    a.part_o = c->part_o[c->parity];
    a.part_ml = c->part_ml[c->parity];
    a.counters = c->counters[c->parity];
    a.err = c->d_err;
    a.err_host = c->err_host;
    a.n_kv = c->n_kv;
    a.scale_log2 = kLog2e / sqrtf(float(c->hd));
    const int st = shape == 0 ? launch_width<0>(c, a, tab, total, overlap, tail)
                              : launch_width<1>(c, a, tab, total, overlap, tail);
    if (st == LEAP_OK) {
        c->parity ^= 1;
        c->last_written_layer = layer;
    }
    return st;
}

}  // namespace leap
