// decode_cluster.cu — decode attention with the split-KV reduction done in
// distributed shared memory inside a thread-block cluster.
//
// Same semantics as decode_attn.cu (the reference block of
// src/inference/FloatTransformer.cpp:404-662: RoPE of q and of the new k
// row, append to cache row `pos`, softmax(q.K^T/sqrt(hd)).V over 0..pos).
//
// One cluster of CS CTAs per (sequence, kv head); CTA rank r streams rows
// [r*per, (r+1)*per) of that head's K/V through a bulk-copy pipeline (one
// CTA per SM, 8 warps, 192 KB of stages) and keeps its partial softmax
// state (M, L, O) in its own shared memory.  After a cluster barrier every
// CTA reads the CS partials of its slice of the output columns from its
// peers' shared memory, combines them and writes the result: no global
// atomics, no L2 round trips, no last-CTA tail.
#include <cooperative_groups.h>

#include "common.cuh"
#include "ctx.h"

namespace cg = cooperative_groups;

namespace leap {
namespace {

constexpr int kCThreads = 256;
constexpr int kCWarps = kCThreads / 32;
constexpr int kCStages = 3;
constexpr int kCTileBytes = 32768;  // per tensor per stage

template <int HD, int G, int CS>
struct CCfg {
    static constexpr int kLpr0 = G * HD / 64;
    static constexpr int LPR = kLpr0 < 8 ? 8 : (kLpr0 > 32 ? 32 : kLpr0);
    static constexpr int RPW = 32 / LPR;
    static constexpr int NGRP = kCWarps * RPW;
    static constexpr int DPL = HD / LPR;
    static constexpr int C4 = DPL / 4;
    static constexpr int TILE = kCTileBytes / (HD * 4);
    static constexpr int RPG = TILE / NGRP;
    static constexpr int NV4 = G * HD / 4;       // float4 outputs per (seq, kv head)
    static constexpr int SLICE = NV4 / CS;       // float4 outputs reduced per CTA
    static constexpr size_t kSmem = size_t(2) * kCStages * TILE * HD * sizeof(float);
    static_assert(DPL % 4 == 0 && C4 >= 1, "lane slice must be float4s");
    static_assert(TILE % NGRP == 0, "tile rows must split over groups");
    static_assert(NV4 % CS == 0 && SLICE >= 1, "output slices per CTA");
    static_assert(size_t(NGRP) * G * HD * sizeof(float) <= kSmem / 2, "merge buffer in K half");
};

struct ClusterArgs {
    const float *q, *k_new, *v_new;
    float *out;
    float *k_cache, *v_cache;
    const float *rope_cos, *rope_sin;
    size_t head_stride, layer_off, slot_stride;
    int *err;
    int *err_host;  // non-null: error codes also go to this host-mapped word
    int n_kv;
    float scale_log2;
};

template <int HD, int G, int CS>
__global__ void __launch_bounds__(kCThreads, 1)
decode_cluster_kernel(const ClusterArgs a, const DecodeSeq tab) {
    using C = CCfg<HD, G, CS>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    float *sK = reinterpret_cast<float *>(smem_raw);  // [stages][TILE][HD]
    float *sV = sK + kCStages * C::TILE * HD;
    __shared__ uint64_t full_bar[kCStages];
    __shared__ float red_m[C::NGRP][G], red_l[C::NGRP][G];
    __shared__ float s_M[G], s_L[G];            // this CTA's partial, read by peers
    __shared__ float s_w[CS][G];                // combine weights of my slice
    __shared__ __align__(16) float s_O[G * HD]; // this CTA's partial O, read by peers

    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int j = lane % C::LPR;
    const int grp = warp * C::RPW + lane / C::LPR;
    const int rank = int(cluster.block_rank());
    const int seq = blockIdx.x / CS;
    const int kvh = blockIdx.y;
    const int pos = tab.pos[seq];
    const int ctx = pos + 1;
    const int per = (ctx + CS - 1) / CS;
    const int row_begin = min(rank * per, ctx);
    const int row_end = min(row_begin + per, ctx);
    const int n_tiles = (row_end - row_begin + C::TILE - 1) / C::TILE;
    const bool owns_pos = (pos >= row_begin && pos < row_end);

    const size_t head_off = size_t(tab.slot[seq]) * a.slot_stride + a.layer_off +
                            size_t(kvh) * a.head_stride;
    float *gK = a.k_cache + head_off;
    float *gV = a.v_cache + head_off;

    if (tid == 0) {
        for (int s = 0; s < kCStages; ++s) mbar_init(&full_bar[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int t = 0; t < min(kCStages, n_tiles); ++t) {
            const int r0 = row_begin + t * C::TILE;
            const uint32_t bytes = min(C::TILE, row_end - r0) * HD * 4;
            mbar_arrive_expect_tx(&full_bar[t], 2 * bytes);
            bulk_g2s(sK + t * C::TILE * HD, gK + size_t(r0) * HD, bytes, &full_bar[t]);
            bulk_g2s(sV + t * C::TILE * HD, gV + size_t(r0) * HD, bytes, &full_bar[t]);
        }
    }
    // Only this layer's cache rows were read so far (see decode_attn.cu).
    grid_dependency_wait();
    grid_launch_dependents();

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

    bool ok = true;
    int t = 0;
    for (; t < n_tiles; ++t) {
        const int s = t % kCStages;
        ok = mbar_wait(&full_bar[s], (t / kCStages) & 1);
        ok = __syncthreads_and(ok);
        if (!ok) break;
        const int r0 = row_begin + t * C::TILE;
        float *tK = sK + s * C::TILE * HD;
        float *tV = sV + s * C::TILE * HD;

        if (owns_pos && pos < r0 + C::TILE) {
            const int rr = pos - r0;
            const float *kn = a.k_new + (size_t(seq) * a.n_kv + kvh) * HD;
            const float *vn = a.v_new + (size_t(seq) * a.n_kv + kvh) * HD;
            for (int d = 2 * tid; d < HD; d += 2 * kCThreads) {
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

        float sc[C::RPG][G];
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
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float mt = m[g];
#pragma unroll
            for (int rr = 0; rr < C::RPG; ++rr) mt = fmaxf(mt, sc[rr][g]);
            const float alpha = (mt == -INFINITY) ? 1.f : fast_exp2(m[g] - mt);
            m[g] = mt;
            l[g] *= alpha;
#pragma unroll
            for (int d = 0; d < C::DPL; ++d) o[g][d] *= alpha;
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
        __syncthreads();
        if (tid == 0 && t + kCStages < n_tiles) {
            const int tn = t + kCStages;
            const int rn = row_begin + tn * C::TILE;
            const uint32_t bytes = min(C::TILE, row_end - rn) * HD * 4;
            mbar_arrive_expect_tx(&full_bar[s], 2 * bytes);
            bulk_g2s(tK, gK + size_t(rn) * HD, bytes, &full_bar[s]);
            bulk_g2s(tV, gV + size_t(rn) * HD, bytes, &full_bar[s]);
        }
    }
    if (!ok) {
        // A wait gave up: let the copies in flight land (bounded), report,
        // and contribute an empty partial so the cluster still completes.
        for (int tt = t + 1; tt < min(t + kCStages, n_tiles); ++tt)
            (void)mbar_wait(&full_bar[tt % kCStages], (tt / kCStages) & 1);
        if (tid == 0) report_error(a.err, a.err_host, kDevWaitTimeout);
#pragma unroll
        for (int g = 0; g < G; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.f;
#pragma unroll
            for (int d = 0; d < C::DPL; ++d) o[g][d] = 0.f;
        }
        __syncthreads();
    }

    // ---- this CTA's partial: merge its row groups -------------------------
    if (j == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            red_m[grp][g] = m[g];
            red_l[grp][g] = l[g];
        }
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int gg = 0; gg < C::NGRP; ++gg) M = fmaxf(M, red_m[gg][tid]);
        float L = 0.f;
        if (M != -INFINITY)
            for (int gg = 0; gg < C::NGRP; ++gg) {
                const float mg = red_m[gg][tid];
                if (mg != -INFINITY) L += red_l[gg][tid] * fast_exp2(mg - M);
            }
        s_M[tid] = M;
        s_L[tid] = L;
    }
    __syncthreads();
    float *red_o = sK;  // [NGRP][G][HD]
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float f = (m[g] == -INFINITY) ? 0.f : fast_exp2(m[g] - s_M[g]);
#pragma unroll
        for (int i = 0; i < C::C4; ++i) {
            float4 v;
            v.x = o[g][4 * i + 0] * f;
            v.y = o[g][4 * i + 1] * f;
            v.z = o[g][4 * i + 2] * f;
            v.w = o[g][4 * i + 3] * f;
            *reinterpret_cast<float4 *>(red_o + (grp * G + g) * HD + 4 * (j + C::LPR * i)) = v;
        }
    }
    __syncthreads();
    for (int e = tid; e < C::NV4; e += kCThreads) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int gg = 0; gg < C::NGRP; ++gg) {
            const float4 v = *reinterpret_cast<const float4 *>(red_o + gg * G * HD + 4 * e);
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
        }
        *reinterpret_cast<float4 *>(s_O + 4 * e) = acc;
    }

    // ---- cluster reduction through distributed shared memory --------------
    cluster.sync();  // every CTA's (M, L, O) partial is in its shared memory
    if (tid < CS * G) {
        const int r = tid / G, g = tid % G;
        const float *pm = cluster.map_shared_rank(s_M, r);
        s_w[r][g] = pm[g];
    }
    __syncthreads();
    if (tid < G) {
        const int g = tid;
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < CS; ++r) M = fmaxf(M, s_w[r][g]);
        float L = 0.f;
#pragma unroll
        for (int r = 0; r < CS; ++r) {
            const float *pl = cluster.map_shared_rank(s_L, r);
            const float mr = s_w[r][g];
            if (mr != -INFINITY) L += pl[g] * fast_exp2(mr - M);
        }
        const float inv = 1.f / L;
#pragma unroll
        for (int r = 0; r < CS; ++r) {
            const float mr = s_w[r][g];
            s_w[r][g] = (mr == -INFINITY) ? 0.f : fast_exp2(mr - M) * inv;
        }
    }
    __syncthreads();
    float *out_seq = a.out + (size_t(seq) * a.n_kv * G + qh0) * HD;
    if (tid < C::SLICE) {
        const int e = rank * C::SLICE + tid;
        const int g = (4 * e) / HD;
        float4 vals[CS];
#pragma unroll
        for (int r = 0; r < CS; ++r)
            vals[r] = *reinterpret_cast<const float4 *>(cluster.map_shared_rank(s_O, r) + 4 * e);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < CS; ++r) {
            const float w = s_w[r][g];
            acc.x = fmaf(w, vals[r].x, acc.x);
            acc.y = fmaf(w, vals[r].y, acc.y);
            acc.z = fmaf(w, vals[r].z, acc.z);
            acc.w = fmaf(w, vals[r].w, acc.w);
        }
        *reinterpret_cast<float4 *>(out_seq + 4 * e) = acc;
    }
    cluster.sync();  // peers may still be reading this CTA's shared memory
}

template <int HD, int G, int CS>
int launch_c(leap_ctx *c, const ClusterArgs &a, const DecodeSeq &tab, bool overlap) {
    using C = CCfg<HD, G, CS>;
    auto kern = decode_cluster_kernel<HD, G, CS>;
    if (const int st = set_kernel_smem(reinterpret_cast<const void *>(kern), C::kSmem,
                                       "cudaFuncSetAttribute(decode_cluster)", CS > 8))
        return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CS * tab.n_seq, c->n_kv);
    cfg.blockDim = dim3(kCThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = overlap ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cuda_status(cudaLaunchKernelEx(&cfg, kern, a, tab), "decode_cluster_kernel launch");
}

template <int HD, int G, int CS>
int max_clusters_t(int device, int *n) {
    using C = CCfg<HD, G, CS>;
    auto kern = decode_cluster_kernel<HD, G, CS>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(C::kSmem));
    if (e == cudaSuccess && CS > 8)
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(decode_cluster)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CS, 1);
    cfg.blockDim = dim3(kCThreads);
    cfg.dynamicSmemBytes = C::kSmem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CS;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    (void)device;
    return cuda_status(cudaOccupancyMaxActiveClusters(n, kern, &cfg),
                       "cudaOccupancyMaxActiveClusters");
}

}  // namespace

constexpr int kClusterSize = 16;

// How many 16-CTA clusters of the decode kernel fit on the device at once.
int decode_cluster_capacity(leap_ctx *c, int *n) {
    *n = 0;
    switch (c->hd * 100 + c->group) {
        case 12801: return max_clusters_t<128, 1, kClusterSize>(c->device, n);
        case 12802: return max_clusters_t<128, 2, kClusterSize>(c->device, n);
        case 12804: return max_clusters_t<128, 4, kClusterSize>(c->device, n);
        case 12808: return max_clusters_t<128, 8, kClusterSize>(c->device, n);
        case 6401: return max_clusters_t<64, 1, kClusterSize>(c->device, n);
        case 6402: return max_clusters_t<64, 2, kClusterSize>(c->device, n);
        case 6404: return max_clusters_t<64, 4, kClusterSize>(c->device, n);
        case 6408: return max_clusters_t<64, 8, kClusterSize>(c->device, n);
        default: return LEAP_OK;
    }
}

int launch_decode_cluster(leap_ctx *c, int layer, const DecodeSeq &tab, const float *q,
                          const float *k_new, const float *v_new, float *out, bool overlap) {
    ClusterArgs a;
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
    a.err = c->d_err;
    a.err_host = c->err_host;
    a.n_kv = c->n_kv;
    a.scale_log2 = kLog2e / sqrtf(float(c->hd));
    switch (c->hd * 100 + c->group) {
        case 12801: return launch_c<128, 1, kClusterSize>(c, a, tab, overlap);
        case 12802: return launch_c<128, 2, kClusterSize>(c, a, tab, overlap);
        case 12804: return launch_c<128, 4, kClusterSize>(c, a, tab, overlap);
        case 12808: return launch_c<128, 8, kClusterSize>(c, a, tab, overlap);
        case 6401: return launch_c<64, 1, kClusterSize>(c, a, tab, overlap);
        case 6402: return launch_c<64, 2, kClusterSize>(c, a, tab, overlap);
        case 6404: return launch_c<64, 4, kClusterSize>(c, a, tab, overlap);
        case 6408: return launch_c<64, 8, kClusterSize>(c, a, tab, overlap);
        default:
            set_error("unsupported head_dim %d / kv_mul %d", c->hd, c->group);
            return LEAP_ERR_INVALID;
    }
}

}  // namespace leap
