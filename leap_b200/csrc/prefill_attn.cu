// prefill_attn.cu — causal prefill: RoPE + KV append for a prompt chunk,
// then causal GQA attention of every prompt token over the cache.
//
// The reference has no batched prefill: it feeds prompt tokens one at a
// time through forward() (src/inference/main.cpp:80-89), each running the
// attention block of src/inference/FloatTransformer.cpp:404-662 at its own
// position.  Running that block for pos = pos0 .. pos0+n-1 in order is the
// same as causal attention of the chunk over cache rows 0..pos0+i, which is
// what these kernels compute.
//
// This file holds the append kernel and the CUDA-core FP32 attention
// kernel (impl 1); the tensor-core 3xTF32 kernel lives in
// prefill_tc.cu.
#include <cstdio>

#include "common.cuh"
#include "ctx.h"

namespace leap {

// Rotate every token's q (into qrot) and k, and append k and v to the cache
// rows pos0 .. pos0+n_tok-1 of one (slot, layer).
template <int HD>
__global__ void __launch_bounds__(256)
prefill_rope_append_kernel(const float *__restrict__ q, const float *__restrict__ k,
                           const float *__restrict__ v, float *__restrict__ qrot,
                           float *__restrict__ kc, float *__restrict__ vc, size_t head_stride,
                           const float *__restrict__ rope_cos,
                           const float *__restrict__ rope_sin, int pos0, int n_heads,
                           int n_kv) {
    const int t = blockIdx.x;
    const int pos = pos0 + t;
    const float *rc = rope_cos + size_t(pos) * (HD / 2);
    const float *rs = rope_sin + size_t(pos) * (HD / 2);
    const int nq = n_heads * (HD / 2), nk = n_kv * (HD / 2);
    for (int p = threadIdx.x; p < nq + nk; p += blockDim.x) {
        if (p < nq) {
            const int h = p / (HD / 2), i = p % (HD / 2);
            const size_t off = (size_t(t) * n_heads + h) * HD + 2 * i;
            const float2 x = *reinterpret_cast<const float2 *>(q + off);
            *reinterpret_cast<float2 *>(qrot + off) = rope_pair(x.x, x.y, rc[i], rs[i]);
        } else {
            const int p2 = p - nq;
            const int h = p2 / (HD / 2), i = p2 % (HD / 2);
            const size_t src = (size_t(t) * n_kv + h) * HD + 2 * i;
            const size_t dst = size_t(h) * head_stride + size_t(pos) * HD + 2 * i;
            const float2 x = *reinterpret_cast<const float2 *>(k + src);
            *reinterpret_cast<float2 *>(kc + dst) = rope_pair(x.x, x.y, rc[i], rs[i]);
            *reinterpret_cast<float2 *>(vc + dst) = *reinterpret_cast<const float2 *>(v + src);
        }
    }
}

namespace {

constexpr int kBM = 64;   // query rows per CTA (tokens x G heads)
constexpr int kBN = 64;   // keys per tile
constexpr int kPT = 256;  // threads

template <int HD>
constexpr size_t fma_smem_bytes() {
    return sizeof(float) * (size_t(kBM) * (HD + 4) + size_t(kBN) * (HD + 4) +
                            size_t(kBN) * HD + size_t(kBM) * (kBN + 1));
}

// Flash-style causal attention on CUDA cores, FP32 throughout.
// CTA = (block of kBM/G tokens, kv head); row r of the CTA is token r/G,
// head kvh*G + r%G.  Thread (ty, tx) owns rows ty+16i and keys tx+16c of
// each 64x64 score tile, and rows ty+16i x cols tx*4+64jj of the output.
template <int HD, int G>
__global__ void __launch_bounds__(kPT)
prefill_fma_kernel(const float *__restrict__ qrot, const float *__restrict__ kc,
                   const float *__restrict__ vc, size_t head_stride, float *__restrict__ out,
                   int pos0, int n_tok, int n_heads, float scale_log2) {
    constexpr int BT = kBM / G;
    constexpr int QS = HD + 4;
    constexpr int PS = kBN + 1;
    constexpr int NJ = HD / 64;
    extern __shared__ __align__(16) float sm[];
    float *sQ = sm;                 // [kBM][QS]
    float *sK = sQ + kBM * QS;      // [kBN][QS]
    float *sV = sK + kBN * QS;      // [kBN][HD]
    float *sP = sV + kBN * HD;      // [kBM][PS]

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int kvh = blockIdx.y;
    const int tb = gridDim.x - 1 - blockIdx.x;  // longest rows first
    const int t0 = tb * BT;
    const float *kb = kc + size_t(kvh) * head_stride;
    const float *vb = vc + size_t(kvh) * head_stride;

    for (int idx = tid; idx < kBM * HD / 4; idx += kPT) {
        const int r = idx / (HD / 4), c4 = idx % (HD / 4);
        const int tok = t0 + r / G;
        float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
        if (tok < n_tok)
            val = *reinterpret_cast<const float4 *>(
                qrot + (size_t(tok) * n_heads + kvh * G + r % G) * HD + 4 * c4);
        *reinterpret_cast<float4 *>(sQ + r * QS + 4 * c4) = val;
    }

    float m[4], l[4], o[4][4 * NJ];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < 4 * NJ; ++c) o[i][c] = 0.f;
    }
    const int last_tok = min(t0 + BT, n_tok) - 1;
    const int kv_end = pos0 + last_tok + 1;
    const int n_kt = (kv_end + kBN - 1) / kBN;

    for (int kt = 0; kt < n_kt; ++kt) {
        __syncthreads();
        const int k0 = kt * kBN;
        for (int idx = tid; idx < kBN * HD / 4; idx += kPT) {
            const int r = idx / (HD / 4), c4 = idx % (HD / 4);
            float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
            if (k0 + r < kv_end) {
                kk = *reinterpret_cast<const float4 *>(kb + size_t(k0 + r) * HD + 4 * c4);
                vv = *reinterpret_cast<const float4 *>(vb + size_t(k0 + r) * HD + 4 * c4);
            }
            *reinterpret_cast<float4 *>(sK + r * QS + 4 * c4) = kk;
            *reinterpret_cast<float4 *>(sV + r * HD + 4 * c4) = vv;
        }
        __syncthreads();

        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            float4 a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                a[i] = *reinterpret_cast<const float4 *>(sQ + (ty + 16 * i) * QS + d);
#pragma unroll
            for (int c = 0; c < 4; ++c)
                b[c] = *reinterpret_cast<const float4 *>(sK + (tx + 16 * c) * QS + d);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    s[i][c] = fmaf(a[i].x, b[c].x, s[i][c]);
                    s[i][c] = fmaf(a[i].y, b[c].y, s[i][c]);
                    s[i][c] = fmaf(a[i].z, b[c].z, s[i][c]);
                    s[i][c] = fmaf(a[i].w, b[c].w, s[i][c]);
                }
        }

#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = ty + 16 * i;
            const int qpos = pos0 + t0 + r / G;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int key = k0 + tx + 16 * c;
                s[i][c] = (key <= qpos) ? s[i][c] * scale_log2 : -INFINITY;
                mx = fmaxf(mx, s[i][c]);
            }
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1)
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[i], mx);
            const float alpha = (mn == -INFINITY) ? 1.f : fast_exp2(m[i] - mn);
            float rs = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const float p = (s[i][c] == -INFINITY) ? 0.f : fast_exp2(s[i][c] - mn);
                rs += p;
                sP[r * PS + tx + 16 * c] = p;
            }
#pragma unroll
            for (int off = 8; off >= 1; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            l[i] = l[i] * alpha + rs;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < 4 * NJ; ++c) o[i][c] *= alpha;
        }
        __syncthreads();

#pragma unroll 4
        for (int kk = 0; kk < kBN; ++kk) {
            float a[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = sP[(ty + 16 * i) * PS + kk];
#pragma unroll
            for (int jj = 0; jj < NJ; ++jj) {
                const float4 b = *reinterpret_cast<const float4 *>(sV + kk * HD + tx * 4 + 64 * jj);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    o[i][4 * jj + 0] = fmaf(a[i], b.x, o[i][4 * jj + 0]);
                    o[i][4 * jj + 1] = fmaf(a[i], b.y, o[i][4 * jj + 1]);
                    o[i][4 * jj + 2] = fmaf(a[i], b.z, o[i][4 * jj + 2]);
                    o[i][4 * jj + 3] = fmaf(a[i], b.w, o[i][4 * jj + 3]);
                }
            }
        }
    }

#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = ty + 16 * i;
        const int tok = t0 + r / G;
        if (tok < n_tok) {
            const float inv = 1.f / l[i];
            float *dst = out + (size_t(tok) * n_heads + kvh * G + r % G) * HD;
#pragma unroll
            for (int jj = 0; jj < NJ; ++jj) {
                float4 v;
                v.x = o[i][4 * jj + 0] * inv;
                v.y = o[i][4 * jj + 1] * inv;
                v.z = o[i][4 * jj + 2] * inv;
                v.w = o[i][4 * jj + 3] * inv;
                *reinterpret_cast<float4 *>(dst + tx * 4 + 64 * jj) = v;
            }
        }
    }
}

template <int HD, int G>
int launch_fma(leap_ctx *c, const float *qrot, const float *kc, const float *vc, float *out,
               int pos0, int n_tok) {
    constexpr size_t smem = fma_smem_bytes<HD>();
    const void *fn = reinterpret_cast<const void *>(prefill_fma_kernel<HD, G>);
    if (const int st = set_kernel_smem(fn, smem, "cudaFuncSetAttribute(prefill)")) return st;
    constexpr int BT = kBM / G;
    dim3 grid((n_tok + BT - 1) / BT, c->n_kv);
    prefill_fma_kernel<HD, G><<<grid, kPT, smem, c->stream>>>(
        qrot, kc, vc, c->head_stride, out, pos0, n_tok, c->n_heads,
        kLog2e / sqrtf(float(HD)));
    return cuda_status(cudaGetLastError(), "prefill_fma_kernel launch");
}

}  // namespace

// tensor-core path (prefill_tc.cu); returns LEAP_ERR_INVALID when the shape
// is not supported there.
int launch_prefill_tc(leap_ctx *c, const float *qrot, const float *kc, const float *vc,
                      float *out, int pos0, int n_tok);
// the same product, software-pipelined across warp roles (prefill_tc_pipe.cu):
// the default
int launch_prefill_tc_pipe(leap_ctx *c, const float *qrot, const float *kc, const float *vc,
                           float *out, int pos0, int n_tok, bool bf16_corrections);

int launch_prefill(leap_ctx *c, int slot, int layer, int pos0, int n_tok, const float *q,
                   const float *k, const float *v, float *out) {
    const size_t need = size_t(n_tok) * c->n_heads * c->hd;
    if (need > c->qrot_cap) {
        cudaError_t e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) return cuda_status(e, "sync before scratch growth");
        cudaFree(c->d_qrot);
        c->d_qrot = nullptr;
        c->qrot_cap = 0;
        e = cudaMalloc(&c->d_qrot, need * sizeof(float));
        if (e != cudaSuccess) return cuda_status(e, "cudaMalloc(prefill scratch)");
        c->qrot_cap = need;
    }
    float *kc = k_head_ptr(c, slot, layer, 0);
    float *vc = v_head_ptr(c, slot, layer, 0);
    if (c->hd == 128)
        prefill_rope_append_kernel<128><<<n_tok, 256, 0, c->stream>>>(
            q, k, v, c->d_qrot, kc, vc, c->head_stride, c->rope_cos, c->rope_sin, pos0,
            c->n_heads, c->n_kv);
    else
        prefill_rope_append_kernel<64><<<n_tok, 256, 0, c->stream>>>(
            q, k, v, c->d_qrot, kc, vc, c->head_stride, c->rope_cos, c->rope_sin, pos0,
            c->n_heads, c->n_kv);
    if (int st = cuda_status(cudaGetLastError(), "prefill_rope_append launch")) return st;

    if (c->prefill_impl != 1) {
        const int st = c->prefill_impl == 2
                           ? launch_prefill_tc(c, c->d_qrot, kc, vc, out, pos0, n_tok)
                           : launch_prefill_tc_pipe(c, c->d_qrot, kc, vc, out, pos0, n_tok,
                                                    c->prefill_impl == 3);
        if (st != LEAP_ERR_INVALID) return st;
        clear_error();  // shape not covered by the tensor-core kernel
    }
    switch (c->hd * 100 + c->group) {
        case 12801: return launch_fma<128, 1>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        case 12802: return launch_fma<128, 2>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        case 12804: return launch_fma<128, 4>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        case 12808: return launch_fma<128, 8>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        case 6401: return launch_fma<64, 1>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        case 6402: return launch_fma<64, 2>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        case 6404: return launch_fma<64, 4>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        case 6408: return launch_fma<64, 8>(c, c->d_qrot, kc, vc, out, pos0, n_tok);
        default:
            set_error("unsupported head_dim %d / kv_mul %d", c->hd, c->group);
            return LEAP_ERR_INVALID;
    }
}

}  // namespace leap
