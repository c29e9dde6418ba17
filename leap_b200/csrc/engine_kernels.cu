// engine_kernels.cu — the support ops around attention in the forward pass
// (src/inference/FloatTransformer.cpp:384-797 and
// src/inference/QuantizedTransformer.cpp:654-1061), on the GPU.
//
// These are correct GPU versions, not the optimisation target: embedding
// gather, RMSNorm, FP32 GEMV/GEMM, per-group activation quantization, the
// W8A8 GEMV/GEMM, SiLU*up, residual adds, greedy argmax, and a synthetic
// weight generator.  Two of them reproduce the reference's compiled
// arithmetic bit for bit: the activation quantization (scale = max * (1/127),
// round half away from zero) and the W8A8 dot (int32 group dots, then per
// output val = fma(float(ival), w_s * x_s, val) over the groups in order).
#include <cstdint>

#include "common.cuh"
#include "engine.h"

namespace leap {
namespace eng {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- embedding -------------------------------------------------------------
// FloatTransformer.cpp:758-759 (copy of the row); W8A8 engines dequantize the
// table at load (QuantizedTransformer.cpp:116-117, :136-216): q * s.
__global__ void embed_f32_kernel(float *__restrict__ x, const float *__restrict__ emb,
                                 const int *__restrict__ tok, int dim) {
    const int row = blockIdx.x;
    const float *src = emb + size_t(tok[row]) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[size_t(row) * dim + i] = src[i];
}

__global__ void embed_q8_kernel(float *__restrict__ x, const int8_t *__restrict__ q,
                                const float *__restrict__ s, const int *__restrict__ tok,
                                int dim, int gs) {
    const int row = blockIdx.x;
    const size_t base = size_t(tok[row]) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        x[size_t(row) * dim + i] = float(q[base + i]) * s[(base + i) / gs];
}

// ---- RMSNorm (FloatTransformer.cpp:79-214) ---------------------------------
// o = w * (r * x), r = 1/sqrt(mean(x^2) + 1e-5).  The reference's AVX2 path
// refines an rsqrt estimate by one Newton step; 1/sqrtf is within 2e-7.
__global__ void rmsnorm_kernel(float *o, const float *x,  // o may alias x
                               const float *__restrict__ w, int dim) {
    __shared__ float red[32];
    const int row = blockIdx.x;
    const float *xr = x + size_t(row) * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    float m = red[0] / float(dim);
    m += 1e-5f;
    const float r = 1.0f / sqrtf(m);
    float *orow = o + size_t(row) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) orow[i] = w[i] * (r * xr[i]);
}

// ---- activation quantization (QuantizedTransformer.cpp:338-357) ------------
// One warp per group of `gs` (<= 128) values.
__global__ void quantize_kernel(int8_t *__restrict__ q, float *__restrict__ s,
                                const float *__restrict__ x, size_t n, int gs) {
    const size_t g = (size_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const size_t i0 = g * gs;
    if (i0 >= n) return;
    const int cur = int(min(size_t(gs), n - i0));
    float mx = 0.f;
    for (int j = lane; j < cur; j += 32) mx = fmaxf(mx, fabsf(x[i0 + j]));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // The reference's release build (-ffast-math) evaluates the source's
    // scale = max/127 as max * (1/127) and id = 1/scale as 127/max.
    const float inv127 = 1.0f / 127.0f;
    const float scale = __fmul_rn(mx, inv127);
    const float id = scale != 0.f ? __fdiv_rn(127.0f, mx) : 0.f;
    if (lane == 0) s[g] = scale;
    for (int j = lane; j < cur; j += 32) q[i0 + j] = int8_t(roundf(__fmul_rn(x[i0 + j], id)));
}

// ---- W8A8 GEMV (QuantizedTransformer.cpp:359-652) --------------------------
// y[r] = (res ? res[r] : 0) + sum_g fma-chain(float(idot_g), ws[r,g]*xs[g]);
// y may alias res (the residual add x += W.v), so neither is __restrict__.
// A CTA takes 32 rows: phase 1 streams the int8 rows (16 bytes per thread,
// coalesced), 4 threads reduce a 64-wide group's int32 dot; phase 2 runs
// each row's group chain in order in one thread, as the reference does.
constexpr int kQRows = 32;
constexpr int kQThreads = 256;

__global__ void __launch_bounds__(kQThreads)
gemv_q8_kernel(float *y, const int8_t *__restrict__ xq, const float *__restrict__ xs,
               const int8_t *__restrict__ wq, const float *__restrict__ ws, int n, int d,
               const float *res) {
    extern __shared__ __align__(16) unsigned char sm[];
    const int ngroups = n / 64;
    const int ng1 = ngroups + 1;  // odd row stride: the per-row chains hit distinct banks
    int8_t *sx = reinterpret_cast<int8_t *>(sm);                          // [n]
    int *sdot = reinterpret_cast<int *>(sm + ((n + 15) & ~15));            // [kQRows][ng1]
    float *sws = reinterpret_cast<float *>(sdot + kQRows * ng1);           // [kQRows][ng1]
    float *sxs = sws + kQRows * ng1;                                       // [ngroups]
    const int r0 = blockIdx.x * kQRows;
    const int nrows = min(kQRows, d - r0);
    for (int i = threadIdx.x * 16; i < n; i += kQThreads * 16)
        *reinterpret_cast<int4 *>(sx + i) = *reinterpret_cast<const int4 *>(xq + i);
    for (int i = threadIdx.x; i < nrows * ngroups; i += kQThreads) {
        const int row = i / ngroups, g = i - row * ngroups;
        sws[row * ng1 + g] = ws[size_t(r0) * ngroups + i];  // rows r0.. are contiguous
    }
    for (int g = threadIdx.x; g < ngroups; g += kQThreads) sxs[g] = xs[g];
    __syncthreads();
    const int chunks_per_row = n / 16;
    const int total = nrows * chunks_per_row;
    for (int f = threadIdx.x; f < kQRows * chunks_per_row; f += kQThreads) {
        // every thread of a 4-lane group takes the same trip count: rows
        // beyond d contribute zeros
        int dot = 0;
        const int row = f / chunks_per_row, ch = f - row * chunks_per_row;
        if (f < total) {
            const int4 w = *reinterpret_cast<const int4 *>(wq + size_t(r0 + row) * n + ch * 16);
            const int4 xv = *reinterpret_cast<const int4 *>(sx + ch * 16);
            dot = __dp4a(w.x, xv.x, dot);
            dot = __dp4a(w.y, xv.y, dot);
            dot = __dp4a(w.z, xv.z, dot);
            dot = __dp4a(w.w, xv.w, dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        if ((ch & 3) == 0 && f < total) sdot[row * ng1 + (ch >> 2)] = dot;
    }
    __syncthreads();
    if (threadIdx.x < nrows) {
        const int row = threadIdx.x;
        float val = 0.f;
#pragma unroll 4
        for (int g = 0; g < ngroups; ++g)
            val = fmaf(float(sdot[row * ng1 + g]), __fmul_rn(sws[row * ng1 + g], sxs[g]), val);
        y[r0 + row] = res ? __fadd_rn(res[r0 + row], val) : val;
    }
}

// ---- W8A8 GEMM (prompt chunks): 64 rows x 32 tokens per CTA ---------------
// Same per-(row, token) arithmetic as the GEMV: the int32 dot of each group,
// then the ordered fma chain over groups.
constexpr int kGR = 64, kGT = 32, kGThreads = 256;

__global__ void __launch_bounds__(kGThreads)
gemm_q8_kernel(float *y, const int8_t *__restrict__ xq, const float *__restrict__ xs,
               const int8_t *__restrict__ wq, const float *__restrict__ ws, int n, int d, int T,
               const float *res) {
    __shared__ __align__(16) int8_t sw[kGR][64];
    __shared__ __align__(16) int8_t sxq[kGT][64];
    __shared__ float sws[kGR], sxs[kGT];
    const int ngroups = n / 64;
    const int r0 = blockIdx.x * kGR, t0 = blockIdx.y * kGT;
    // thread -> 8 (row, token) pairs: rows ty*? ; tokens
    const int tr = threadIdx.x >> 3;        // 0..31 : rows tr and tr+32
    const int tt = (threadIdx.x & 7) * 4;   // tokens tt..tt+3
    float acc[2][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
    for (int g = 0; g < ngroups; ++g) {
        __syncthreads();
        // stage W [64 rows][64] and X [32 tok][64] (16 bytes per thread)
        {
            const int row = threadIdx.x >> 2, c = (threadIdx.x & 3) * 16;
            int4 v = make_int4(0, 0, 0, 0);
            if (r0 + row < d) v = *reinterpret_cast<const int4 *>(wq + size_t(r0 + row) * n + g * 64 + c);
            *reinterpret_cast<int4 *>(&sw[row][c]) = v;
            if (threadIdx.x < kGT * 4) {
                int4 u = make_int4(0, 0, 0, 0);
                if (t0 + row < T) u = *reinterpret_cast<const int4 *>(xq + size_t(t0 + row) * n + g * 64 + c);
                *reinterpret_cast<int4 *>(&sxq[row][c]) = u;
            }
            if (threadIdx.x < kGR) sws[threadIdx.x] = (r0 + threadIdx.x < d) ? ws[size_t(r0 + threadIdx.x) * ngroups + g] : 0.f;
            if (threadIdx.x < kGT) sxs[threadIdx.x] = (t0 + threadIdx.x < T) ? xs[size_t(t0 + threadIdx.x) * ngroups + g] : 0.f;
        }
        __syncthreads();
        int dot[2][4];
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) dot[a][b] = 0;
#pragma unroll
        for (int k = 0; k < 64; k += 16) {
            int4 w[2], x[4];
#pragma unroll
            for (int a = 0; a < 2; ++a) w[a] = *reinterpret_cast<const int4 *>(&sw[tr + 32 * a][k]);
#pragma unroll
            for (int b = 0; b < 4; ++b) x[b] = *reinterpret_cast<const int4 *>(&sxq[tt + b][k]);
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    dot[a][b] = __dp4a(w[a].x, x[b].x, dot[a][b]);
                    dot[a][b] = __dp4a(w[a].y, x[b].y, dot[a][b]);
                    dot[a][b] = __dp4a(w[a].z, x[b].z, dot[a][b]);
                    dot[a][b] = __dp4a(w[a].w, x[b].w, dot[a][b]);
                }
        }
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b)
                acc[a][b] = fmaf(float(dot[a][b]), __fmul_rn(sws[tr + 32 * a], sxs[tt + b]), acc[a][b]);
    }
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int r = r0 + tr + 32 * a, t = t0 + tt + b;
            if (r < d && t < T) {
                const size_t o = size_t(t) * d + r;
                y[o] = res ? __fadd_rn(res[o], acc[a][b]) : acc[a][b];
            }
        }
}

// ---- FP32 GEMV (FloatTransformer.cpp:240-382) ------------------------------
// One warp per output row, float4 loads; y = (res ? res : 0) + W.x
__global__ void __launch_bounds__(256)
gemv_f32_kernel(float *y, const float *__restrict__ x, const float *__restrict__ w,
                int n, int d, const float *res) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= d) return;
    const float4 *wr = reinterpret_cast<const float4 *>(w + size_t(row) * n);
    const float4 *xv = reinterpret_cast<const float4 *>(x);
    float acc = 0.f;
    for (int i = lane; i < n / 4; i += 32) {
        const float4 a = wr[i], b = xv[i];
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc);
        acc = fmaf(a.w, b.w, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = res ? __fadd_rn(res[row], acc) : acc;
}

// ---- FP32 GEMM (prompt chunks): Y[t][r] = res + sum_k X[t][k] W[r][k] -------
constexpr int kFR = 64, kFT = 64, kFK = 16;

__global__ void __launch_bounds__(256)
gemm_f32_kernel(float *y, const float *__restrict__ x, const float *__restrict__ w,
                int n, int d, int T, const float *res) {
    __shared__ float sw[kFK][kFR + 4], sx[kFK][kFT + 4];
    const int r0 = blockIdx.x * kFR, t0 = blockIdx.y * kFT;
    const int tr = (threadIdx.x & 15) * 4, tt = (threadIdx.x >> 4) * 4;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < n; k0 += kFK) {
        __syncthreads();
        for (int i = threadIdx.x; i < kFR * kFK; i += 256) {
            const int r = i / kFK, k = i % kFK;
            sw[k][r] = (r0 + r < d && k0 + k < n) ? w[size_t(r0 + r) * n + k0 + k] : 0.f;
            sx[k][r] = (t0 + r < T && k0 + k < n) ? x[size_t(t0 + r) * n + k0 + k] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kFK; ++k) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = sw[k][tr + i];
                b[i] = sx[k][tt + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) acc[i][jj] = fmaf(a[i], b[jj], acc[i][jj]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int r = r0 + tr + i, t = t0 + tt + jj;
            if (r < d && t < T) {
                const size_t o = size_t(t) * d + r;
                y[o] = res ? __fadd_rn(res[o], acc[i][jj]) : acc[i][jj];
            }
        }
}

// ---- SiLU(h1) * h3 (FloatTransformer.cpp:690-728) ---------------------------
__global__ void silu_mul_kernel(float *__restrict__ h, const float *__restrict__ h3, size_t n) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) {
        float v = h[i];
        v = __fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))));
        h[i] = __fmul_rn(v, h3[i]);
    }
}

// ---- greedy argmax (Sampler.cpp:20-68) -------------------------------------
// The reference keeps 8 lanes (index i in lane i % 8, first strict maximum
// per lane), then takes lanes 0..7 in order with a strict '>', then the
// tail past the last multiple of 8.  Equivalent total order used here:
// larger value; then lane (i % 8, tail indices after every lane); then the
// smaller index.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi, int n8) {
    if (v != bv) return v > bv;
    const int li = i < n8 ? (i & 7) : 8, lb = bi < n8 ? (bi & 7) : 8;
    if (li != lb) return li < lb;
    return i < bi;
}

__global__ void argmax_kernel(int *__restrict__ out, const float *__restrict__ v, int n) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const int n8 = n & ~7;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (bi == 0x7fffffff || better(v[i], i, bv, bi, n8)) {
            bv = v[i];
            bi = i;
        }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi != 0x7fffffff && (bi == 0x7fffffff || better(ov, oi, bv, bi, n8))) {
            bv = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < int(blockDim.x >> 5); ++w)
            if (si[w] != 0x7fffffff && (si[0] == 0x7fffffff || better(sv[w], si[w], sv[0], si[0], n8))) {
                sv[0] = sv[w];
                si[0] = si[w];
            }
        *out = si[0];
    }
}

// ---- synthetic weights -------------------------------------------------------
// N(mean 0, std) from a counter-based hash (splitmix64) and Box-Muller.
__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void synth_normal_kernel(float *__restrict__ w, size_t n, uint64_t seed, float std,
                                    float fill) {
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n) return;
    if (std == 0.f) {
        w[i] = fill;
        return;
    }
    const uint64_t h = splitmix64(seed ^ (i * 0xD1B54A32D192ED03ull));
    const float u1 = (float((h >> 40) & 0xFFFFFF) + 1.0f) * (1.0f / 16777217.0f);
    const float u2 = float((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    w[i] = std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

}  // namespace

int embed(cudaStream_t st, float *x, const float *emb_f32, const int8_t *emb_q, const float *emb_s,
          const int *tok_dev, int n, int dim, int gs) {
    if (emb_f32)
        embed_f32_kernel<<<n, 256, 0, st>>>(x, emb_f32, tok_dev, dim);
    else
        embed_q8_kernel<<<n, 256, 0, st>>>(x, emb_q, emb_s, tok_dev, dim, gs);
    return cuda_status(cudaGetLastError(), "embed");
}

int rmsnorm(cudaStream_t st, float *o, const float *x, const float *w, int rows, int dim) {
    rmsnorm_kernel<<<rows, 256, 0, st>>>(o, x, w, dim);
    return cuda_status(cudaGetLastError(), "rmsnorm");
}

int quantize(cudaStream_t st, int8_t *q, float *s, const float *x, size_t n, int gs) {
    const size_t groups = (n + gs - 1) / gs;
    const int threads = 256;
    const size_t blocks = (groups * 32 + threads - 1) / threads;
    quantize_kernel<<<unsigned(blocks), threads, 0, st>>>(q, s, x, n, gs);
    return cuda_status(cudaGetLastError(), "quantize");
}

int gemv_q8(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
            const float *ws, int n, int d, const float *res) {
    const size_t ng1 = size_t(n / 64) + 1;
    const size_t smem = ((n + 15) & ~15) + 2 * kQRows * ng1 * 4 + size_t(n / 64) * 4;
    if (n % 64 != 0) {
        set_error("gemv_q8: n %d is not a multiple of 64", n);
        return LEAP_ERR_INVALID;
    }
    // x and the per-row partials live in shared memory; beyond ~40k columns the
    // tiled kernel (same accumulation order) takes over.
    if (smem > 200 * 1024) return gemm_q8(st, y, xq, xs, wq, ws, n, d, 1, res);
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(
            gemv_q8_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return cuda_status(e, "cudaFuncSetAttribute(gemv_q8)");
        attr[dev] = true;
    }
    gemv_q8_kernel<<<(d + kQRows - 1) / kQRows, kQThreads, smem, st>>>(y, xq, xs, wq, ws, n, d, res);
    return cuda_status(cudaGetLastError(), "gemv_q8");
}

int gemm_q8(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
            const float *ws, int n, int d, int T, const float *res) {
    dim3 grid((d + kGR - 1) / kGR, (T + kGT - 1) / kGT);
    gemm_q8_kernel<<<grid, kGThreads, 0, st>>>(y, xq, xs, wq, ws, n, d, T, res);
    return cuda_status(cudaGetLastError(), "gemm_q8");
}

int gemv_f32(cudaStream_t st, float *y, const float *x, const float *w, int n, int d,
             const float *res) {
    gemv_f32_kernel<<<(d + 7) / 8, 256, 0, st>>>(y, x, w, n, d, res);
    return cuda_status(cudaGetLastError(), "gemv_f32");
}

int gemm_f32(cudaStream_t st, float *y, const float *x, const float *w, int n, int d, int T,
             const float *res) {
    dim3 grid((d + kFR - 1) / kFR, (T + kFT - 1) / kFT);
    gemm_f32_kernel<<<grid, 256, 0, st>>>(y, x, w, n, d, T, res);
    return cuda_status(cudaGetLastError(), "gemm_f32");
}

int silu_mul(cudaStream_t st, float *h, const float *h3, size_t n) {
    silu_mul_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(h, h3, n);
    return cuda_status(cudaGetLastError(), "silu_mul");
}

int argmax(cudaStream_t st, int *out, const float *v, int n) {
    argmax_kernel<<<1, 1024, 0, st>>>(out, v, n);
    return cuda_status(cudaGetLastError(), "argmax");
}

int synth_normal(cudaStream_t st, float *w, size_t n, uint64_t seed, float std, float fill) {
    synth_normal_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(w, n, seed, std, fill);
    return cuda_status(cudaGetLastError(), "synth_normal");
}

}  // namespace eng
}  // namespace leap
