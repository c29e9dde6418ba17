// engine_kernels.cu — the support ops around attention in the forward pass
// (src/inference/FloatTransformer.cpp:384-797 and
// src/inference/QuantizedTransformer.cpp:654-1061), on the GPU.
//
// Embedding gather, RMSNorm (optionally fused with the activation
// quantization that follows it), FP32 GEMV/GEMM, per-group activation
// quantization, the W8A8 GEMV/GEMM, SiLU*up (optionally fused with its
// quantization), residual adds, greedy argmax, and a synthetic weight
// generator.  Two reproduce the reference's compiled arithmetic bit for bit:
// the activation quantization (scale = max * (1/127), id = 127/max, round
// half away from zero) and the W8A8 dot (int32 group dots, then per output
// val = fma(float(ival), w_s * x_s, val) over the groups in order).
//
// Batch-1 decode runs ~10 of these kernels per layer back to back, so the
// decode-path kernels use programmatic dependent launch: each is launched
// while its predecessor still runs, may read only constant data (weights)
// before griddepcontrol.wait, and lets its own successor launch once it has
// passed that wait.  The GEMVs use the window to start their weight stream.
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <vector>

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

__device__ __forceinline__ int4 ld_stream(const int4 *p) { return __ldcs(p); }
__device__ __forceinline__ float4 ld_stream(const float4 *p) { return __ldcs(p); }

// Programmatic dependent launch: wait for the predecessor kernel's results,
// then allow the successor to start launching.
__device__ __forceinline__ void pdl_enter() {
    grid_dependency_wait();
    grid_launch_dependents();
}

// One 64-value quantization group held as one float4 by each of 16
// consecutive lanes (QuantizedTransformer.cpp:338-357 as compiled:
// scale = max * (1/127), id = 127 / max, q = round half away (x * id)).
// Every lane of the warp must call it (shuffles over the full warp).
__device__ __forceinline__ void quantize16(float4 v, bool valid, char4 *q4, float *s, size_t i4) {
    float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float inv127 = 1.0f / 127.0f;
    const float scale = __fmul_rn(mx, inv127);
    const float id = scale != 0.f ? __fdiv_rn(127.0f, mx) : 0.f;
    if (!valid) return;
    q4[i4] = make_char4(static_cast<signed char>(roundf(__fmul_rn(v.x, id))),
                        static_cast<signed char>(roundf(__fmul_rn(v.y, id))),
                        static_cast<signed char>(roundf(__fmul_rn(v.z, id))),
                        static_cast<signed char>(roundf(__fmul_rn(v.w, id))));
    if ((i4 & 15) == 0) s[i4 >> 4] = scale;
}

// ---- embedding -------------------------------------------------------------
// FloatTransformer.cpp:758-759 (copy of the row); W8A8 engines dequantize the
// table at load (QuantizedTransformer.cpp:116-117, :136-216): q * s.  Token
// ids come from the device (a pipeline's last stage may have produced them):
// an id outside [0, vocab) reads row 0 and raises the error word.
__device__ __forceinline__ int checked_token(const int *tok, int row, int vocab, int *err) {
    const int t = tok[row];
    if (t >= 0 && t < vocab) return t;
    if (threadIdx.x == 0) report_error(err, kDevErrBadToken);
    return 0;
}

__global__ void embed_f32_kernel(float *__restrict__ x, const float *__restrict__ emb,
                                 const int *__restrict__ tok, int dim, int vocab, int *err) {
    pdl_enter();
    const int row = blockIdx.x;
    const float *src = emb + size_t(checked_token(tok, row, vocab, err)) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) x[size_t(row) * dim + i] = src[i];
}

__global__ void embed_q8_kernel(float *__restrict__ x, const int8_t *__restrict__ q,
                                const float *__restrict__ s, const int *__restrict__ tok,
                                int dim, int gs, int vocab, int *err) {
    pdl_enter();
    const int row = blockIdx.x;
    const size_t base = size_t(checked_token(tok, row, vocab, err)) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x)
        x[size_t(row) * dim + i] = float(q[base + i]) * s[(base + i) / gs];
}

// ---- RMSNorm (FloatTransformer.cpp:79-214), optionally + quantize ----------
// o = w * (r * x), r = 1/sqrt(mean(x^2) + 1e-5).  The reference's AVX2 path
// refines an rsqrt estimate by one Newton step; 1/sqrtf is within 2e-7.
// One CTA per row, one float4 per thread per pass.  QUANT: the normalised
// row is quantized in groups of 64 (q, s) instead of being stored (the
// W8A8 engine only consumes it quantized, QuantizedTransformer.cpp:925-951).
template <bool QUANT>
__global__ void __launch_bounds__(1024)
rmsnorm_kernel(float *o, char4 *q4, float *s, const float *x,  // o may alias x
               const float *__restrict__ w, int dim) {
    pdl_enter();
    __shared__ float red[32];
    const int row = blockIdx.x, n4 = dim >> 2;
    const float4 *xr = reinterpret_cast<const float4 *>(x + size_t(row) * dim);
    const float4 *w4 = reinterpret_cast<const float4 *>(w);
    float ss = 0.f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = xr[i];
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
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
    const int lim = (n4 + 31) & ~31;  // whole warps take part in the group shuffles
    for (int i = threadIdx.x; i < lim; i += blockDim.x) {
        const bool valid = i < n4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) {
            const float4 xv = xr[i], wv = w4[i];
            v = make_float4(wv.x * (r * xv.x), wv.y * (r * xv.y), wv.z * (r * xv.z),
                            wv.w * (r * xv.w));
        }
        if (QUANT)
            quantize16(v, valid, q4 + size_t(row) * n4, s + size_t(row) * (dim >> 6), size_t(i));
        else if (valid)
            reinterpret_cast<float4 *>(o + size_t(row) * dim)[i] = v;
    }
}

// ---- activation quantization (QuantizedTransformer.cpp:338-357) ------------
// Any group size <= 128: one warp per group.
__global__ void quantize_kernel(int8_t *__restrict__ q, float *__restrict__ s,
                                const float *__restrict__ x, size_t n, int gs) {
    pdl_enter();
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

// Group size 64: one float4 per thread, 16 lanes per group.
__global__ void quantize64_kernel(char4 *__restrict__ q4, float *__restrict__ s,
                                  const float *__restrict__ x, size_t n4) {
    pdl_enter();
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;  // grid covers whole warps
    const bool valid = i < n4;
    const float4 v = valid ? reinterpret_cast<const float4 *>(x)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    quantize16(v, valid, q4, s, i);
}

// ---- W8A8 GEMV (QuantizedTransformer.cpp:359-652) --------------------------
// y[r] = (res ? res[r] : 0) + sum_g fma-chain(float(idot_g), ws[r,g]*xs[g]);
// y may alias res (the residual add x += W.v), so neither is __restrict__.
// A CTA takes kQR rows, two per warp.  Phase 1 streams the int8 rows with
// kGemvUnroll 16-byte loads in flight per lane and row (the first batch is
// issued before griddepcontrol.wait: weights do not depend on the previous
// kernel); a 64-wide group is 4 consecutive chunks on 4 consecutive lanes,
// whose dp4a partial dots meet by two xor-shuffles and go to shared memory
// as float(int32 dot).  Phase 2 runs each row's chain over the groups in
// order in one thread, as the reference's loop does.
constexpr int kQR = 16;
constexpr int kGemvWarps = 8;
constexpr int kGemvUnroll = 8;

__device__ __forceinline__ void q8_group_dots(const int4 (&w)[kGemvUnroll], const int4 *sx, int nch,
                                              int base, int lane, float *sdot_row) {
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
        const int c = base + u * 32 + lane;
        int dot = 0;
        if (c < nch) {
            const int4 xv = sx[c];
            dot = __dp4a(w[u].x, xv.x, dot);
            dot = __dp4a(w[u].y, xv.y, dot);
            dot = __dp4a(w[u].z, xv.z, dot);
            dot = __dp4a(w[u].w, xv.w, dot);
        }
        dot += __shfl_xor_sync(0xffffffffu, dot, 1);
        dot += __shfl_xor_sync(0xffffffffu, dot, 2);
        if ((lane & 3) == 0 && c < nch) sdot_row[c >> 2] = float(dot);
    }
}

__device__ __forceinline__ void q8_load(int4 (&w)[kGemvUnroll], const int4 *wr, bool row_ok, int nch,
                                        int base, int lane) {
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
        const int c = base + u * 32 + lane;
        w[u] = (row_ok && c < nch) ? ld_stream(wr + c) : make_int4(0, 0, 0, 0);
    }
}

__global__ void __launch_bounds__(kGemvWarps * 32)
gemv_q8_kernel(float *y, const int8_t *__restrict__ xq, const float *__restrict__ xs,
               const int8_t *__restrict__ wq, const float *__restrict__ ws, int n, int d,
               const float *res) {
    extern __shared__ int4 smx[];
    const int nch = n >> 4, ng = n >> 6, ng1 = ng | 1;  // odd stride: phase 2 is conflict-free
    int4 *sx = smx;                                      // [nch] x chunks
    float *sxs = reinterpret_cast<float *>(sx + nch);    // [ng]
    float *sdot = sxs + ng;                              // [kQR][ng1] float(int32 dot)
    float *st = sdot + kQR * ng1;                        // [kQR][ng1] ws * xs
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int r0 = blockIdx.x * kQR;
    const int ra = r0 + warp, rb = r0 + warp + kGemvWarps;
    const bool oka = ra < d, okb = rb < d;
    const int4 *wa = reinterpret_cast<const int4 *>(wq + size_t(oka ? ra : 0) * n);
    const int4 *wb = reinterpret_cast<const int4 *>(wq + size_t(okb ? rb : 0) * n);
    int4 pa[kGemvUnroll], pb[kGemvUnroll];
    q8_load(pa, wa, oka, nch, 0, lane);
    q8_load(pb, wb, okb, nch, 0, lane);
    pdl_enter();
    for (int i = threadIdx.x; i < nch; i += blockDim.x) sx[i] = reinterpret_cast<const int4 *>(xq)[i];
    for (int g = threadIdx.x; g < ng; g += blockDim.x) sxs[g] = xs[g];
    __syncthreads();
    for (int i = threadIdx.x; i < kQR * ng; i += blockDim.x) {
        const int rr = i / ng, g = i - rr * ng;
        st[rr * ng1 + g] = (r0 + rr < d) ? __fmul_rn(ws[size_t(r0) * ng + i], sxs[g]) : 0.f;
    }
    for (int base = 0; base < nch; base += 32 * kGemvUnroll) {
        if (base > 0) {
            q8_load(pa, wa, oka, nch, base, lane);
            q8_load(pb, wb, okb, nch, base, lane);
        }
        q8_group_dots(pa, sx, nch, base, lane, sdot + warp * ng1);
        q8_group_dots(pb, sx, nch, base, lane, sdot + (warp + kGemvWarps) * ng1);
    }
    __syncthreads();
    if (threadIdx.x < kQR && r0 + threadIdx.x < d) {
        const float *dr = sdot + threadIdx.x * ng1, *tr = st + threadIdx.x * ng1;
        float val = 0.f;
#pragma unroll 8
        for (int g = 0; g < ng; ++g) val = fmaf(dr[g], tr[g], val);
        const int row = r0 + threadIdx.x;
        y[row] = res ? __fadd_rn(res[row], val) : val;
    }
}

// ---- W8A8 GEMV, one row per lane ------------------------------------------
// The same arithmetic as gemv_q8_kernel.  A CTA takes kSR rows; its 8 warps
// split each row's groups into kSK contiguous slices (two per warp: lanes
// 0..15 and 16..31), so lane (row r, slice k) computes the int32 dots of
// row r's groups in slice k by itself — 16 dp4a over 4 chunks per group, no
// shuffles — with kSU 16-byte loads in flight, and writes float(dot) and
// ws*xs into a [row][group] table in shared memory.  Then kSR lanes run the
// rows' chains over all groups, in order.  The first loads are issued
// before griddepcontrol.wait.  (Measured end to end on the 8B decode step,
// this beats both a persistent variant of it and the register-staged
// kernel: its 64 registers let 4 CTAs per SM start their weight stream
// while the previous kernel still runs.)
constexpr int kSR = 16;   // rows per CTA
constexpr int kSK = 16;   // slices of a row's groups per CTA (2 per warp)
constexpr int kSU = 8;    // chunks (16 bytes) in flight per lane

__global__ void __launch_bounds__(256, 4)
gemv_q8_slice_kernel(float *y, const int8_t *__restrict__ xq, const float *__restrict__ xs,
                     const int8_t *__restrict__ wq, const float *__restrict__ ws, int n, int d,
                     const float *res) {
    extern __shared__ int4 ssm[];
    const int nch = n >> 4, ng = n >> 6, ng1 = ng | 1;
    int4 *sx = ssm;                                     // [nch]
    float *sxs = reinterpret_cast<float *>(sx + nch);   // [ng]
    float *tdot = sxs + ng;                             // [kSR][ng1]
    float *tt = tdot + kSR * ng1;                       // [kSR][ng1]
    const int tid = threadIdx.x, lane = tid & 31;
    const int rr = lane & (kSR - 1), k = (tid >> 5) * 2 + (lane >> 4);
    const int row = blockIdx.x * kSR + rr;
    const bool ok = row < d;
    const int g0 = k * ng / kSK, g1 = (k + 1) * ng / kSK;  // this lane's groups
    const int c0 = 4 * g0, c1 = 4 * g1;                     // and chunks
    const int4 *wr = reinterpret_cast<const int4 *>(wq + size_t(ok ? row : 0) * n);
    const float *wsr = ws + size_t(ok ? row : 0) * ng;
    int4 w[kSU];
#pragma unroll
    for (int u = 0; u < kSU; ++u) w[u] = (ok && c0 + u < c1) ? __ldg(wr + c0 + u) : make_int4(0, 0, 0, 0);
    pdl_enter();
    for (int i = tid; i < nch; i += blockDim.x) sx[i] = reinterpret_cast<const int4 *>(xq)[i];
    for (int g = tid; g < ng; g += blockDim.x) sxs[g] = xs[g];
    __syncthreads();
    for (int cb = c0; cb < c1; cb += kSU) {  // kSU % 4 == 0: whole groups per batch
        if (cb > c0) {
#pragma unroll
            for (int u = 0; u < kSU; ++u)
                w[u] = (ok && cb + u < c1) ? __ldg(wr + cb + u) : make_int4(0, 0, 0, 0);
        }
#pragma unroll
        for (int q = 0; q < kSU / 4; ++q) {
            const int g = (cb >> 2) + q;
            if (g < g1) {
                int dot = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int4 xv = sx[4 * g + j];
                    const int4 wv = w[4 * q + j];
                    dot = __dp4a(wv.x, xv.x, dot);
                    dot = __dp4a(wv.y, xv.y, dot);
                    dot = __dp4a(wv.z, xv.z, dot);
                    dot = __dp4a(wv.w, xv.w, dot);
                }
                tdot[rr * ng1 + g] = float(dot);
                tt[rr * ng1 + g] = ok ? __fmul_rn(__ldg(wsr + g), sxs[g]) : 0.f;
            }
        }
    }
    __syncthreads();
    if (tid < kSR && blockIdx.x * kSR + tid < d) {
        const float *dr = tdot + tid * ng1, *tr = tt + tid * ng1;
        float val = 0.f;
#pragma unroll 8
        for (int g = 0; g < ng; ++g) val = fmaf(dr[g], tr[g], val);
        const int r = blockIdx.x * kSR + tid;
        y[r] = res ? __fadd_rn(res[r], val) : val;
    }
}

// ---- W8A8 GEMV, persistent bulk-copy pipeline -------------------------------
// Work = (block of 8 rows, 2048-byte column chunk) items, taken in order by
// a persistent CTA (blocks blockIdx.x, +gridDim.x, ...).  An item's 8 row
// chunks move with one 1-D bulk copy each into one of kPS stages.  Ten warps:
//   warps 0-7  one group dot each per item (warp w = row w, lane l = group l
//              of the chunk; the lane's four 16-byte reads are rotated so a
//              quarter-warp touches eight bank groups) into a [row][group]
//              table (two buffers), then release the stage;
//   warp 8     issues the copies, each as soon as its stage is released
//              (the first kPre before griddepcontrol.wait: weights are
//              constant);
//   warp 9     prefetches the next block's weight scales with cp.async and
//              runs each row's chain
//              val = fma(float(dot), w_s * x_s, val) through the chunk's
//              groups in order — the reference's arithmetic — while the dot
//              warps already work on the next item.
// All hand-offs are mbarriers; every wait is bounded.
constexpr int kPR = 8;                   // rows per block = dot warps
constexpr int kPK = 2048;                // bytes of a row per item
constexpr int kPS = 3;                   // stages
constexpr int kPre = 1;                  // stages requested before griddepcontrol.wait
constexpr int kPG = kPK / 64;            // groups per item = lanes
constexpr int kPStage = kPR * kPK;       // bytes per stage
constexpr int kPThreads = 32 * (kPR + 2);

__device__ __forceinline__ void cp_async4(void *dst_smem, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst_smem)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst_smem, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst_smem)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// The activation comes in one of three forms (PRO):
//   kProQ8     x already quantized (xq, xs);
//   kProNorm   fp32 x and a norm weight: the CTA computes rmsnorm_kernel's
//              normalised row and its 64-groups quantization itself, in
//              rmsnorm_kernel's operation order (its sum of squares runs as
//              that kernel's row_threads(n) threads would: thread t sums
//              float4s t, t + T, ... with fmas, warps reduce by xor
//              shuffles, then the warp sums), so q/s are bit-identical to
//              leap_op_rmsnorm_quantize's and the separate kernel goes away;
//   kProQuant  fp32 x quantized as quantize64_kernel does.
// The last two take n <= 4096, held in the dot warps' registers.
constexpr int kProQ8 = 0, kProNorm = 1, kProQuant = 2;
constexpr int kXV = 4;  // float4s of x per dot-warp thread: n <= 32 * kPR * kXV * 4 = 4096

template <int PRO>
__global__ void __launch_bounds__(kPThreads)
gemv_q8_stream_kernel(float *y, const int8_t *__restrict__ xq, const float *__restrict__ xs,
                      const float *__restrict__ xf, const float *__restrict__ nw,
                      const int8_t *__restrict__ wq, const float *__restrict__ ws, int n, int d,
                      const float *res, int *err) {
    extern __shared__ __align__(128) unsigned char psm[];
    const int ng = n >> 6;
    unsigned char *stg = psm;                                    // [kPS][kPR][kPK]
    int4 *sx = reinterpret_cast<int4 *>(psm + kPS * kPStage);     // [n / 16]
    float *sxs = reinterpret_cast<float *>(sx + (n >> 4));       // [ng]
    float *sws = sxs + ng;                                       // [2][kPR][ng]
    __shared__ uint64_t full[kPS], empty[kPS], ready[2], done[2];
    __shared__ float tab[2][kPR][kPG + 1];
    __shared__ int issued, failed;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nblocks = (d + kPR - 1) / kPR;
    const int nchunks = (n + kPK - 1) / kPK;

    // ---- work: row blocks blockIdx.x, +gridDim.x, ..., each in nchunks items.
    // Each role walks its items with a (block, chunk) cursor instead of
    // dividing the item index by the chunk count per item (measured 8 %
    // faster on the 8B decode step).
    const int my_blocks = blockIdx.x < nblocks ? (nblocks - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int items = my_blocks * nchunks;
    auto block_of = [&](int k) { return blockIdx.x + k * gridDim.x; };
    struct Cursor {  // item = (row block rb, chunk c)
        int rb = 0, c = 0;
    };
    auto advance = [&](Cursor &u) {
        if (++u.c == nchunks) {
            u.c = 0;
            u.rb += gridDim.x;
        }
    };
    auto rows_of = [&](int rb) { return min(kPR, d - rb * kPR); };
    auto issue = [&](int it, const Cursor &u) {  // producer warp: item `it` into stage it % kPS
        const int s = it % kPS, rb = u.rb, c = u.c;
        const int k0 = c * kPK, nr = rows_of(rb);
        const uint32_t kb = uint32_t(min(kPK, n - k0));
        if (lane == 0) mbar_arrive_expect_tx(&full[s], kb * uint32_t(nr));
        __syncwarp();
        if (lane < nr)
            bulk_g2s(stg + s * kPStage + lane * kPK, wq + size_t(rb * kPR + lane) * n + k0, kb,
                     &full[s]);
        if (lane == 0) issued = it + 1;
    };
    auto fetch_scales = [&](int k) {  // chain warp: block k's weight scales -> sws[k & 1]
        if (k >= my_blocks) return;
        const int rb = block_of(k);
        const float *src = ws + size_t(rb) * kPR * ng;
        float *dst = sws + (k & 1) * kPR * ng;
        for (int i = lane; i < rows_of(rb) * ng; i += 32) cp_async4(dst + i, src + i);
    };

    if (tid == 0) {
        for (int s = 0; s < kPS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kPR);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ready[b], kPR);
            mbar_init(&done[b], 1);
        }
        issued = 0;
        failed = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // Only kPre stages are requested before the dependency wait, the rest
    // right after it: what is requested after the wait (x) queues behind the
    // weight bytes still in flight (8B W8A8 decode step: 2.40 ms with one
    // stage before the wait, 2.44 ms with two).
    if (warp == kPR) {
        Cursor u;
        u.rb = blockIdx.x;
        for (int it = 0; it < min(kPre, items); ++it, advance(u)) issue(it, u);
    }
    if (warp == kPR + 1) fetch_scales(0);
    auto issue_rest = [&]() {  // producer warp: stages kPre .. kPS-1
        Cursor u;
        u.rb = blockIdx.x;
        for (int it = 0; it < min(kPre, items); ++it) advance(u);
        for (int it = kPre; it < min(kPS, items); ++it, advance(u)) issue(it, u);
    };
    if (PRO != kProQ8) {
        // x (and the norm weight) in registers: dot-warp thread (warp, lane)
        // holds float4s (warp + 8 k) * 32 + lane, k < kXV, i.e. for k it is
        // lane `lane` of rmsnorm_kernel's warp warp + 8 k (n <= 4096: that
        // kernel's threads then hold one float4 each)
        const int n4 = n >> 2;
        const float4 *x4 = reinterpret_cast<const float4 *>(xf);
        float4 xv[kXV], wv[kXV];
        if (PRO == kProNorm && warp < kPR) {  // the norm weight is constant
#pragma unroll
            for (int k = 0; k < kXV; ++k) {
                const int i = (warp + kPR * k) * 32 + lane;
                wv[k] = i < n4 ? reinterpret_cast<const float4 *>(nw)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        pdl_enter();
        __shared__ float red[32];
        if (warp == kPR) {
            issue_rest();
        } else if (warp < kPR) {
#pragma unroll
            for (int k = 0; k < kXV; ++k) {
                const int i = (warp + kPR * k) * 32 + lane;
                xv[k] = i < n4 ? x4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            if (PRO == kProNorm) {
                // rmsnorm_kernel's per-thread fma chain and warp reduction
#pragma unroll
                for (int k = 0; k < kXV; ++k) {
                    const int vw = warp + kPR * k;
                    if (vw * 32 >= n4) break;  // warp-uniform
                    float ss = 0.f;
                    ss = fmaf(xv[k].x, xv[k].x, ss);
                    ss = fmaf(xv[k].y, xv[k].y, ss);
                    ss = fmaf(xv[k].z, xv[k].z, ss);
                    ss = fmaf(xv[k].w, xv[k].w, ss);
                    ss = warp_sum(ss);
                    if (lane == 0) red[vw] = ss;
                }
            }
        }
        if (PRO == kProNorm) __syncthreads();
        if (warp < kPR) {
            float r = 1.f;
            if (PRO == kProNorm) {
                // that kernel's second reduction over its n4 / 32 warp sums
                // (rounded up; every lane ends the xor reduction with the same
                // value)
                const int nvw = (n4 + 31) >> 5;
                const float tot = warp_sum(lane < nvw ? red[lane] : 0.f);
                float m = tot / float(n);
                m += 1e-5f;
                r = 1.0f / sqrtf(m);
            }
#pragma unroll
            for (int k = 0; k < kXV; ++k) {
                const int i = (warp + kPR * k) * 32 + lane;
                if ((warp + kPR * k) * 32 >= n4) break;  // whole warps take part in the shuffles
                const bool valid = i < n4;
                float4 v = xv[k];
                if (PRO == kProNorm)
                    v = make_float4(wv[k].x * (r * v.x), wv[k].y * (r * v.y), wv[k].z * (r * v.z),
                                    wv[k].w * (r * v.w));
                quantize16(v, valid, reinterpret_cast<char4 *>(sx), sxs, size_t(i));
            }
        }
        __syncthreads();
    } else {
        pdl_enter();
        if (warp == kPR) {
            issue_rest();
        } else if (warp < kPR) {
            // x and its scales as asynchronous copies, all in flight at once
            // (a load-then-store loop waits one L2 round trip per
            // iteration), by the dot warps only: the chain warp's scale
            // copies, issued before the wait, may still be queued behind
            // weight bytes and need not have landed here
            const int nt = kPR * 32;
            for (int i = tid; i < (n >> 4); i += nt)
                cp_async16(sx + i, reinterpret_cast<const int4 *>(xq) + i);
            for (int g = tid; g < ng; g += nt) cp_async4(sxs + g, xs + g);
            cp_async_wait_all();
        }
        __syncthreads();
    }

    if (warp < kPR) {
        // ---- dot warps ------------------------------------------------------
        const int rot = (lane >> 1) & 3;
        Cursor u;
        u.rb = blockIdx.x;
        for (int it = 0; it < items; ++it, advance(u)) {
            const int s = it % kPS, b = it & 1, c = u.c;
            const int gcount = min(kPK, n - c * kPK) >> 6;
            bool ok = mbar_wait(&full[s], uint32_t(it / kPS) & 1u);
            if (ok && it >= 2) ok = mbar_wait(&done[b], uint32_t((it - 2) >> 1) & 1u);
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0) atomicExch(&failed, 1);
                break;
            }
            if (lane < gcount) {
                const int4 *wr = reinterpret_cast<const int4 *>(stg + s * kPStage + warp * kPK + lane * 64);
                const int4 *xr = sx + (c * kPG + lane) * 4;
                // all eight 16-byte operands first, then four independent
                // dp4a chains (integer sums: exact in any order)
                int4 wv[4], xv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int cc = (j + rot) & 3;
                    wv[j] = wr[cc];
                    xv[j] = xr[cc];
                }
                int d4[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    d4[j] = __dp4a(wv[j].x, xv[j].x, 0);
                    d4[j] = __dp4a(wv[j].y, xv[j].y, d4[j]);
                    d4[j] = __dp4a(wv[j].z, xv[j].z, d4[j]);
                    d4[j] = __dp4a(wv[j].w, xv[j].w, d4[j]);
                }
                tab[b][warp][lane] = float((d4[0] + d4[1]) + (d4[2] + d4[3]));
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&empty[s]);
                mbar_arrive(&ready[b]);
            }
        }
    } else if (warp == kPR) {
        // ---- producer: refill each stage as soon as the dot warps release it
        bool ok = true;
        Cursor u;
        u.rb = blockIdx.x;
        for (int it = 0; it < min(kPS, items); ++it) advance(u);
        for (int it = kPS; it < items && ok; ++it, advance(u)) {
            ok = __all_sync(0xffffffffu,
                            mbar_wait(&empty[it % kPS], uint32_t((it - kPS) / kPS) & 1u));
            if (ok) issue(it, u);
        }
        if (!ok && lane == 0) atomicExch(&failed, 1);
    } else if (warp == kPR + 1) {
        // ---- chains ---------------------------------------------------------
        int it = 0;
        bool ok = true;
        for (int k = 0; k < my_blocks && ok; ++k) {
            const int rb = block_of(k), nr = rows_of(rb);
            cp_async_wait_all();  // this block's scales (issued a block ago)
            __syncwarp();
            fetch_scales(k + 1);
            const float *wsr = sws + (k & 1) * kPR * ng + lane * ng;
            float val = 0.f;
            for (int c = 0; c < nchunks; ++c, ++it) {
                const int b = it & 1, g0 = c * kPG;
                const int gcount = min(kPK, n - c * kPK) >> 6;
                ok = __all_sync(0xffffffffu, mbar_wait(&ready[b], uint32_t(it >> 1) & 1u));
                if (!ok) break;
                if (lane < nr) {
                    // the ordered chain over the item's groups; the operands of
                    // 8 steps are loaded first, so only the fmas are serial
                    const float *tr = &tab[b][lane][0];
                    int g = 0;
                    for (; g + 8 <= gcount; g += 8) {
                        float t[8], m[8];
#pragma unroll
                        for (int u = 0; u < 8; ++u) {
                            t[u] = tr[g + u];
                            m[u] = __fmul_rn(wsr[g0 + g + u], sxs[g0 + g + u]);
                        }
#pragma unroll
                        for (int u = 0; u < 8; ++u) val = fmaf(t[u], m[u], val);
                    }
                    for (; g < gcount; ++g)
                        val = fmaf(tr[g], __fmul_rn(wsr[g0 + g], sxs[g0 + g]), val);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&done[b]);
            }
            if (!ok) break;
            if (lane < nr) {
                const int r = rb * kPR + lane;
                y[r] = res ? __fadd_rn(res[r], val) : val;
            }
        }
        cp_async_wait_all();
        if (!ok && lane == 0) atomicExch(&failed, 1);
    }
    __syncthreads();
    if (failed) {
        // a wait gave up: let the copies in flight land, then report
        for (int i2 = max(0, issued - kPS); i2 < issued; ++i2)
            (void)mbar_wait(&full[i2 % kPS], uint32_t(i2 / kPS) & 1u);
        if (tid == 0) report_error(err, kDevWaitTimeout);
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
// One warp per row (grid-stride), kGemvUnroll float4 weight loads in flight
// per lane, x in shared memory (asynchronous copies, all in flight at once);
// y = (res ? res : 0) + W.a.  The first row's first batch of weights is
// loaded before griddepcontrol.wait.  a = x, or (NORM) rmsnorm_kernel's
// normalised row w * (r * x), formed in shared memory by this CTA with that
// kernel's operation order (its sum of squares as its row_threads(n)
// threads would run it), so the separate RMSNorm launch goes away and the
// bits stay the same.
template <bool NORM>
__global__ void __launch_bounds__(kGemvWarps * 32)
gemv_f32_kernel(float *y, const float *__restrict__ x, const float *__restrict__ nw,
                const float *__restrict__ w, int n, int d, const float *res) {
    extern __shared__ float4 sx4[];  // [n4] x (normalised); NORM: then [n4] norm weight
    const int n4 = n >> 2;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int row = blockIdx.x * kGemvWarps + warp;
    float4 a[kGemvUnroll];
    {
        const float4 *wr = reinterpret_cast<const float4 *>(w + size_t(row < d ? row : 0) * n);
#pragma unroll
        for (int u = 0; u < kGemvUnroll; ++u) {
            const int c = u * 32 + lane;
            a[u] = (row < d && c < n4) ? ld_stream(wr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    if (NORM)  // the norm weight is constant
        for (int i = threadIdx.x; i < n4; i += blockDim.x)
            cp_async16(sx4 + n4 + i, reinterpret_cast<const float4 *>(nw) + i);
    pdl_enter();
    for (int i = threadIdx.x; i < n4; i += blockDim.x)
        cp_async16(sx4 + i, reinterpret_cast<const float4 *>(x) + i);
    cp_async_wait_all();
    __syncthreads();
    if (NORM) {
        __shared__ float red[32];
        const int T = min(1024, max(32, ((n4 + 31) / 32) * 32));  // rmsnorm_kernel's block
        for (int vw = warp; vw < (T >> 5); vw += kGemvWarps) {
            float ss = 0.f;
            for (int i = vw * 32 + lane; i < n4; i += T) {
                const float4 v = sx4[i];
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
            ss = warp_sum(ss);
            if (lane == 0) red[vw] = ss;
        }
        __syncthreads();
        // every lane ends the xor reduction with the same sum
        const float tot = warp_sum(lane < (T >> 5) ? red[lane] : 0.f);
        float m = tot / float(n);
        m += 1e-5f;
        const float r = 1.0f / sqrtf(m);
        for (int i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 xv = sx4[i], wv = sx4[n4 + i];
            sx4[i] = make_float4(wv.x * (r * xv.x), wv.y * (r * xv.y), wv.z * (r * xv.z),
                                 wv.w * (r * xv.w));
        }
        __syncthreads();
    }
    for (; row < d; row += gridDim.x * kGemvWarps) {
        const float4 *wr = reinterpret_cast<const float4 *>(w + size_t(row) * n);
        float acc = 0.f;
        for (int base = 0; base < n4; base += 32 * kGemvUnroll) {
            if (base > 0 || row != int(blockIdx.x * kGemvWarps + warp)) {
#pragma unroll
                for (int u = 0; u < kGemvUnroll; ++u) {
                    const int c = base + u * 32 + lane;
                    a[u] = c < n4 ? ld_stream(wr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u) {
                const int c = base + u * 32 + lane;
                if (c < n4) {
                    const float4 b = sx4[c];
                    acc = fmaf(a[u].x, b.x, acc);
                    acc = fmaf(a[u].y, b.y, acc);
                    acc = fmaf(a[u].z, b.z, acc);
                    acc = fmaf(a[u].w, b.w, acc);
                }
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) y[row] = res ? __fadd_rn(res[row], acc) : acc;
    }
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

// ---- SiLU(h1) * h3 (FloatTransformer.cpp:690-728), optionally + quantize --
// (val * (1 / (1 + exp(-val)))) * h3 per element; QUANT quantizes the
// result in groups of 64 (QuantizedTransformer.cpp:953-997) instead of
// storing it.
template <bool QUANT>
__global__ void silu_mul_kernel(float *h, char4 *q4, float *s, const float *__restrict__ h3,
                                size_t n4) {
    pdl_enter();
    const size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x;  // grid covers whole warps
    const bool valid = i < n4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid) {
        const float4 a = reinterpret_cast<const float4 *>(h)[i];
        const float4 b = reinterpret_cast<const float4 *>(h3)[i];
        auto f = [](float t, float u) {
            return __fmul_rn(__fmul_rn(t, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-t)))), u);
        };
        v = make_float4(f(a.x, b.x), f(a.y, b.y), f(a.z, b.z), f(a.w, b.w));
    }
    if (QUANT)
        quantize16(v, valid, q4, s, i);
    else if (valid)
        reinterpret_cast<float4 *>(h)[i] = v;
}

// ---- greedy argmax (Sampler.cpp:20-68) -------------------------------------
// The reference keeps 8 lanes (index i in lane i % 8, first strict maximum
// per lane), then takes lanes 0..7 in order with a strict '>', then the
// tail past the last multiple of 8.  Equivalent total order used here:
// larger value; then lane (i % 8, tail indices after every lane); then the
// smaller index.  One CTA; each thread keeps 8 float4 loads in flight.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi, int n8) {
    if (v != bv) return v > bv;
    const int li = i < n8 ? (i & 7) : 8, lb = bi < n8 ? (bi & 7) : 8;
    if (li != lb) return li < lb;
    return i < bi;
}

__device__ __forceinline__ void take(float v, int i, float &bv, int &bi, int n8) {
    if (bi == 0x7fffffff || better(v, i, bv, bi, n8)) {
        bv = v;
        bi = i;
    }
}

__global__ void __launch_bounds__(1024) argmax_kernel(int *__restrict__ out, const float *__restrict__ v, int n) {
    pdl_enter();
    __shared__ float sv[32];
    __shared__ int si[32];
    const int n8 = n & ~7;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    const int n4 = ((reinterpret_cast<uintptr_t>(v) & 15) == 0) ? (n >> 2) : 0;
    const float4 *v4 = reinterpret_cast<const float4 *>(v);
    constexpr int U = 8;
    for (int base = 0; base < n4; base += U * int(blockDim.x)) {
        float4 a[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = base + u * int(blockDim.x) + int(threadIdx.x);
            a[u] = j < n4 ? v4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int j = base + u * int(blockDim.x) + int(threadIdx.x);
            if (j < n4) {
                take(a[u].x, 4 * j, bv, bi, n8);
                take(a[u].y, 4 * j + 1, bv, bi, n8);
                take(a[u].z, 4 * j + 2, bv, bi, n8);
                take(a[u].w, 4 * j + 3, bv, bi, n8);
            }
        }
    }
    for (int i = 4 * n4 + threadIdx.x; i < n; i += blockDim.x) take(v[i], i, bv, bi, n8);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi != 0x7fffffff) take(ov, oi, bv, bi, n8);
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < int(blockDim.x >> 5); ++w)
            if (si[w] != 0x7fffffff) take(sv[w], si[w], sv[0], si[0], n8);
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

// Launch with programmatic stream serialization (the kernel calls
// pdl_enter() before touching anything a previous kernel wrote).
template <typename... KArgs, typename... Args>
int launch_pdl(const char *what, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
               cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...), what);
}

int embed(cudaStream_t st, float *x, const float *emb_f32, const int8_t *emb_q, const float *emb_s,
          const int *tok_dev, int n, int dim, int gs, int vocab, int *err) {
    if (emb_f32)
        return launch_pdl("embed", embed_f32_kernel, dim3(n), dim3(256), 0, st, x, emb_f32, tok_dev,
                          dim, vocab, err);
    return launch_pdl("embed", embed_q8_kernel, dim3(n), dim3(256), 0, st, x, emb_q, emb_s, tok_dev,
                      dim, gs, vocab, err);
}

static unsigned row_threads(int dim) {
    const int n4 = dim >> 2;
    int t = ((n4 + 31) / 32) * 32;
    return unsigned(t < 32 ? 32 : (t > 1024 ? 1024 : t));
}

int rmsnorm(cudaStream_t st, float *o, const float *x, const float *w, int rows, int dim) {
    if (dim % 4) {
        set_error("rmsnorm: dim %d must be a multiple of 4", dim);
        return LEAP_ERR_INVALID;
    }
    return launch_pdl("rmsnorm", rmsnorm_kernel<false>, dim3(rows), dim3(row_threads(dim)), 0, st, o,
                      static_cast<char4 *>(nullptr), static_cast<float *>(nullptr), x, w, dim);
}

int rmsnorm_quantize(cudaStream_t st, int8_t *q, float *s, const float *x, const float *w, int rows,
                     int dim) {
    if (dim % 64) {
        set_error("rmsnorm_quantize: dim %d must be a multiple of 64", dim);
        return LEAP_ERR_INVALID;
    }
    return launch_pdl("rmsnorm_quantize", rmsnorm_kernel<true>, dim3(rows), dim3(row_threads(dim)),
                      0, st, static_cast<float *>(nullptr), reinterpret_cast<char4 *>(q), s, x, w,
                      dim);
}

int quantize(cudaStream_t st, int8_t *q, float *s, const float *x, size_t n, int gs) {
    if (gs == 64 && n % 64 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(q) & 3) == 0) {
        const size_t n4 = n / 4, threads = 256;
        const size_t blocks = (n4 + threads - 1) / threads;
        return launch_pdl("quantize", quantize64_kernel, dim3(unsigned(blocks)), dim3(unsigned(threads)),
                          0, st, reinterpret_cast<char4 *>(q), s, x, n4);
    }
    const size_t groups = (n + gs - 1) / gs;
    const int threads = 256;
    const size_t blocks = (groups * 32 + threads - 1) / threads;
    return launch_pdl("quantize", quantize_kernel, dim3(unsigned(blocks)), dim3(threads), 0, st, q, s,
                      x, n, gs);
}

// Grid for the warp-per-row FP32 GEMV: one warp per row, capped at the CTAs
// the SMs hold at once, since each CTA stages x once and then walks rows
// grid-stride.  Residency comes from
// the occupancy calculator, cached per (device, kernel, shared memory).
unsigned gemv_grid(const void *kernel, int items, size_t smem) {
    struct Entry {
        int dev;
        const void *kernel;
        size_t smem;
        int ctas;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    cudaGetDevice(&dev);
    int ctas = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Entry &e : cache)
            if (e.dev == dev && e.kernel == kernel && e.smem == smem) ctas = e.ctas;
        if (!ctas) {
            int sms = 0, per_sm = 0;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kGemvWarps * 32, smem);
            ctas = (sms > 0 ? sms : 148) * (per_sm > 0 ? per_sm : 1);
            cache.push_back({dev, kernel, smem, ctas});
        }
    }
    const int want = (items + kGemvWarps - 1) / kGemvWarps;
    return unsigned(want < ctas ? want : ctas);
}


constexpr size_t kGemvSmemMax = 200 * 1024;

bool g_q8_slice = true;
bool g_q8_tma = true;  // the persistent bulk-copy kernel is the default

size_t gemv_q8_stream_smem(int n) {
    return size_t(kPS) * kPStage + size_t(n) + size_t(n / 64) * 4 * (1 + 2 * kPR);
}

template <int PRO>
int gemv_q8_stream(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const float *xf,
                   const float *nw, const int8_t *wq, const float *ws, int n, int d,
                   const float *res, int *err) {
    const size_t smem = gemv_q8_stream_smem(n);
    const int r = set_kernel_smem(reinterpret_cast<const void *>(gemv_q8_stream_kernel<PRO>),
                                  kGemvSmemMax, "cudaFuncSetAttribute(gemv_q8_stream)");
    if (r != LEAP_OK) return r;
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, gemv_q8_stream_kernel<PRO>, kPThreads, smem);
    if (e != cudaSuccess) return cuda_status(e, "gemv_q8_stream occupancy");
    const int nblocks = (d + kPR - 1) / kPR;
    const int grid = std::max(1, std::min(nblocks, sms * std::max(per_sm, 1)));
    return launch_pdl("gemv_q8_stream", gemv_q8_stream_kernel<PRO>, dim3(unsigned(grid)),
                      dim3(kPThreads), smem, st, y, xq, xs, xf, nw, wq, ws, n, d, res, err);
}

// y = W . q(a) (+ res) where a is rmsnorm(x, nw) (pro 1, nw non-null) or x
// itself (pro 2), q the 64-group activation quantization: the quantization
// (and norm) run in the GEMV's prologue when the persistent kernel is
// selected and n <= 4096; otherwise rmsnorm_quantize /
// quantize write (aq, as) and gemv_q8 follows.  Same bits either way.
int gemv_q8_fused(cudaStream_t st, float *y, const float *x, const float *nw, int8_t *aq,
                  float *as, const int8_t *wq, const float *ws, int n, int d, const float *res,
                  int *err) {
    const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(nw) & 15) == 0;
    if (g_q8_tma && n % 64 == 0 && aligned && n <= 32 * kPR * kXV * 4)
        return nw ? gemv_q8_stream<kProNorm>(st, y, nullptr, nullptr, x, nw, wq, ws, n, d, res, err)
                  : gemv_q8_stream<kProQuant>(st, y, nullptr, nullptr, x, nullptr, wq, ws, n, d,
                                              res, err);
    if (int rc = nw ? rmsnorm_quantize(st, aq, as, x, nw, 1, n) : quantize(st, aq, as, x, n, 64))
        return rc;
    return gemv_q8(st, y, aq, as, wq, ws, n, d, res, err);
}

int gemv_q8_slice(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
                  const float *ws, int n, int d, const float *res, size_t smem) {
    const int r = set_kernel_smem(reinterpret_cast<const void *>(gemv_q8_slice_kernel),
                                  kGemvSmemMax, "cudaFuncSetAttribute(gemv_q8_slice)");
    if (r != LEAP_OK) return r;
    return launch_pdl("gemv_q8_slice", gemv_q8_slice_kernel, dim3(unsigned((d + kSR - 1) / kSR)),
                      dim3(256), smem, st, y, xq, xs, wq, ws, n, d, res);
}

int gemv_q8(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
            const float *ws, int n, int d, const float *res, int *err) {
    if (n % 64 != 0) {
        set_error("gemv_q8: n %d is not a multiple of 64", n);
        return LEAP_ERR_INVALID;
    }
    const size_t ng = size_t(n / 64), ng1 = ng | 1;
    const size_t smem = size_t(n) + ng * 4 + 2 * kQR * ng1 * 4;
    // x, its scales and the per-row group dots live in shared memory; beyond
    // that the tiled kernel (same accumulation order) takes over
    if (smem > kGemvSmemMax) return gemm_q8(st, y, xq, xs, wq, ws, n, d, 1, res);
    if (g_q8_tma && gemv_q8_stream_smem(n) <= kGemvSmemMax)
        return gemv_q8_stream<kProQ8>(st, y, xq, xs, nullptr, nullptr, wq, ws, n, d, res, err);
    if (g_q8_slice) return gemv_q8_slice(st, y, xq, xs, wq, ws, n, d, res, smem);
    const int r = set_kernel_smem(reinterpret_cast<const void *>(gemv_q8_kernel), kGemvSmemMax,
                                "cudaFuncSetAttribute(gemv_q8)");
    if (r != LEAP_OK) return r;
    return launch_pdl("gemv_q8", gemv_q8_kernel, dim3(unsigned((d + kQR - 1) / kQR)),
                      dim3(kGemvWarps * 32), smem, st, y, xq, xs, wq, ws, n, d, res);
}

bool g_q8_gemm_tc = true;

int gemm_q8(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
            const float *ws, int n, int d, int T, const float *res, int *err) {
    if (g_q8_gemm_tc && gemm_q8_tc_supported(xq, xs, wq, ws, n, T))
        return gemm_q8_tc(st, y, xq, xs, wq, ws, n, d, T, res, err);
    dim3 grid((d + kGR - 1) / kGR, (T + kGT - 1) / kGT);
    gemm_q8_kernel<<<grid, kGThreads, 0, st>>>(y, xq, xs, wq, ws, n, d, T, res);
    return cuda_status(cudaGetLastError(), "gemm_q8");
}

int gemv_f32(cudaStream_t st, float *y, const float *x, const float *w, int n, int d,
             const float *res, const float *nw, float *xb) {
    if (n % 4 != 0) {
        set_error("gemv_f32: n %d is not a multiple of 4", n);
        return LEAP_ERR_INVALID;
    }
    const bool aligned = (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                         (reinterpret_cast<uintptr_t>(nw) & 15) == 0;
    const size_t smem = size_t(n) * 4 * (nw ? 2 : 1);
    if (!aligned || smem > kGemvSmemMax) {
        // unfused: RMSNorm into xb (nw), then the GEMV or the tiled GEMM
        if (nw) {
            if (!xb) {
                set_error("gemv_f32: a normalised input this size needs a scratch row");
                return LEAP_ERR_INVALID;
            }
            if (int rc = rmsnorm(st, xb, x, nw, 1, n)) return rc;
            x = xb;
        }
        if (size_t(n) * 4 > kGemvSmemMax || (reinterpret_cast<uintptr_t>(x) & 15))
            return gemm_f32(st, y, x, w, n, d, 1, res);
        return gemv_f32(st, y, x, w, n, d, res);
    }
    const void *fn = nw ? reinterpret_cast<const void *>(gemv_f32_kernel<true>)
                        : reinterpret_cast<const void *>(gemv_f32_kernel<false>);
    const int r = set_kernel_smem(fn, kGemvSmemMax, "cudaFuncSetAttribute(gemv_f32)");
    if (r != LEAP_OK) return r;
    const unsigned grid = gemv_grid(fn, d, smem);
    return nw ? launch_pdl("gemv_f32", gemv_f32_kernel<true>, dim3(grid), dim3(kGemvWarps * 32),
                           smem, st, y, x, nw, w, n, d, res)
              : launch_pdl("gemv_f32", gemv_f32_kernel<false>, dim3(grid), dim3(kGemvWarps * 32),
                           smem, st, y, x, static_cast<const float *>(nullptr), w, n, d, res);
}

int gemm_f32(cudaStream_t st, float *y, const float *x, const float *w, int n, int d, int T,
             const float *res) {
    dim3 grid((d + kFR - 1) / kFR, (T + kFT - 1) / kFT);
    gemm_f32_kernel<<<grid, 256, 0, st>>>(y, x, w, n, d, T, res);
    return cuda_status(cudaGetLastError(), "gemm_f32");
}

int silu_mul(cudaStream_t st, float *h, const float *h3, size_t n) {
    if (n % 4) {
        set_error("silu_mul: n must be a multiple of 4");
        return LEAP_ERR_INVALID;
    }
    const size_t n4 = n / 4, blocks = (n4 + 255) / 256;
    return launch_pdl("silu_mul", silu_mul_kernel<false>, dim3(unsigned(blocks)), dim3(256), 0, st,
                      h, static_cast<char4 *>(nullptr), static_cast<float *>(nullptr), h3, n4);
}

int silu_mul_quantize(cudaStream_t st, int8_t *q, float *s, const float *h, const float *h3,
                      size_t n) {
    if (n % 64) {
        set_error("silu_mul_quantize: n must be a multiple of 64");
        return LEAP_ERR_INVALID;
    }
    const size_t n4 = n / 4, blocks = (n4 + 255) / 256;
    return launch_pdl("silu_mul_quantize", silu_mul_kernel<true>, dim3(unsigned(blocks)), dim3(256),
                      0, st, const_cast<float *>(h), reinterpret_cast<char4 *>(q), s, h3, n4);
}

int argmax(cudaStream_t st, int *out, const float *v, int n) {
    return launch_pdl("argmax", argmax_kernel, dim3(1), dim3(1024), 0, st, out, v, n);
}

int synth_normal(cudaStream_t st, float *w, size_t n, uint64_t seed, float std, float fill) {
    synth_normal_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(w, n, seed, std, fill);
    return cuda_status(cudaGetLastError(), "synth_normal");
}

}  // namespace eng
}  // namespace leap
