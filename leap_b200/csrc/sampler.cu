// sampler.cu — the reference Sampler on the GPU (src/inference/Sampler.cpp,
// src/inference/Utils.h:18-29), so a pipeline's last stage can turn logits
// into a token without moving them to the host.
//
// Sampler::sample(logits): temperature 0 -> argmax (:199-202; the engine's
// argmax kernel, same lane tie order).  Otherwise logits *= 1/temperature,
// softmax (max, exp(x - max), sum, *= 1/sum: :169-185), coin = random_f32
// (xorshift*, advanced on the host exactly as the reference advances its
// state, one draw per call), then
//   topp <= 0 or >= 1: the first i whose running sum of p (index order)
//                      exceeds coin (sample_mult, :122-131);
//   else:              candidates p >= (1 - topp) / (n - 1), taken in
//                      descending p until their mass exceeds topp (or all
//                      of them), r = coin * that mass, and the first
//                      candidate (descending) whose running mass exceeds r
//                      (sample_topp, :133-167).
// One CTA of 1024 threads does a draw.  The reference's walks are running
// float sums whose rounding decides the token on flat distributions, so they
// are run as the reference runs them: the multinomial walk by one thread in
// index order; for top-p the candidates in play are found with exact 62-bit
// fixed-point masses (p * 2^62) and a 3-pass radix select on the
// probability bits (11 + 11 + 10), gathered and sorted in shared memory
// (p descending, index ascending: the reference's std::sort leaves equal
// probabilities unordered), and one thread walks them in float.  Beyond
// 16384 candidates in play the walks use the exact fixed-point sums instead.
// The probabilities themselves differ from the reference's in the last bits
// (exp, summation order of the softmax), so a token can differ only when
// the coin or topp lies within that rounding of a running sum.
#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "ctx.h"
#include "engine.h"

struct leap_sampler {
    int vocab = 0;
    float temperature = 0.f, topp = 0.f;
    unsigned long long state = 0;
    int device = 0;
    float *probs = nullptr;  // [vocab] device scratch
};

namespace leap {
namespace {

constexpr int kSmpThreads = 1024;
constexpr int kBuckets = 2048;
constexpr int kSortCap = 16384;  // candidates sorted in shared memory (128 KB)

__device__ __forceinline__ uint64_t fixed62(float p) {
    return __float2ull_rz(p * 4611686018427387904.0f);  // p * 2^62, p in [0, 1]
}

// Inclusive scan of one value per thread over the block (any associative
// exact type); returns the inclusive value, *total the block total.
template <typename T>
__device__ T block_scan(T v, T *warp_tot, T *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const T u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
    }
    if (lane == 31) warp_tot[warp] = v;
    __syncthreads();
    if (warp == 0) {
        T w = lane < int(blockDim.x >> 5) ? warp_tot[lane] : T(0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const T u = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += u;
        }
        warp_tot[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const T before = warp > 0 ? warp_tot[warp - 1] : T(0);
    *total = warp_tot[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before + v;
}

struct SmpShared {
    uint64_t mass[kBuckets];
    unsigned cnt[kBuckets];
    uint64_t wtot[32];
    float fred[32];
    int ired[32];
    uint64_t sel_rem;
    unsigned sel_prefix, sel_bucket;
    int sel_found;
};

// Descending walk over candidates (p >= cutoff): the element at which the
// running mass first exceeds `target`.  Returns its probability bits and
// which copy of that value (1-based) it is; *above = mass of all strictly
// larger candidates.  Requires target < total candidate mass.
__device__ void select_desc(SmpShared &sh, const float *probs, int n, float cutoff,
                            uint64_t target, unsigned *v_bits, unsigned *copy, uint64_t *above) {
    const int tid = threadIdx.x;
    unsigned prefix = 0, pmask = 0;
    uint64_t rem = target, acc_above = 0;
    const int shifts[3] = {21, 10, 0}, widths[3] = {11, 11, 10};
    for (int pass = 0; pass < 3; ++pass) {
        const int sh_ = shifts[pass], nb = 1 << widths[pass];
        for (int b = tid; b < nb; b += blockDim.x) {
            sh.mass[b] = 0;
            sh.cnt[b] = 0;
        }
        __syncthreads();
        for (int i = tid; i < n; i += blockDim.x) {
            const float p = probs[i];
            if (p >= cutoff) {
                const unsigned u = __float_as_uint(p);
                if ((u & pmask) == prefix) {
                    const unsigned b = (u >> sh_) & unsigned(nb - 1);
                    atomicAdd(&sh.cnt[b], 1u);
                    atomicAdd(reinterpret_cast<unsigned long long *>(&sh.mass[b]),
                              (unsigned long long)fixed62(p));
                }
            }
        }
        __syncthreads();
        // warp 0: buckets from the highest value down; lane l owns a
        // contiguous run of nb/32 buckets
        if (tid < 32) {
            const int per = nb / 32;
            const int hi = nb - 1 - tid * per;  // this lane's first (largest) bucket
            uint64_t s = 0;
            for (int k = 0; k < per; ++k) s += sh.mass[hi - k];
            // exclusive prefix over lanes (descending order)
            uint64_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t u = __shfl_up_sync(0xffffffffu, incl, o);
                if (tid >= o) incl += u;
            }
            const uint64_t excl = incl - s;
            const bool here = excl <= rem && rem < incl;
            const unsigned ballot = __ballot_sync(0xffffffffu, here);
            if (ballot) {
                const int owner = __ffs(ballot) - 1;
                if (tid == owner) {
                    uint64_t c = excl;
                    int bsel = hi - per + 1;
                    for (int k = 0; k < per; ++k) {
                        const int b = hi - k;
                        if (rem < c + sh.mass[b]) {
                            bsel = b;
                            break;
                        }
                        c += sh.mass[b];
                    }
                    sh.sel_bucket = unsigned(bsel);
                    sh.sel_rem = rem - c;
                    sh.sel_found = 1;
                    sh.wtot[0] = c;
                }
            } else if (tid == 0) {
                sh.sel_found = 0;
            }
        }
        __syncthreads();
        if (!sh.sel_found) break;  // cannot happen when target < total mass
        acc_above += sh.wtot[0];
        rem = sh.sel_rem;
        prefix |= sh.sel_bucket << sh_;
        pmask |= unsigned(nb - 1) << sh_;
        __syncthreads();
    }
    const uint64_t fv = fixed62(__uint_as_float(prefix));
    *v_bits = prefix;
    *copy = fv ? unsigned(rem / fv) + 1u : 1u;
    *above = acc_above;
}

// Index of the `copy`-th element (index order) whose probability bits equal
// v_bits.
__device__ int find_copy(SmpShared &sh, const float *probs, int n, unsigned v_bits, unsigned copy) {
    const int tid = threadIdx.x, T = blockDim.x;
    const int chunk = (n + T - 1) / T;
    const int i0 = tid * chunk, i1 = min(n, i0 + chunk);
    unsigned c = 0;
    for (int i = i0; i < i1; ++i) c += (__float_as_uint(probs[i]) == v_bits);
    unsigned tot;
    const unsigned incl = block_scan<unsigned>(c, reinterpret_cast<unsigned *>(sh.wtot), &tot);
    const unsigned excl = incl - c;
    if (tid == 0) sh.ired[0] = -1;
    __syncthreads();
    if (excl < copy && copy <= incl) {
        unsigned k = excl;
        for (int i = i0; i < i1; ++i)
            if (__float_as_uint(probs[i]) == v_bits && ++k == copy) {
                sh.ired[0] = i;
                break;
            }
    }
    __syncthreads();
    return sh.ired[0];
}

__global__ void __launch_bounds__(kSmpThreads)
sample_kernel(const float *__restrict__ logits, float *__restrict__ probs, int *token, int n,
              float inv_temp, float topp, unsigned coin24) {
    grid_dependency_wait();  // the logits come from the previous kernel
    grid_launch_dependents();
    __shared__ SmpShared sh;
    extern __shared__ uint64_t keys[];  // [kSortCap] sort keys
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    // ---- softmax of logits * (1/temperature) --------------------------------
    float mx = -INFINITY;
    for (int i = tid; i < n; i += blockDim.x) mx = fmaxf(mx, logits[i] * inv_temp);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) sh.fred[warp] = mx;
    __syncthreads();
    mx = sh.fred[0];
    for (int w = 1; w < nw; ++w) mx = fmaxf(mx, sh.fred[w]);
    __syncthreads();
    float sum = 0.f;
    for (int i = tid; i < n; i += blockDim.x) {
        const float e = expf(logits[i] * inv_temp - mx);
        probs[i] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (lane == 0) sh.fred[warp] = sum;
    __syncthreads();
    sum = 0.f;
    for (int w = 0; w < nw; ++w) sum += sh.fred[w];
    const float inv_sum = 1.0f / sum;
    for (int i = tid; i < n; i += blockDim.x) probs[i] *= inv_sum;
    __syncthreads();  // probs complete (global, same block)

    const float coin = float(coin24) * (1.0f / 16777216.0f);  // random_f32, exactly
    if (!(topp > 0.f && topp < 1.f)) {
        // ---- sample_mult (:122-131): the reference's running float sum in
        // index order, so one thread walks it as the reference does
        if (tid == 0) {
            float cdf = 0.f;
            int pick = n - 1;
            for (int i = 0; i < n; ++i) {
                cdf += probs[i];
                if (coin < cdf) {
                    pick = i;
                    break;
                }
            }
            *token = pick;
        }
        return;
    }

    // ---- sample_topp (:133-167) ----------------------------------------------
    const float cutoff = (1.0f - topp) / (float(n) - 1.0f);
    uint64_t total = 0;
    unsigned n0 = 0;
    {
        uint64_t s = 0;
        unsigned c = 0;
        for (int i = tid; i < n; i += blockDim.x) {
            const float p = probs[i];
            if (p >= cutoff) {
                s += fixed62(p);
                ++c;
            }
        }
        block_scan<uint64_t>(s, sh.wtot, &total);
        block_scan<unsigned>(c, reinterpret_cast<unsigned *>(sh.wtot), &n0);
    }
    if (total == 0) {  // no candidate: cannot happen, the largest p is >= 1/n > cutoff
        if (tid == 0) *token = 0;
        return;
    }
    // The reference sorts the candidates by descending p and walks them with
    // float running sums.  Gather the candidates down to where the exact mass
    // exceeds topp by 2^-10 (more than any float walk of <= kSortCap terms can
    // drift: 16384 roundings of at most 2^-24 each), sort them (p descending, index ascending), and let one thread
    // run the reference's two walks in float.
    const uint64_t t1 = fixed62(topp);
    const uint64_t tg = t1 + (uint64_t(1) << 52);
    unsigned vg, mg;
    uint64_t aboveg;
    select_desc(sh, probs, n, cutoff, tg < total ? tg : total - 1, &vg, &mg, &aboveg);
    const float pg = __uint_as_float(vg);
    if (tid == 0) sh.ired[1] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) {
        const float p = probs[i];
        if (p >= cutoff && p >= pg) {
            const unsigned k = atomicAdd(reinterpret_cast<unsigned *>(&sh.ired[1]), 1u);
            if (k < unsigned(kSortCap))
                keys[k] = (uint64_t(~__float_as_uint(p)) << 32) | unsigned(i);
        }
    }
    __syncthreads();
    const int kg = sh.ired[1];
    if (kg <= kSortCap) {
        int np2 = 1;
        while (np2 < kg) np2 <<= 1;
        for (int k = kg + tid; k < np2; k += blockDim.x) keys[k] = ~uint64_t(0);
        __syncthreads();
        // bitonic sort, ascending key = descending p, then ascending index
        for (int size = 2; size <= np2; size <<= 1)
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int k = tid; k < np2; k += blockDim.x) {
                    const int l = k ^ stride;
                    if (l > k) {
                        const bool up = (k & size) == 0;
                        const uint64_t a = keys[k], b = keys[l];
                        if ((a > b) == up) {
                            keys[k] = b;
                            keys[l] = a;
                        }
                    }
                }
                __syncthreads();
            }
        if (tid == 0) {
            auto prob = [&](int k) { return __uint_as_float(~unsigned(keys[k] >> 32)); };
            float cum = 0.f;
            int last = -1;
            for (int k = 0; k < kg; ++k) {
                cum += prob(k);
                if (cum > topp) {
                    last = k;
                    break;
                }
            }
            if (last < 0) last = kg - 1;  // all candidates (kg == n0 then)
            const float r = coin * cum;
            float cdf = 0.f;
            int pick = int(keys[last] & 0xffffffffu);
            for (int k = 0; k <= last; ++k) {
                cdf += prob(k);
                if (r < cdf) {
                    pick = int(keys[k] & 0xffffffffu);
                    break;
                }
            }
            *token = pick;
        }
        return;
    }
    // More than kSortCap candidates in play (a very flat distribution): the
    // same walks on exact fixed-point sums, selected by radix passes.
    unsigned v1, m1;
    uint64_t above1;
    select_desc(sh, probs, n, cutoff, t1 < total ? t1 : total - 1, &v1, &m1, &above1);
    const uint64_t cumx = above1 + uint64_t(m1) * fixed62(__uint_as_float(v1));
    const uint64_t rx = __umul64hi(cumx, uint64_t(coin24) << 40);  // coin * cum, exactly
    unsigned v2, m2;
    uint64_t above2;
    select_desc(sh, probs, n, cutoff, rx < cumx ? rx : cumx - 1, &v2, &m2, &above2);
    const int idx = find_copy(sh, probs, n, v2, m2);
    if (tid == 0) *token = idx >= 0 ? idx : 0;
}

}  // namespace

int sampler_launch(leap_sampler *s, cudaStream_t st, const float *logits, int *token_dev) {
    if (s->temperature == 0.0f) return eng::argmax(st, token_dev, logits, s->vocab);
    // random_f32 (src/inference/Utils.h:18-29), state advanced as the reference does
    unsigned long long x = s->state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    s->state = x;
    const unsigned u = unsigned((x * 0x2545F4914F6CDD1Dull) >> 32);
    const unsigned coin24 = u >> 8;  // coin = coin24 / 2^24 exactly
    const float inv_temp = 1.0f / s->temperature;
    if (s->device < 0 || s->device >= kMaxDevices) {
        set_error("sampler: device index out of range");
        return LEAP_ERR_INVALID;
    }
    if (const int r = set_kernel_smem(reinterpret_cast<const void *>(sample_kernel),
                                      kSortCap * sizeof(uint64_t),
                                      "cudaFuncSetAttribute(sample_kernel)"))
        return r;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kSmpThreads);
    cfg.dynamicSmemBytes = kSortCap * sizeof(uint64_t);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, sample_kernel, logits, s->probs, token_dev,
                                          s->vocab, inv_temp, s->topp, coin24),
                       "sample_kernel launch");
}

}  // namespace leap

extern "C" {

int leap_sampler_create(int vocab, float temperature, float topp, unsigned long long seed,
                        int device, leap_sampler **out) {
    leap::clear_error();
    if (!out || vocab < 2 || !(temperature >= 0.f) || std::isnan(topp)) {
        leap::set_error("sampler: bad arguments");
        return LEAP_ERR_INVALID;
    }
    *out = nullptr;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return leap::cuda_status(e, "cudaSetDevice");
    leap_sampler *s = new leap_sampler;
    s->vocab = vocab;
    s->temperature = temperature;
    s->topp = topp;
    s->state = seed;
    s->device = device;
    e = cudaMalloc(&s->probs, sizeof(float) * size_t(vocab));
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        delete s;
        return leap::cuda_status(e, "cudaMalloc(sampler)");
    }
    *out = s;
    return LEAP_OK;
}

int leap_sampler_destroy(leap_sampler *s) {
    leap::clear_error();
    if (!s) return LEAP_OK;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaFree(s->probs);
    cudaSetDevice(prev);
    delete s;
    return LEAP_OK;
}

int leap_sampler_sample(leap_sampler *s, void *stream, const float *logits, int *token_dev) {
    leap::clear_error();
    if (!s || !logits || !token_dev) {
        leap::set_error("sampler: null argument");
        return LEAP_ERR_INVALID;
    }
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != s->device) cudaSetDevice(s->device);
    const int st = leap::sampler_launch(s, static_cast<cudaStream_t>(stream), logits, token_dev);
    if (prev != s->device) cudaSetDevice(prev);
    return st;
}

int leap_sampler_state(const leap_sampler *s, unsigned long long *state) {
    leap::clear_error();
    if (!s || !state) {
        leap::set_error("sampler: null argument");
        return LEAP_ERR_INVALID;
    }
    *state = s->state;
    return LEAP_OK;
}

}  // extern "C"
