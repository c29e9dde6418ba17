// context.cu — the C ABI (include/leap_b200.h): context lifetime, device KV
// cache, host staging, argument checks and error reporting.
//
// Error convention: every entry point returns 0 or a LEAP_ERR_* code and
// leaves a message for leap_last_error(); nothing throws across the ABI.
// A C++ caller maps non-zero to std::runtime_error like the reference
// (src/inference/main.cpp:498-501).
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <vector>

#include <mutex>
#include <set>
#include <utility>

#include "ctx.h"

namespace leap {
namespace {
thread_local char g_err[1024] = {0};

// Select a device for the duration of one ABI call and restore the
// caller's current device afterwards.
struct DeviceGuard {  // makes `dev` current; restores the previous device if it differed
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        ok = prev == dev || cudaSetDevice(dev) == cudaSuccess;
        if (prev == dev) prev = -1;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

size_t stage_floats(const leap_ctx *c) {
    // q | k | v | out | error word (padded to 16 bytes)
    return size_t(2) * c->n_heads * c->hd + size_t(2) * c->n_kv * c->hd + 4;
}

void free_ctx(leap_ctx *c) {
    if (!c) return;
    DeviceGuard g(c->device);
    if (c->own_stream) cudaStreamSynchronize(c->own_stream);
    if (c->stream && c->stream != c->own_stream) cudaStreamSynchronize(c->stream);
    cudaFree(c->k_cache);
    cudaFree(c->v_cache);
    cudaFree(c->rope_cos);
    cudaFree(c->rope_sin);
    for (int i = 0; i < 2; ++i) {
        cudaFree(c->part_o[i]);
        cudaFree(c->part_ml[i]);
        cudaFree(c->counters[i]);
    }
    cudaFree(c->d_stage);
    cudaFree(c->d_qrot);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->own_stream) cudaStreamDestroy(c->own_stream);
    delete c;
}

#define LEAP_TRY_CUDA(expr, what)                     \
    do {                                              \
        cudaError_t e_ = (expr);                      \
        if (e_ != cudaSuccess) {                      \
            int st_ = leap::cuda_status(e_, what);    \
            return st_;                               \
        }                                             \
    } while (0)

#define LEAP_CHECK_CTX(c)                                       \
    do {                                                        \
        if (!(c)) {                                             \
            leap::set_error("null context");                    \
            return LEAP_ERR_INVALID;                            \
        }                                                       \
    } while (0)

// Read and clear the device error word after the stream has drained.
int check_device_error(leap_ctx *c) {
    int err = 0;
    const int *d_err = reinterpret_cast<const int *>(c->d_err);
    LEAP_TRY_CUDA(cudaMemcpy(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost),
                  "read device error word");
    if (err == 0) return LEAP_OK;
    // A CTA that gave up never reached its split-KV ticket: clear the
    // tickets and the error word so the next call starts clean.
    cudaMemset(c->d_err, 0, sizeof(int));
    for (int i = 0; i < 2; ++i)
        cudaMemset(c->counters[i], 0, sizeof(unsigned) * kMaxSeqPerLaunch * c->n_kv);
    if (err == kDevErrBadToken)
        set_error("a device-side token id was outside [0, vocab_size)");
    else
        set_error("a kernel reported device error %d (bounded wait timed out)", err);
    return LEAP_ERR_DEVICE;
}

}  // namespace

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int cuda_status(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return LEAP_OK;
    cudaGetLastError();  // clear a non-sticky error
    set_error("%s: %s", what, cudaGetErrorString(e));
    return e == cudaErrorMemoryAllocation ? LEAP_ERR_NOMEM : LEAP_ERR_CUDA;
}

int set_kernel_smem(const void *fn, size_t bytes, const char *what, bool nonportable_cluster) {
    static std::mutex mu;
    static std::set<std::pair<const void *, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(mu);
    if (done.count({fn, dev})) return LEAP_OK;
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    if (e == cudaSuccess && nonportable_cluster)
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return cuda_status(e, what);
    done.insert({fn, dev});
    return LEAP_OK;
}

}  // namespace leap

using leap::DeviceGuard;

extern "C" {

const char *leap_last_error(void) { return leap::g_err; }

const char *leap_version(void) { return "leap_b200 0.1 (sm_100a)"; }

int leap_rope_table(int seq_len, int head_dim, float theta, float *rope_cos, float *rope_sin) {
    leap::clear_error();
    if (seq_len < 1 || head_dim < 2 || (head_dim & 1) || !rope_cos || !rope_sin || !(theta > 0.f)) {
        leap::set_error("invalid rope table arguments");
        return LEAP_ERR_INVALID;
    }
    const int half = head_dim / 2;
    const float log_theta = logf(theta);
    for (int pos = 0; pos < seq_len; ++pos) {
        for (int i = 0; i < head_dim; i += 2) {
            const float e = float(i) / float(head_dim);
            const float freq = expf(-(e * log_theta));
            const float val = float(pos) * freq;
            rope_cos[size_t(pos) * half + i / 2] = cosf(val);
            rope_sin[size_t(pos) * half + i / 2] = sinf(val);
        }
    }
    return LEAP_OK;
}

int leap_ctx_create(const leap_ctx_desc *d, leap_ctx **out) {
    leap::clear_error();
    if (!d || !out) {
        leap::set_error("null argument");
        return LEAP_ERR_INVALID;
    }
    *out = nullptr;
    if (d->n_layers < 1 || d->n_heads < 1 || d->n_kv_heads < 1 ||
        d->n_heads % d->n_kv_heads != 0 || d->max_seq < 1 || d->max_batch < 1) {
        leap::set_error("invalid shape: n_layers %d n_heads %d n_kv_heads %d max_seq %d max_batch %d",
                        d->n_layers, d->n_heads, d->n_kv_heads, d->max_seq, d->max_batch);
        return LEAP_ERR_INVALID;
    }
    const int group = d->n_heads / d->n_kv_heads;
    if ((d->head_dim != 64 && d->head_dim != 128) ||
        (group != 1 && group != 2 && group != 4 && group != 8)) {
        leap::set_error("unsupported head_dim %d / kv_mul %d (head_dim 64|128, kv_mul 1|2|4|8)",
                        d->head_dim, group);
        return LEAP_ERR_INVALID;
    }
    if (!d->rope_cos || !d->rope_sin) {
        leap::set_error("rope_cos/rope_sin tables are required");
        return LEAP_ERR_INVALID;
    }
    int n_dev = 0;
    LEAP_TRY_CUDA(cudaGetDeviceCount(&n_dev), "cudaGetDeviceCount");
    if (d->device < 0 || d->device >= n_dev || d->device >= leap::kMaxDevices) {
        leap::set_error("device %d out of range (%d devices)", d->device, n_dev);
        return LEAP_ERR_INVALID;
    }
    DeviceGuard guard(d->device);
    if (!guard.ok) {
        leap::set_error("cudaSetDevice(%d) failed", d->device);
        return LEAP_ERR_CUDA;
    }

    leap_ctx *c = new (std::nothrow) leap_ctx();
    if (!c) {
        leap::set_error("host allocation failed");
        return LEAP_ERR_NOMEM;
    }
    c->device = d->device;
    c->n_layers = d->n_layers;
    c->layer0 = d->layer0;
    c->n_heads = d->n_heads;
    c->n_kv = d->n_kv_heads;
    c->hd = d->head_dim;
    c->group = group;
    c->max_seq = d->max_seq;
    c->max_seq_pad = (d->max_seq + 63) / 64 * 64;
    c->max_batch = d->max_batch;
    int st = LEAP_OK;
    auto fail = [&](cudaError_t e, const char *what) {
        st = leap::cuda_status(e, what);
        leap::free_ctx(c);
        return st;
    };
    cudaError_t e = cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->device);
    if (e != cudaSuccess) return fail(e, "cudaDeviceGetAttribute");

    c->head_stride = size_t(c->max_seq_pad) * c->hd;
    c->layer_stride = size_t(c->n_kv) * c->head_stride;
    c->slot_stride = size_t(c->n_layers) * c->layer_stride;
    c->cache_bytes = size_t(c->max_batch) * c->slot_stride * sizeof(float);
    if ((e = cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking)) != cudaSuccess)
        return fail(e, "cudaStreamCreate");
    c->stream = c->own_stream;
    if ((e = cudaMalloc(&c->k_cache, c->cache_bytes)) != cudaSuccess) return fail(e, "cudaMalloc(k_cache)");
    if ((e = cudaMalloc(&c->v_cache, c->cache_bytes)) != cudaSuccess) return fail(e, "cudaMalloc(v_cache)");
    if ((e = cudaMemset(c->k_cache, 0, c->cache_bytes)) != cudaSuccess) return fail(e, "cudaMemset");
    if ((e = cudaMemset(c->v_cache, 0, c->cache_bytes)) != cudaSuccess) return fail(e, "cudaMemset");
    c->device_bytes += 2 * c->cache_bytes;

    const size_t rope_bytes = size_t(c->max_seq) * (c->hd / 2) * sizeof(float);
    if ((e = cudaMalloc(&c->rope_cos, rope_bytes)) != cudaSuccess) return fail(e, "cudaMalloc(rope)");
    if ((e = cudaMalloc(&c->rope_sin, rope_bytes)) != cudaSuccess) return fail(e, "cudaMalloc(rope)");
    if ((e = cudaMemcpy(c->rope_cos, d->rope_cos, rope_bytes, cudaMemcpyHostToDevice)) != cudaSuccess)
        return fail(e, "copy rope_cos");
    if ((e = cudaMemcpy(c->rope_sin, d->rope_sin, rope_bytes, cudaMemcpyHostToDevice)) != cudaSuccess)
        return fail(e, "copy rope_sin");
    c->device_bytes += 2 * rope_bytes;

    c->max_parts = leap::max_decode_parts(c->hd, c->n_kv, c->max_batch, c->max_seq_pad, c->num_sms);
    const size_t po = size_t(c->max_parts) * c->group * c->hd * sizeof(float);
    // (M, L) per head per partial, records padded to 16 bytes
    const size_t pml = size_t(c->max_parts) * 2 * (c->group < 2 ? 2 : c->group) * sizeof(float);
    const size_t cnt = size_t(leap::kMaxSeqPerLaunch) * c->n_kv * sizeof(unsigned);
    for (int i = 0; i < 2; ++i) {
        if ((e = cudaMalloc(&c->part_o[i], po)) != cudaSuccess) return fail(e, "cudaMalloc(partials)");
        if ((e = cudaMalloc(&c->part_ml[i], pml)) != cudaSuccess) return fail(e, "cudaMalloc(partials)");
        if ((e = cudaMalloc(&c->counters[i], cnt)) != cudaSuccess) return fail(e, "cudaMalloc(counters)");
        if ((e = cudaMemset(c->counters[i], 0, cnt)) != cudaSuccess) return fail(e, "cudaMemset(counters)");
    }
    c->device_bytes += 2 * (po + pml + cnt);

    const size_t sb = leap::stage_floats(c) * sizeof(float);
    if ((e = cudaMallocHost(&c->h_stage, sb)) != cudaSuccess) return fail(e, "cudaMallocHost(stage)");
    if ((e = cudaHostGetDevicePointer(reinterpret_cast<void **>(&c->h_stage_dev), c->h_stage, 0)) !=
        cudaSuccess)
        return fail(e, "cudaHostGetDevicePointer(stage)");
    if ((e = cudaMalloc(&c->d_stage, sb)) != cudaSuccess) return fail(e, "cudaMalloc(stage)");
    if ((e = cudaMemset(c->d_stage, 0, sb)) != cudaSuccess) return fail(e, "cudaMemset(stage)");
    c->d_err = reinterpret_cast<int *>(c->d_stage + leap::stage_floats(c) - 4);
    c->device_bytes += sb;

    if (int cst = leap::decode_cluster_capacity(c, &c->cluster_capacity)) {
        leap::free_ctx(c);
        return cst;
    }
    if ((e = cudaDeviceSynchronize()) != cudaSuccess) return fail(e, "cudaDeviceSynchronize");
    *out = c;
    return LEAP_OK;
}

int leap_ctx_destroy(leap_ctx *c) {
    leap::clear_error();
    if (!c) return LEAP_OK;
    leap::free_ctx(c);
    return LEAP_OK;
}

int leap_ctx_set_stream(leap_ctx *c, void *stream) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    c->stream = static_cast<cudaStream_t>(stream);  // NULL: the default stream
    c->last_written_layer = leap_ctx::kWroteAll;   // other work may precede
    return LEAP_OK;
}

int leap_ctx_use_own_stream(leap_ctx *c) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    c->stream = c->own_stream;
    c->last_written_layer = leap_ctx::kWroteAll;
    return LEAP_OK;
}

int leap_set_decode_impl(leap_ctx *c, int impl) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (impl < 0 || impl > 4) {
        leap::set_error("decode impl %d unknown", impl);
        return LEAP_ERR_INVALID;
    }
    c->decode_impl = impl;
    return LEAP_OK;
}

int leap_decode_cluster_capacity(const leap_ctx *c, int *n) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (!n) {
        leap::set_error("null argument");
        return LEAP_ERR_INVALID;
    }
    *n = c->cluster_capacity;
    return LEAP_OK;
}

int leap_set_overlap(leap_ctx *c, int enable) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    c->overlap = enable ? 1 : 0;
    return LEAP_OK;
}

int leap_sync(leap_ctx *c) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    DeviceGuard g(c->device);
    LEAP_TRY_CUDA(cudaStreamSynchronize(c->stream), "cudaStreamSynchronize");
    return leap::check_device_error(c);
}

int leap_ctx_device_bytes(const leap_ctx *c, size_t *bytes) {
    LEAP_CHECK_CTX(c);
    if (!bytes) {
        leap::set_error("null argument");
        return LEAP_ERR_INVALID;
    }
    *bytes = c->device_bytes + c->qrot_cap * sizeof(float);
    return LEAP_OK;
}

int leap_kv_clear(leap_ctx *c) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    DeviceGuard g(c->device);
    c->last_written_layer = leap_ctx::kWroteAll;
    LEAP_TRY_CUDA(cudaMemsetAsync(c->k_cache, 0, c->cache_bytes, c->stream), "clear k");
    LEAP_TRY_CUDA(cudaMemsetAsync(c->v_cache, 0, c->cache_bytes, c->stream), "clear v");
    return LEAP_OK;
}

static int kv_range_check(const leap_ctx *c, int slot, int layer, int pos0, int n_pos) {
    if (slot < 0 || slot >= c->max_batch || layer < 0 || layer >= c->n_layers || pos0 < 0 ||
        n_pos < 0 || pos0 + n_pos > c->max_seq) {
        leap::set_error("kv range out of bounds: slot %d layer %d pos0 %d n_pos %d", slot, layer,
                        pos0, n_pos);
        return LEAP_ERR_INVALID;
    }
    return LEAP_OK;
}

int leap_kv_write(leap_ctx *c, int slot, int layer, int pos0, int n_pos, const float *k,
                  const float *v, int from_host) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (int st = kv_range_check(c, slot, layer, pos0, n_pos)) return st;
    if (n_pos == 0) return LEAP_OK;
    if (!k || !v) {
        leap::set_error("null k/v");
        return LEAP_ERR_INVALID;
    }
    DeviceGuard g(c->device);
    c->last_written_layer = leap_ctx::kWroteAll;
    const cudaMemcpyKind kind = from_host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
    const size_t row = size_t(c->hd) * sizeof(float);
    for (int h = 0; h < c->n_kv; ++h) {
        LEAP_TRY_CUDA(cudaMemcpy2DAsync(leap::k_head_ptr(c, slot, layer, h) + size_t(pos0) * c->hd,
                                        row, k + size_t(h) * c->hd, row * c->n_kv, row, n_pos,
                                        kind, c->stream),
                      "kv_write k");
        LEAP_TRY_CUDA(cudaMemcpy2DAsync(leap::v_head_ptr(c, slot, layer, h) + size_t(pos0) * c->hd,
                                        row, v + size_t(h) * c->hd, row * c->n_kv, row, n_pos,
                                        kind, c->stream),
                      "kv_write v");
    }
    if (from_host) LEAP_TRY_CUDA(cudaStreamSynchronize(c->stream), "kv_write sync");
    return LEAP_OK;
}

int leap_kv_read(leap_ctx *c, int slot, int layer, int pos0, int n_pos, float *k, float *v,
                 int to_host) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (int st = kv_range_check(c, slot, layer, pos0, n_pos)) return st;
    if (n_pos == 0) return LEAP_OK;
    if (!k || !v) {
        leap::set_error("null k/v");
        return LEAP_ERR_INVALID;
    }
    DeviceGuard g(c->device);
    const cudaMemcpyKind kind = to_host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
    const size_t row = size_t(c->hd) * sizeof(float);
    for (int h = 0; h < c->n_kv; ++h) {
        LEAP_TRY_CUDA(cudaMemcpy2DAsync(k + size_t(h) * c->hd, row * c->n_kv,
                                        leap::k_head_ptr(c, slot, layer, h) + size_t(pos0) * c->hd,
                                        row, row, n_pos, kind, c->stream),
                      "kv_read k");
        LEAP_TRY_CUDA(cudaMemcpy2DAsync(v + size_t(h) * c->hd, row * c->n_kv,
                                        leap::v_head_ptr(c, slot, layer, h) + size_t(pos0) * c->hd,
                                        row, row, n_pos, kind, c->stream),
                      "kv_read v");
    }
    if (to_host) LEAP_TRY_CUDA(cudaStreamSynchronize(c->stream), "kv_read sync");
    return LEAP_OK;
}

static int decode_check(const leap_ctx *c, int layer, const float *q, const float *k,
                        const float *v, const float *out) {
    if (layer < 0 || layer >= c->n_layers) {
        leap::set_error("layer %d out of range [0,%d)", layer, c->n_layers);
        return LEAP_ERR_INVALID;
    }
    if (!q || !k || !v || !out) {
        leap::set_error("null q/k/v/out");
        return LEAP_ERR_INVALID;
    }
    if (!leap::aligned16(q) || !leap::aligned16(k) || !leap::aligned16(v) ||
        !leap::aligned16(out)) {
        leap::set_error("q/k/v/out must be 16-byte aligned");
        return LEAP_ERR_INVALID;
    }
    return LEAP_OK;
}

int leap_attn_decode(leap_ctx *c, int layer, int pos, const float *q, const float *k_new,
                     const float *v_new, float *out) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (int st = decode_check(c, layer, q, k_new, v_new, out)) return st;
    if (pos < 0 || pos >= c->max_seq) {
        leap::set_error("pos %d out of range [0,%d)", pos, c->max_seq);
        return LEAP_ERR_INVALID;
    }
    DeviceGuard g(c->device);
    leap::DecodeSeq tab;
    tab.n_seq = 1;
    tab.pos[0] = pos;
    tab.slot[0] = 0;
    return leap::launch_decode(c, layer, tab, q, k_new, v_new, out);
}

int leap_attn_decode_host(leap_ctx *c, int layer, int pos, const float *q, const float *k_new,
                          const float *v_new, float *out) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (!q || !k_new || !v_new || !out) {
        leap::set_error("null q/k/v/out");
        return LEAP_ERR_INVALID;
    }
    if (layer < 0 || layer >= c->n_layers || pos < 0 || pos >= c->max_seq) {
        leap::set_error("layer %d / pos %d out of range", layer, pos);
        return LEAP_ERR_INVALID;
    }
    DeviceGuard g(c->device);
    const size_t nq = size_t(c->n_heads) * c->hd, nk = size_t(c->n_kv) * c->hd;
    float *hq = c->h_stage, *hk = hq + nq, *hv = hk + nk, *ho = hv + nk;
    float *dq = c->d_stage, *dk = dq + nq, *dv = dk + nk;
    std::memcpy(hq, q, nq * sizeof(float));
    std::memcpy(hk, k_new, nk * sizeof(float));
    std::memcpy(hv, v_new, nk * sizeof(float));
    // q|k|v in by a copy kernel reading the mapped pinned buffer
    // (stage_host.cu), then the decode, chained by programmatic dependent
    // launch; the decode writes the output, and any error code, straight into
    // the mapped buffer.  One synchronization.
    float *hq_dev = c->h_stage_dev, *ho_dev = hq_dev + nq + 2 * nk;
    int *herr = reinterpret_cast<int *>(ho + nq);
    *reinterpret_cast<volatile int *>(herr) = 0;
    if (int st = leap::launch_stage_in(c->stream, hq_dev, dq, int((nq + 2 * nk) / 4))) return st;
    // the grid before the decode is stage_in, which writes no cache row: the
    // decode may start its K/V copies while it runs
    c->last_written_layer = leap_ctx::kWroteNone;
    leap::DecodeSeq tab;
    tab.n_seq = 1;
    tab.pos[0] = pos;
    tab.slot[0] = 0;
    c->err_host = reinterpret_cast<int *>(ho_dev + nq);
    const int st = leap::launch_decode(c, layer, tab, dq, dk, dv, ho_dev);
    c->err_host = nullptr;
    if (st) return st;
    LEAP_TRY_CUDA(cudaStreamSynchronize(c->stream), "cudaStreamSynchronize");
    if (*reinterpret_cast<volatile int *>(herr)) return leap::check_device_error(c);
    std::memcpy(out, ho, nq * sizeof(float));
    return LEAP_OK;
}

int leap_attn_decode_batched(leap_ctx *c, int layer, int n_seq, const int *slots,
                             const int *positions, const float *q, const float *k_new,
                             const float *v_new, float *out) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (int st = decode_check(c, layer, q, k_new, v_new, out)) return st;
    if (n_seq < 0 || (n_seq > 0 && (!slots || !positions))) {
        leap::set_error("bad n_seq / slots / positions");
        return LEAP_ERR_INVALID;
    }
    std::vector<char> seen(c->max_batch, 0);
    for (int i = 0; i < n_seq; ++i) {
        if (slots[i] < 0 || slots[i] >= c->max_batch || seen[slots[i]]) {
            leap::set_error("slot %d of sequence %d is out of range or repeated", slots[i], i);
            return LEAP_ERR_INVALID;
        }
        seen[slots[i]] = 1;
        if (positions[i] < 0 || positions[i] >= c->max_seq) {
            leap::set_error("position %d of sequence %d out of range", positions[i], i);
            return LEAP_ERR_INVALID;
        }
    }
    DeviceGuard g(c->device);
    const size_t nq = size_t(c->n_heads) * c->hd, nk = size_t(c->n_kv) * c->hd;
    for (int b0 = 0; b0 < n_seq; b0 += leap::kMaxSeqPerLaunch) {
        const int nb = (n_seq - b0) < leap::kMaxSeqPerLaunch ? (n_seq - b0) : leap::kMaxSeqPerLaunch;
        leap::DecodeSeq tab;
        tab.n_seq = nb;
        for (int i = 0; i < nb; ++i) {
            tab.pos[i] = positions[b0 + i];
            tab.slot[i] = slots[b0 + i];
        }
            if (int st = leap::launch_decode(c, layer, tab, q + b0 * nq, k_new + b0 * nk,
                                         v_new + b0 * nk, out + b0 * nq))
            return st;
    }
    return LEAP_OK;
}

int leap_attn_prefill(leap_ctx *c, int slot, int layer, int pos0, int n_tok, const float *q,
                      const float *k, const float *v, float *out) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (int st = decode_check(c, layer, q, k, v, out)) return st;
    if (slot < 0 || slot >= c->max_batch || pos0 < 0 || n_tok < 0 || pos0 + n_tok > c->max_seq) {
        leap::set_error("prefill range out of bounds: slot %d pos0 %d n_tok %d (max_seq %d)", slot,
                        pos0, n_tok, c->max_seq);
        return LEAP_ERR_INVALID;
    }
    if (n_tok == 0) return LEAP_OK;
    DeviceGuard g(c->device);
    const int st = leap::launch_prefill(c, slot, layer, pos0, n_tok, q, k, v, out);
    c->last_written_layer = layer;
    return st;
}

int leap_set_prefill_impl(leap_ctx *c, int impl) {
    leap::clear_error();
    LEAP_CHECK_CTX(c);
    if (impl < 0 || impl > 3) {
        leap::set_error("prefill impl %d unknown", impl);
        return LEAP_ERR_INVALID;
    }
    c->prefill_impl = impl;
    return LEAP_OK;
}

}  // extern "C"
