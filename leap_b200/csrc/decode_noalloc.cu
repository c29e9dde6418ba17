// decode_noalloc.cu — decode attention for callers that cannot allocate.
//
// Some callers cannot call cudaMalloc at all: code running under an
// allocator that owns every device byte (a framework's caching allocator, or
// a serving process that reserves all device memory as one arena at
// start-up and hands out slices of it), or an embedding whose host side is
// not allowed to touch CUDA's allocator.  leap_attn_decode_noalloc serves
// them: the caller passes its own K/V cache, RoPE table, inputs and output,
// and the only memory beyond those — the split-KV partials, the combine
// tickets and the kernel's error word — lives in the file-scope array below,
// which every GPU that loads this library holds until the process exits.
// Nothing here calls cudaMalloc or cudaFree.
//
// The kernel's copy waits are bounded (they give up after about two seconds,
// which a healthy GPU never reaches).  A wait that gives up is recorded in the
// array's error word, which no call reads back and the next call clears:
// this entry point cannot report it.  Callers that need that report use the
// context entry point leap_attn_decode, whose synchronising calls return it.
#include <mutex>

#include "common.cuh"
#include "ctx.h"

namespace leap {
namespace {

// 4 MiB of split-KV scratch per device: [tickets | error word | (M, L) | O].
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;
constexpr size_t kNoAllocHeader = 1024;  // tickets (<= 128 kv heads) + error word
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
unsigned char *g_scratch_addr[kMaxDevices] = {};

// Device address of the array on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is taken once
// per device with cudaGetSymbolAddress (this device current).
int scratch_address(int device, unsigned char **out) {
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_addr[device]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_status(e, "cudaGetSymbolAddress(noalloc scratch)");
        g_scratch_addr[device] = static_cast<unsigned char *>(p);
    }
    *out = g_scratch_addr[device];
    return LEAP_OK;
}

}  // namespace
}  // namespace leap

extern "C" int leap_attn_decode_noalloc(void *stream, int n_heads, int n_kv_heads, int head_dim,
                                        int pos, const float *rope_cos, const float *rope_sin,
                                        float *k_cache, float *v_cache, long long head_stride,
                                        const float *q, const float *k_new, const float *v_new,
                                        float *out) {
    using namespace leap;
    clear_error();
    if (n_heads < 1 || n_kv_heads < 1 || n_heads % n_kv_heads != 0 || n_kv_heads > 128) {
        set_error("noalloc decode: invalid heads %d / kv heads %d (kv heads <= 128)", n_heads,
                  n_kv_heads);
        return LEAP_ERR_INVALID;
    }
    const int group = n_heads / n_kv_heads;
    if ((head_dim != 64 && head_dim != 128) ||
        (group != 1 && group != 2 && group != 4 && group != 8)) {
        set_error("noalloc decode: unsupported head_dim %d / kv_mul %d", head_dim, group);
        return LEAP_ERR_INVALID;
    }
    // Far beyond what the scratch holds (about 64k positions); refused here so
    // that no int below can overflow.
    if (pos >= (1 << 24)) {
        set_error("noalloc decode: pos %d is beyond what the fixed scratch can hold", pos);
        return LEAP_ERR_INVALID;
    }
    if (pos < 0 || head_stride < ((long long)pos + 1) * head_dim || head_stride % 4 != 0) {
        set_error("noalloc decode: pos %d does not fit head_stride %lld (a multiple of 4 floats)",
                  pos, head_stride);
        return LEAP_ERR_INVALID;
    }
    const void *ptrs[] = {rope_cos, rope_sin, k_cache, v_cache, q, k_new, v_new, out};
    for (const void *p : ptrs) {
        if (!p || (reinterpret_cast<uintptr_t>(p) & 15u)) {
            set_error("noalloc decode: every pointer must be non-null and 16-byte aligned");
            return LEAP_ERR_INVALID;
        }
    }
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return cuda_status(e, "cudaGetDevice");
    if (device >= kMaxDevices) {
        set_error("noalloc decode: device %d out of range", device);
        return LEAP_ERR_INVALID;
    }
    unsigned char *scratch = nullptr;
    if (int st = scratch_address(device, &scratch)) return st;

    // A context shim on the stack describing the caller's memory, so the
    // regular split-KV launcher plans and launches the kernel unchanged.
    leap_ctx shim;
    shim.device = device;
    shim.n_layers = 1;
    shim.n_heads = n_heads;
    shim.n_kv = n_kv_heads;
    shim.hd = head_dim;
    shim.group = group;
    shim.max_seq = pos + 1;
    shim.max_batch = 1;
    e = cudaDeviceGetAttribute(&shim.num_sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_status(e, "cudaDeviceGetAttribute");
    shim.stream = static_cast<cudaStream_t>(stream);
    shim.k_cache = k_cache;
    shim.v_cache = v_cache;
    shim.head_stride = size_t(head_stride);
    shim.rope_cos = const_cast<float *>(rope_cos);
    shim.rope_sin = const_cast<float *>(rope_sin);
    const size_t mls = size_t(2) * (group < 2 ? 2 : group);
    const size_t part_bytes = (size_t(group) * head_dim + mls) * sizeof(float);
    shim.max_parts = int((kNoAllocScratchBytes - kNoAllocHeader) / part_bytes);
    unsigned *tickets = reinterpret_cast<unsigned *>(scratch);
    int *err = reinterpret_cast<int *>(scratch + kNoAllocHeader - 16);
    float *part_ml = reinterpret_cast<float *>(scratch + kNoAllocHeader);
    float *part_o = part_ml + size_t(shim.max_parts) * mls;
    for (int i = 0; i < 2; ++i) {
        shim.part_o[i] = part_o;
        shim.part_ml[i] = part_ml;
        shim.counters[i] = tickets;
    }
    shim.d_err = err;
    shim.overlap = 0;
    shim.decode_impl = 1;  // split-KV kernel, 128-thread CTAs

    DecodeSeq tab;
    tab.n_seq = 1;
    tab.pos[0] = pos;
    tab.slot[0] = 0;
    DecodeSeq planned = tab;
    const int total = plan_decode(&shim, planned, 0);  // the 128-thread shape
    if (long(total) * n_kv_heads > shim.max_parts) {
        set_error("noalloc decode: context %d needs %d split-KV partials, the %zu-byte scratch "
                  "holds %d",
                  pos + 1, total * n_kv_heads, kNoAllocScratchBytes, shim.max_parts);
        return LEAP_ERR_INVALID;
    }
    // Tickets and the error word must start at zero; the array keeps the
    // previous call's contents.
    e = cudaMemsetAsync(scratch, 0, kNoAllocHeader, shim.stream);
    if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync(noalloc tickets)");
    return launch_decode(&shim, 0, tab, q, k_new, v_new, out);
}
