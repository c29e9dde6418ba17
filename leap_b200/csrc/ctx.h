// ctx.h — host-side definition of the opaque leap_ctx and shared helpers.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>

#include "leap_b200.h"

struct leap_ctx {
    // shape (reference Config fields, src/inference/Config.h:5-13)
    int device = 0;
    int n_layers = 0, layer0 = 0;
    int n_heads = 0, n_kv = 0, hd = 0, group = 0;
    int max_seq = 0, max_seq_pad = 0, max_batch = 0;
    int num_sms = 148;

    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;

    // KV cache [slot][layer][kv_head][max_seq_pad][hd] (floats)
    float *k_cache = nullptr, *v_cache = nullptr;
    size_t head_stride = 0, layer_stride = 0, slot_stride = 0;
    size_t cache_bytes = 0;  // per tensor (K or V)

    // RoPE table [max_seq][hd/2]
    float *rope_cos = nullptr, *rope_sin = nullptr;

    // split-KV scratch, two sets: consecutive decode launches alternate so
    // that a launch overlapping the previous one's tail never shares it
    float *part_o[2] = {nullptr, nullptr};      // [max_parts][group*hd]
    float *part_ml[2] = {nullptr, nullptr};     // [max_parts][2*max(group,2)]
    unsigned *counters[2] = {nullptr, nullptr}; // [kMaxSeqPerLaunch][n_kv]
    int max_parts = 0;
    int parity = 0;

    // Launch overlap (programmatic dependent launch): a decode kernel may
    // start streaming its layer's K/V while the previous kernel finishes,
    // unless the previous op of this context wrote that layer.
    int overlap = 1;
    int last_written_layer = kWroteAll;  // layer the previous op wrote
    static constexpr int kWroteAll = -2;
    static constexpr int kWroteNone = -1;  // the previous grid wrote no cache row

    // decode kernel choice: 0 auto, 1 split-KV (global combine),
    // 2 cluster (distributed-shared-memory combine)
    int decode_impl = 0;
    int cluster_capacity = 0;  // co-resident 16-CTA decode clusters

    // device error word (kernels report bounded-wait timeouts here)
    int *d_err = nullptr;
    // set only inside leap_attn_decode_host: the decode kernels also store an
    // error code to this host-mapped word (the caller waits on the host)
    int *err_host = nullptr;

    // host-pointer entry points: pinned staging and device mirrors
    float *h_stage = nullptr;  // pinned: q | k | v | out for one token
    float *h_stage_dev = nullptr;  // the same pinned buffer as device code addresses it
    float *d_stage = nullptr;

    // prefill scratch (rotated q), grown on demand
    float *d_qrot = nullptr;
    size_t qrot_cap = 0;  // floats
    int prefill_impl = 3;  // see leap_set_prefill_impl

    size_t device_bytes = 0;
};

namespace leap {

constexpr int kMaxDevices = 64;

// Device error word codes (bounded waits use small positive codes).
constexpr int kDevErrBadToken = 0x70;  // a device-side token id outside [0, vocab)

// thread-local last error
void set_error(const char *fmt, ...);
void clear_error();

// Convert a CUDA error into a LEAP status (sets the message).
int cuda_status(cudaError_t e, const char *what);

// Opt kernel `fn` into `bytes` of dynamic shared memory on the current
// device (and, with `nonportable_cluster`, into clusters above 8 CTAs).
// Done once per (kernel, device) under a lock, so launches from several host
// threads do not race.
int set_kernel_smem(const void *fn, size_t bytes, const char *what,
                    bool nonportable_cluster = false);

inline float *k_head_ptr(const leap_ctx *c, int slot, int layer, int kvh) {
    return c->k_cache + slot * c->slot_stride + layer * c->layer_stride +
           kvh * c->head_stride;
}
inline float *v_head_ptr(const leap_ctx *c, int slot, int layer, int kvh) {
    return c->v_cache + slot * c->slot_stride + layer * c->layer_stride +
           kvh * c->head_stride;
}

// ---- decode attention (decode_attn.cu) -----------------------------------
constexpr int kMaxSeqPerLaunch = 128;

struct DecodeSeq {
    int n_seq;
    int chunk;                         // rows per split
    int pos[kMaxSeqPerLaunch];
    int slot[kMaxSeqPerLaunch];
    int split0[kMaxSeqPerLaunch + 1];  // prefix sum of splits per sequence
};

// Launch one batch of decode work (n_seq <= kMaxSeqPerLaunch; only n_seq,
// pos and slot of `seqs` need to be set: the split plan is made here).
// q/k_new/v_new/out point at the first sequence of the batch.
int launch_decode(leap_ctx *c, int layer, const DecodeSeq &tab, const float *q,
                  const float *k_new, const float *v_new, float *out);

// Fill tab.chunk / tab.split0 for the given positions; returns total splits.
int plan_decode(const leap_ctx *c, DecodeSeq &tab, int shape);

// decode_cluster.cu: co-resident 16-CTA clusters, and the launch.
int decode_cluster_capacity(leap_ctx *c, int *n);
// Host-pointer staging kernel (stage_host.cu): n4 float4s pinned host ->
// device after everything before on the stream.
int launch_stage_in(cudaStream_t st, const float *h_src, float *d_dst, int n4);

int launch_decode_cluster(leap_ctx *c, int layer, const DecodeSeq &tab, const float *q,
                          const float *k_new, const float *v_new, float *out, bool overlap);

// Upper bound on split-KV partials one decode launch can need.
int max_decode_parts(int hd, int n_kv, int max_batch, int max_seq_pad, int num_sms);

// ---- prefill attention (prefill_attn.cu) ---------------------------------
int launch_prefill(leap_ctx *c, int slot, int layer, int pos0, int n_tok,
                   const float *q, const float *k, const float *v, float *out);

}  // namespace leap
